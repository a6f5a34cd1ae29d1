"""The reference's own CPU path, timed on the host -- TEST / BASELINE
INFRASTRUCTURE ONLY (bench.py's ``cpu_baseline`` leg and ``--impl reference``).

Loads ``attention_reference`` (flash_attention/reference.py:9-61) from the
unmodified copy that ``oracle/build_ref.py`` stages under
``baseline/_ref/flash_attention/`` and calls it through its public signature
with FP32 inputs, one (batch, head) slice at a time (the reference
materialises the [B, H, N, N] FP32 scores, 256 MiB per slice at N=8192), with
every host core available to torch.  When the staged copy is absent the
numpy restatement in ``oracle/attention_oracle.py`` stands in and the result
says ``kind: "port"``.
"""

from __future__ import annotations

import importlib.util
import os
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
STAGED = ROOT / "baseline" / "_ref" / "flash_attention" / "reference.py"


def load_attention_reference():
    """``attention_reference`` of the staged reference package, or None."""
    if not STAGED.is_file():
        return None
    spec = importlib.util.spec_from_file_location("flash_attention_reference_cpu", STAGED)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.attention_reference


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def use_all_cores() -> int:
    """Give torch and the BLAS pools every core this process may run on
    (torchrun sets OMP_NUM_THREADS=1 in every rank)."""
    import torch

    n = host_cores()
    torch.set_num_threads(n)
    try:
        import threadpoolctl

        threadpoolctl.threadpool_limits(n)
    except Exception:  # pragma: no cover
        pass
    return n


def time_slices(q, k, v, causal: bool, scale: float, budget_s: float, max_slices: int,
                min_slices: int = 1, warmup: int = 1):
    """Time the reference CPU path on whole (batch, head) slices of q, k, v
    ([B, H, N, D] fp16 CPU tensors), spread evenly over the batch*heads (and
    wrapping around when more slices than exist are asked for), until at
    least ``min_slices`` slices and ``budget_s`` seconds of work, at most
    ``max_slices`` slices.  ``warmup`` untimed slices first.  Returns
    (seconds, slices, kind, threads)."""
    import torch

    threads = use_all_cores()
    fn = load_attention_reference()
    kind = "reference" if fn is not None else "port"
    qf = q.reshape(-1, 1, 1, q.shape[2], q.shape[3])
    kf = k.reshape(-1, 1, 1, k.shape[2], k.shape[3])
    vf = v.reshape(-1, 1, 1, v.shape[2], v.shape[3])
    total = qf.shape[0]
    stride = max(1, total // max(1, max_slices))
    if fn is None:
        from oracle.attention_oracle import attention_slice

        def run(i):
            attention_slice(qf[i, 0, 0].float().numpy(), kf[i, 0, 0].float().numpy(),
                            vf[i, 0, 0].float().numpy(), causal, scale)
    else:
        def run(i):
            with torch.inference_mode():
                fn(qf[i].float(), kf[i].float(), vf[i].float(), causal=causal, scale=scale)
    for w in range(warmup):
        run(w % total)
    done, secs = 0, 0.0
    while (done < min_slices or secs < budget_s) and done < max_slices:
        i = (done * stride) % total
        t0 = time.perf_counter()
        run(i)
        secs += time.perf_counter() - t0
        done += 1
    return secs, done, kind, threads
