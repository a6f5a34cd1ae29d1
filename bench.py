"""Benchmark of the sm_100a attention forward (one JSON line on rank 0).

Workload (the multi-GPU configuration, also the single-GPU headline):
attention forward B=32, H=32, N=8192, D=64, fp16, causal; the 32 batch
elements are split over the GPUs (strong scaling: total work fixed).  A step
is one forward over the rank's shard with the inputs resident in HBM.  Inputs
(3.2 GB) exceed the 126 MB L2, so no flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

For N > 1 launch one process per GPU with torch.distributed.run; the timed
region is bracketed by a barrier and a device synchronise on every rank and
the reported time is the maximum over ranks.

After the timed loop every rank checks its first and last (batch, head)
slices against an FP32 restatement on its GPU (the north-star bound
|out - ref| <= 2e-3 + 1e-2 |ref|); the verdicts are combined by a max over
ranks and printed as ``parity``.  At N = 1 the line also carries the other
BASELINE configurations, timed the way the reference's harness times them
(benchmarks/harness.py:34-71: warm-up, samples of back-to-back calls
between CUDA events, median): the short sweep C1/C2 (B1 H8 N 128..1024),
C3 (B4 H32 N8192) and the stress configuration C5 (B2 H16 N16384), each
causal and noncausal, with PyTorch SDPA on the same inputs as context.

``--impl reference`` times the reference's CPU path, ``attention_reference``
(flash_attention/reference.py:9-61, staged unmodified under baseline/_ref/),
on every host core, rank 0 only, one (batch, head) slice of the same
workload per step.
"""

from __future__ import annotations

import argparse
import csv
import io
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CFG = dict(batch=32, heads=32, seq_len=8192, head_dim=64, causal=True)
WORKLOAD = "attn-fwd C4: B32 H32 N8192 D64 fp16 causal, (b,h) sharded over GPUs"
METRIC = "attn-fwd TFLOPS (causal, B32 H32 N8192 D64)"
NVIDIA_DENSE_FP16_TFLOPS = 2250.0
PROFILE_TRAFFIC = ROOT / "profiles" / "fa_fwd_kernel_c4_causal_traffic.txt"
ATOL, RTOL = 2e-3, 1e-2  # north-star parity bound against the FP32 reference
SWEEP_N = (128, 256, 512, 1024)  # C1 / C2: B1 H8


def flops_of(batch, heads, n, causal, d=64):
    f = 4.0 * batch * heads * n * n * d
    return f / 2 if causal else f


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", 0)), "measured"
    return 1590.0, 1400.0, "fallback"


def traffic_per_launch(shard_batches):
    """DRAM bytes (read + write) of one kernel launch from the committed ncu
    summary, scaled from the captured case to this launch by (b, h) slices."""
    if not PROFILE_TRAFFIC.exists():
        return None
    vals = {}
    for line in PROFILE_TRAFFIC.read_text().splitlines():
        if ":" in line:
            key, _, val = line.partition(":")
            vals[key.strip()] = val.strip()
    try:
        bytes_ = float(vals["dram_bytes_per_launch"])
        units = float(vals["batch_heads_captured"])
    except (KeyError, ValueError):
        return None
    return bytes_ * (shard_batches * CFG["heads"]) / units


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu_index = gpu_index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu_index), "-lms", "100"],
                stdout=self.file, stderr=subprocess.DEVNULL)
            time.sleep(0.5)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.2)
        self.proc.terminate()
        self.proc.wait(timeout=5)
        self.file.flush()
        self.file.seek(0)
        rows = list(csv.reader(io.StringIO(self.file.read())))
        self.file.close()
        os.unlink(self.file.name)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
            except ValueError:
                continue
            for name, val in zip(names, r[5:9]):
                if val.strip().lower().startswith("active"):
                    reasons.add(name)
        loaded = [s for s in sm if s > 0.5 * max(sm)] if sm else []
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- helpers
def max_over_ranks_vec(values, dev):
    """Element-wise max of a list of floats over the ranks (identity at N=1)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return [float(v) for v in values]
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]


def sum_over_ranks(value, dev):
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def fp32_slice_reference(q, k, v, causal, scale):
    """softmax(q k^T scale [+ top-left causal mask]) v in FP32 on the GPU for
    one [N, 64] slice: the algorithm of flash_attention/reference.py:9-61."""
    import torch

    s = torch.matmul(q.float(), k.float().t()) * scale
    if causal:
        mask = torch.ones(q.shape[0], k.shape[0], dtype=torch.bool, device=q.device).triu(1)
        s.masked_fill_(mask, float("-inf"))
    return torch.softmax(s, -1) @ v.float()


def slice_parity(out, q, k, v, causal, scale, slices):
    """(max abs error, worst error / bound) over the given flattened (b, h)
    slices of one forward's output."""
    qf, kf, vf, of = (t.reshape(-1, t.shape[2], t.shape[3]) for t in (q, k, v, out))
    max_abs, worst = 0.0, 0.0
    for i in slices:
        ref = fp32_slice_reference(qf[i], kf[i], vf[i], causal, scale)
        err = (of[i].float() - ref).abs()
        max_abs = max(max_abs, float(err.max()))
        worst = max(worst, float((err / (ATOL + RTOL * ref.abs())).max()))
        if not bool(of[i].float().isfinite().all()):
            worst = float("inf")
    return max_abs, worst


def time_device(fn, steps, stream):
    import torch

    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end)


def harness_ms(fn, warmup=25, samples=20, iters=100):
    """Median per-call time (ms) by the reference harness's method
    (benchmarks/harness.py:34-71)."""
    import torch

    with torch.inference_mode():
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        out = []
        for _ in range(samples):
            start.record()
            for _ in range(iters):
                fn()
            end.record()
            end.synchronize()
            out.append(start.elapsed_time(end) / iters)
    return statistics.median(out)


def gpu_numa_node(local):
    """(NUMA node, CPU ids) nearest the GPU, from NVML's read-only queries
    (node -1 / no CPUs when the system does not say)."""
    import torch

    node, cpus = -1, []
    try:
        import pynvml

        pynvml.nvmlInit()
        try:
            bus = torch.cuda.get_device_properties(local)
            h = pynvml.nvmlDeviceGetHandleByPciBusId(
                f"{bus.pci_domain_id:08x}:{bus.pci_bus_id:02x}:{bus.pci_device_id:02x}.0")
            words = 4
            mask = pynvml.nvmlDeviceGetCpuAffinity(h, words)
            for w, bits in enumerate(mask):
                cpus += [w * 64 + b for b in range(64) if (int(bits) >> b) & 1]
            try:
                node = int(pynvml.nvmlDeviceGetNumaNodeId(h))
            except Exception:
                node = -1
        finally:
            pynvml.nvmlShutdown()
    except Exception:
        pass
    return node, cpus


def bind_to_cpus(cpus):
    """Run this process on ``cpus`` (the GPU's nearest) so its pinned host
    buffers are first touched, and placed, on that NUMA node."""
    if not cpus:
        return 0
    try:
        os.sched_setaffinity(0, set(cpus))
        return len(cpus)
    except (OSError, AttributeError):
        return 0


def host_link_ceiling(dev, world, local, d2h_share=1.0, nbytes=1 << 30, reps=3,
                      chunk_up=0, chunk_down=0, chunks=0):
    """Concurrent plain pinned copies on every rank at once: host->device,
    device->host, both directions with equal bytes, and both directions with
    the e2e step's own mix (``d2h_share`` bytes device->host per byte
    host->device).  With ``chunks`` > 0 also "pipe": the e2e step's copy
    schedule without its kernels (``chunks`` rounds of ``chunk_up`` bytes up
    on one stream and ``chunk_down`` bytes down on another).  Returns the
    whole-job GB/s of each (bytes of all ranks / the max-over-ranks time of
    the best repetition)."""
    import torch
    import torch.distributed as dist

    host = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    host2 = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    devb = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    devb2 = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    s1, s2 = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    mix_d2h = max(16, (int(nbytes * min(d2h_share, 1.0)) // 16) * 16)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local])

    def timed(kind):
        up = nbytes if kind in ("h2d", "both", "mix") else 0
        down = {"d2h": nbytes, "both": nbytes, "mix": mix_d2h}.get(kind, 0)
        times = []
        for _ in range(reps):
            barrier()
            t0 = time.perf_counter()
            if up:
                with torch.cuda.stream(s1):
                    devb[:up].copy_(host[:up], non_blocking=True)
            if down:
                with torch.cuda.stream(s2):
                    host2[:down].copy_(devb2[:down], non_blocking=True)
            s1.synchronize()
            s2.synchronize()
            times.append(max_over_ranks_vec([time.perf_counter() - t0], dev)[0])
        return (up + down) * world / min(times) / 1e9

    out = {k: round(timed(k), 2) for k in ("h2d", "d2h", "both", "mix")}
    if chunks > 0 and chunk_up <= nbytes and chunk_down <= nbytes:
        times = []
        for _ in range(reps):
            barrier()
            t0 = time.perf_counter()
            for _ in range(chunks):
                with torch.cuda.stream(s1):
                    devb[:chunk_up].copy_(host[:chunk_up], non_blocking=True)
                with torch.cuda.stream(s2):
                    host2[:chunk_down].copy_(devb2[:chunk_down], non_blocking=True)
            s1.synchronize()
            s2.synchronize()
            times.append(max_over_ranks_vec([time.perf_counter() - t0], dev)[0])
        out["pipe"] = round((chunk_up + chunk_down) * chunks * world / min(times) / 1e9, 2)
    del host, host2, devb, devb2
    return out


# ----------------------------------------------------------------- reference arm
def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return
    from flash_attention_2_lab_b200 import workloads
    from oracle import reference_cpu

    cfg = workloads.Config("c4", CFG["batch"], CFG["heads"], CFG["seq_len"])
    q, k, v = workloads.make_inputs(cfg, seed=0, batches=range(1))  # batch element 0
    scale = 1.0 / 8.0
    secs, done, kind, threads = reference_cpu.time_slices(
        q, k, v, True, scale, budget_s=0.0, max_slices=args.steps, min_slices=args.steps,
        warmup=args.warmup)
    ms = secs / done * 1e3
    tflops = flops_of(1, done, cfg.seq_len, True) / secs / 1e12
    sample = (f"{done} (b,h) slices of C4 (N=8192 causal, FP32 inputs), one per step, "
              f"after {args.warmup} untimed slices")
    api = ("flash_attention.reference.attention_reference (unmodified, staged under "
           "baseline/_ref)" if kind == "reference" else
           "numpy restatement oracle/attention_oracle.py (reference package not staged)")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tflops, 6), "unit": "TFLOPS",
        "n_gpus": world, "steps": done, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) fp16 inputs)",
        "config": {"workload": WORKLOAD, "sample": sample, "same_config": False,
                   "note": "CPU rate on a bounded sample of the C4 workload (TFLOPS "
                           "is size-independent per slice); the full workload would take "
                           "minutes"},
        "cpu_baseline": {"value": round(tflops, 6), "unit": "TFLOPS", "cores": threads,
                         "kind": kind, "sample": sample, "api": api},
        "e2e": {"value": round(tflops, 6), "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- our arm
def single_gpu_extras(dev, stream, fwd):
    """Other BASELINE configurations at N = 1 (timing keys, SDPA as context)."""
    import torch
    import torch.nn.functional as F

    from flash_attention_2_lab_b200 import workloads

    extra = {}
    # C1 / C2: B1 H8 N in 128..1024, through the drop-in binding, harness method
    sweep = {}
    for n in SWEEP_N:
        q, k, v = workloads.make_inputs(workloads.Config(f"c2_{n}", 1, 8, n), seed=0, device=dev)
        for c in (False, True):
            ms = harness_ms(lambda: fwd(q, k, v, c))
            sd = harness_ms(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=c))
            sweep[f"n{n}_{'causal' if c else 'noncausal'}"] = {
                "us": round(ms * 1e3, 2), "tflops": round(flops_of(1, 8, n, c) / ms / 1e9, 2),
                "sdpa_us": round(sd * 1e3, 2)}
    extra["c1_c2_sweep"] = sweep
    # C3 (B4 H32 N8192), both masks: the configuration of the 60 % target
    q3, k3, v3 = workloads.make_inputs("c3", seed=0, device=dev)
    for c in (False, True):
        for _ in range(3):
            fwd(q3, k3, v3, c)
        torch.cuda.synchronize()
        t = time_device(lambda: fwd(q3, k3, v3, c), 20, stream) / 20
        tf = flops_of(4, 32, 8192, c) / (t / 1e3) / 1e12
        extra["c3_causal" if c else "c3_noncausal"] = {"ms": round(t, 4), "tflops": round(tf, 1)}
    for c in (False, True):
        sdpa = lambda: F.scaled_dot_product_attention(q3, k3, v3, is_causal=c)  # noqa: E731
        for _ in range(3):
            sdpa()
        torch.cuda.synchronize()
        t = time_device(sdpa, 20, stream) / 20
        extra["sdpa_c3_causal" if c else "sdpa_c3_noncausal"] = {
            "ms": round(t, 4), "tflops": round(flops_of(4, 32, 8192, c) / (t / 1e3) / 1e12, 1),
            "note": "PyTorch SDPA (vendor kernel) on the same inputs, context only"}
    del q3, k3, v3
    # C5 stress (B2 H16 N16384, peaky logits and +-30 outlier keys), both masks,
    # with its parity on two slices
    q5, k5, v5 = workloads.make_inputs("c5", seed=0, device=dev)
    for c in (False, True):
        for _ in range(3):
            fwd(q5, k5, v5, c)
        torch.cuda.synchronize()
        t = time_device(lambda: fwd(q5, k5, v5, c), 10, stream) / 10
        out = fwd(q5, k5, v5, c)
        max_abs, worst = slice_parity(out, q5, k5, v5, c, 0.125, (0, 31))
        extra["c5_causal" if c else "c5_noncausal"] = {
            "ms": round(t, 4), "tflops": round(flops_of(2, 16, 16384, c) / (t / 1e3) / 1e12, 1),
            "parity": {"ok": worst <= 1.0, "max_abs": round(max_abs, 6),
                       "worst_err_over_bound": round(worst, 4), "slices": [0, 31]}}
    del q5, k5, v5
    # Backward (training) on C3, both masks: fa_bwd_sm100 on the saved (o, lse),
    # and SDPA's autograd on the same inputs as context; TFLOPS counts the
    # five GEMMs (2.5 x the forward's FLOPs).
    from flash_attention_2_lab_b200.autograd import attention_backward, attention_forward_lse

    q3, k3, v3 = workloads.make_inputs("c3", seed=0, device=dev)
    g = torch.Generator(device=dev).manual_seed(1)
    do = torch.randn(q3.shape, device=dev, generator=g).half()
    for c in (False, True):
        o, lse = attention_forward_lse(q3, k3, v3, c)
        bwd = lambda: attention_backward(q3, k3, v3, o, do, lse, c)  # noqa: E731
        for _ in range(2):
            bwd()
        torch.cuda.synchronize()
        t = time_device(bwd, 5, stream) / 5
        qs, ks, vs = (x.detach().requires_grad_(True) for x in (q3, k3, v3))
        out = F.scaled_dot_product_attention(qs, ks, vs, is_causal=c)
        sd = lambda: torch.autograd.grad(out, (qs, ks, vs), do, retain_graph=True)  # noqa: E731
        for _ in range(2):
            sd()
        torch.cuda.synchronize()
        ts = time_device(sd, 5, stream) / 5
        fl = 2.5 * flops_of(4, 32, 8192, c)
        extra["c3_backward_causal" if c else "c3_backward_noncausal"] = {
            "ms": round(t, 4), "tflops": round(fl / (t / 1e3) / 1e12, 1),
            "sdpa_ms": round(ts, 4), "sdpa_tflops": round(fl / (ts / 1e3) / 1e12, 1)}
        del o, lse, out, qs, ks, vs
    del q3, k3, v3, do
    return extra


def run_ours(args):
    import torch
    import torch.distributed as dist

    import flash_attention_2_lab_b200 as fa
    from flash_attention_2_lab_b200 import workloads
    from flash_attention_2_lab_b200.sharded import max_over_ranks, shard_range

    torch.backends.cuda.matmul.allow_tf32 = False
    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    numa, near_cpus = gpu_numa_node(local)
    all_cpus = os.sched_getaffinity(0)
    bound_cpus = bind_to_cpus(near_cpus)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    cfg = workloads.Config("c4", args.batch, CFG["heads"], CFG["seq_len"])
    mine = shard_range(cfg.batch, world, rank)
    q, k, v = workloads.make_inputs(cfg, seed=0, device=dev, batches=mine)
    causal = CFG["causal"]
    fwd = fa.tensorcore_attention_forward_production_128x128
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(args.warmup):
        fwd(q, k, v, causal)
    torch.cuda.synchronize()

    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    barrier()
    torch.cuda.synchronize()
    ms_local = time_device(lambda: fwd(q, k, v, causal), args.steps, stream) / args.steps
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop() if sampler else None
    ms = max_over_ranks(ms_local, dev)

    total_flops = flops_of(cfg.batch, cfg.heads, cfg.seq_len, causal)
    value = total_flops / (ms / 1e3) / 1e12
    local_flops = flops_of(len(mine), cfg.heads, cfg.seq_len, causal)
    achieved = local_flops / (ms_local / 1e3) / 1e12

    # ---- parity of this rank's shard (outside the timed region): first and
    # last (b, h) slice against the FP32 restatement, max over ranks
    out = fwd(q, k, v, causal)
    n_slices = len(mine) * cfg.heads
    checked = sorted({0, n_slices - 1}) if n_slices else []
    max_abs, worst = slice_parity(out, q, k, v, causal, 1.0 / 8.0, checked) if checked else (0, 0)
    del out
    max_abs, worst = max_over_ranks_vec([max_abs, worst], dev)
    parity = {"ok": worst <= 1.0, "max_abs": round(max_abs, 6),
              "worst_err_over_bound": round(worst, 4),
              "checked": f"first and last (b,h) slice of every rank's shard vs FP32 "
                         f"(bound {ATOL} + {RTOL}|ref|)"}

    if args.kernel_only:
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": round(value, 2), "unit": "TFLOPS",
                              "ms_per_step": round(ms, 4), "batch": cfg.batch,
                              "kernel_only": True, "clocks": clocks, "parity": parity}),
                  flush=True)
        if world > 1:
            dist.destroy_process_group()
        return

    # ---- end to end through the public host-input call (pinned host buffers;
    # chunks of one batch element stream H2D / kernel / D2H on three streams)
    from flash_attention_2_lab_b200.host_pipeline import attention_forward_host

    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hout = torch.empty(q.shape, dtype=q.dtype).pin_memory()

    def e2e_step():
        attention_forward_host(hq, hk, hv, causal, out=hout, device=dev, chunk_batches=1)

    e2e_steps = max(3, min(args.steps, 10))
    e2e_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e2e_ms_local = time_device(e2e_step, e2e_steps, stream) / e2e_steps
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e2e_ms_local, dev)
    e2e_value = total_flops / (e2e_ms / 1e3) / 1e12
    h2d = int(sum_over_ranks(sum(t.numel() * t.element_size() for t in (hq, hk, hv)), dev))
    d2h = int(sum_over_ranks(hout.numel() * hout.element_size(), dev))
    del hq, hk, hv, hout
    per_b = q[0].numel() * q.element_size()  # one batch element of one tensor
    link = host_link_ceiling(dev, world, local, d2h_share=d2h / max(h2d, 1),
                             chunk_up=3 * per_b, chunk_down=per_b, chunks=len(mine))
    e2e_gbs = (h2d + d2h) / (e2e_ms / 1e3) / 1e9
    # The host-link bound of one step: the copies alone at the concurrent
    # ceilings (each direction on its own, and both together), whichever is
    # slowest; the kernel itself is far shorter than any of them.
    link_ms = max(h2d / (link["h2d"] * 1e9), d2h / (link["d2h"] * 1e9),
                  (h2d + d2h) / (max(link["mix"], link.get("pipe", 0.0)) * 1e9)) * 1e3
    nodes = max_over_ranks_vec([numa], dev)  # all ranks' nodes agree here or the max shows one

    extra = {}
    cpu_baseline = None
    if rank == 0 and world == 1:
        extra = single_gpu_extras(dev, stream, fwd)
        from oracle import reference_cpu

        os.sched_setaffinity(0, all_cpus)  # the CPU baseline gets every host core
        secs, done, kind, threads = reference_cpu.time_slices(
            q.cpu(), k.cpu(), v.cpu(), causal, 1.0 / 8.0, budget_s=12.0, max_slices=64)
        cpu_tf = flops_of(1, done, cfg.seq_len, causal) / secs / 1e12
        cpu_baseline = {"value": round(cpu_tf, 6), "unit": "TFLOPS", "cores": threads,
                        "kind": kind,
                        "sample": f"{done} (b,h) slices of the C4 workload (N=8192 causal, "
                                  f"FP32 inputs), {secs:.1f} s on the host",
                        "api": "flash_attention.reference.attention_reference"
                               if kind == "reference" else "oracle numpy restatement"}

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    peak_burst, peak_sustained, peak_kind = measured_peaks()
    traffic = traffic_per_launch(len(mine))
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOPS", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded N(0,1) fp16 q, k, v generated on device per batch element)",
        "config": {"workload": WORKLOAD, "global_batch": cfg.batch, "heads": cfg.heads,
                   "seq_len": cfg.seq_len, "head_dim": 64, "causal": causal,
                   "parallelism": f"(b,h) shards x{world}, no collective",
                   "l2": "inputs 3.2 GB > 126 MB L2 (no flush needed)"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak_burst,
                     "unit": "TFLOP/s", "frac": round(achieved / peak_burst, 4),
                     "traffic": traffic,
                     "peak_kind": f"{peak_kind} cuBLAS bf16 burst",
                     "frac_of_nvidia_dense_fp16": round(achieved / NVIDIA_DENSE_FP16_TFLOPS, 4),
                     "frac_of_sustained": (round(achieved / peak_sustained, 4)
                                           if peak_sustained else None)},
        "parity": parity,
        "e2e": {"value": round(e2e_value, 2), "unit": "TFLOPS", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "api": "flash_attention_2_lab_b200.host_pipeline.attention_forward_host",
                "host_gbs": round(e2e_gbs, 2),
                "h2d_ceiling_gbs": link["h2d"], "d2h_ceiling_gbs": link["d2h"],
                "bidir_ceiling_gbs": link["both"], "mixed_ceiling_gbs": link["mix"],
                "pipeline_copy_ceiling_gbs": link.get("pipe"),
                "frac_of_bidir_ceiling": round(e2e_gbs / link["both"], 4),
                "link_bound_ms": round(link_ms, 3),
                "frac_of_link_bound": round(link_ms / e2e_ms, 4),
                "ceiling": "pinned copies on all ranks at once, max-over-ranks time: 1 GiB up / "
                           "down / both, the e2e byte mix, and the e2e copy schedule without "
                           "kernels (pipeline); the bound uses the faster of the last two",
                "numa_node": int(nodes[0]), "bound_cpus": bound_cpus},
        "gpu_launches": args.steps,
        "clocks": clocks,
    }
    if cpu_baseline:
        line["cpu_baseline"] = cpu_baseline
    line.update(extra)
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=CFG["batch"],
                    help="override the workload's batch (smaller cases for ncu captures)")
    ap.add_argument("--kernel-only", action="store_true",
                    help="time only the device loop (no e2e, extras or CPU baseline)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)  # timing rule: at least 3 untimed warm-up steps
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
