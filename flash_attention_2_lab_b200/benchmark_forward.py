"""Command-line benchmark of the attention forward, flag-compatible with the
reference's ``python -m benchmarks.benchmark_forward`` (benchmarks/benchmark_forward.py:24-53)
and its timing method (benchmarks/harness.py:34-71: warm-up, then samples x
iterations between CUDA events, median / p10 / p90 per call).

Added columns: TFLOPS (4*B*H*Nq*Nk*D, halved for causal) and the fraction of
the measured B200 peak.  Added modes: ``--gpus N`` splits the (batch, head)
slices over N devices of this process and reports the slowest device's time;
``--sustained S`` runs each kernel (forward, or backward with ``--backward``)
back to back for S seconds while
nvidia-smi samples device 0's SM clock and power, and reports the sustained
TFLOPS with the median clock, the median power and TFLOPS per GHz (the
per-clock efficiency, which is what decides throughput once a long run sits
at the board's power limit).

    python -m flash_attention_2_lab_b200.benchmark_forward --batch 4 --heads 32 \\
        --query-length 8192 --causal --dtype float16 --kernels sm100 sdpa
"""

from __future__ import annotations

import argparse
import json
import statistics
import subprocess
import time
from pathlib import Path

import torch
import torch.nn.functional as F

from . import attention_forward
from .sharded import shard_range

DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}
ROOT = Path(__file__).resolve().parent.parent


def percentile(values, fraction):
    ordered = sorted(values)
    return ordered[round((len(ordered) - 1) * fraction)]


def measured_peak_tflops() -> float:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["bf16_tflops"])
    return 1590.0


def time_on_devices(ops, samples, iterations, warmup):
    """ops: list of (device, callable). Returns per-call ms samples, each the
    maximum over devices."""
    for dev, op in ops:
        with torch.cuda.device(dev):
            for _ in range(warmup):
                op()
    for dev, _ in ops:
        torch.cuda.synchronize(dev)
    out = []
    for _ in range(samples):
        events = []
        for dev, op in ops:
            with torch.cuda.device(dev):
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                for _ in range(iterations):
                    op()
                e.record()
                events.append((s, e))
        for s, e in events:
            e.synchronize()
        out.append(max(s.elapsed_time(e) for s, e in events) / iterations)
    return out


def sustained(ops, seconds):
    """Back-to-back calls for ``seconds`` with nvidia-smi sampling of device 0.
    Returns (ms per call, median SM MHz under load, median W, reasons seen)."""
    for dev, op in ops:
        with torch.cuda.device(dev):
            for _ in range(5):
                op()
    torch.cuda.synchronize()
    try:
        smi = subprocess.Popen(["nvidia-smi", "-i", "0", "--query-gpu=clocks.sm,power.draw,"
                                "clocks_event_reasons.active", "--format=csv,noheader,nounits",
                                "-lms", "100"], stdout=subprocess.PIPE, text=True)
    except OSError:
        smi = None
    time.sleep(0.3)
    calls = 0
    start = time.perf_counter()
    while time.perf_counter() - start < seconds:
        for _ in range(10):
            for dev, op in ops:
                with torch.cuda.device(dev):
                    op()
        calls += 10
        torch.cuda.synchronize()
    elapsed = time.perf_counter() - start
    mhz, watts, reasons = [], [], set()
    if smi is not None:
        smi.terminate()
        for row in smi.communicate()[0].strip().splitlines():
            parts = [x.strip() for x in row.split(",")]
            if len(parts) != 3:
                continue
            try:
                mhz.append(float(parts[0]))
                watts.append(float(parts[1]))
            except ValueError:
                continue
            reasons.add(parts[2])
    loaded = [m for m in mhz if m > 0.5 * max(mhz)] if mhz else []
    return (elapsed * 1e3 / calls, statistics.median(loaded) if loaded else None,
            statistics.median(watts) if watts else None, sorted(reasons))


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--heads", type=int, default=8)
    ap.add_argument("--query-length", type=int, default=512)
    ap.add_argument("--key-length", type=int, default=None)
    ap.add_argument("--head-dim", type=int, default=64)
    ap.add_argument("--causal", action="store_true")
    ap.add_argument("--dtype", choices=list(DTYPES), default="float16")
    ap.add_argument("--samples", type=int, default=20)
    ap.add_argument("--iterations", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=25)
    ap.add_argument("--kernels", nargs="+", default=None,
                    help="kernel names: sm100 (this library), sdpa (PyTorch, for context)")
    ap.add_argument("--gpus", type=int, default=1, help="devices to split (b, h) over")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--backward", action="store_true",
                    help="time the backward pass (sm100: fa_bwd_sm100 on saved (o, lse); sdpa: "
                         "autograd of its forward); TFLOPS = 2.5 x the forward's FLOPs")
    ap.add_argument("--sustained", type=float, default=0.0,
                    help="seconds of back-to-back calls per kernel with clock/power sampling")
    args = ap.parse_args(argv)

    nk = args.key_length if args.key_length is not None else args.query_length
    dtype = DTYPES[args.dtype]
    kernels = args.kernels or ["sm100", "sdpa"]
    g = torch.Generator(device="cuda").manual_seed(args.seed)
    q = torch.randn(args.batch, args.heads, args.query_length, args.head_dim, device="cuda",
                    dtype=dtype, generator=g)
    k = torch.randn(args.batch, args.heads, nk, args.head_dim, device="cuda", dtype=dtype,
                    generator=g)
    v = torch.randn(args.batch, args.heads, nk, args.head_dim, device="cuda", dtype=dtype,
                    generator=g)
    flops = 4.0 * args.batch * args.heads * args.query_length * nk * args.head_dim
    if args.causal:
        flops /= 2
    peak = measured_peak_tflops()

    shards = []
    for r in range(args.gpus):
        rng = shard_range(args.batch * args.heads, args.gpus, r)
        dev = torch.device("cuda", r)
        sl = slice(rng.start, rng.stop)
        shards.append((dev, *(t.reshape(-1, 1, *t.shape[2:])[sl].transpose(0, 1)
                              .contiguous().to(dev) for t in (q, k, v))))

    print(f"workload: B={args.batch} H={args.heads} Nq={args.query_length} Nk={nk} "
          f"D={args.head_dim} causal={args.causal} dtype={args.dtype} gpus={args.gpus}")
    print(f"{'kernel':10s} {'median ms':>10s} {'p10 ms':>9s} {'p90 ms':>9s} {'TFLOPS':>9s} "
          f"{'% peak':>7s}")
    results = {}
    if args.backward:
        flops *= 2.5  # five GEMMs of the forward's size instead of two
    for name in kernels:
        if name == "sm100" and args.backward:
            supported = dtype == torch.float16 and args.head_dim == 64 and nk == args.query_length

            def mk(dq, dk, dv):
                from .autograd import attention_backward, attention_forward_lse

                o, lse = attention_forward_lse(dq, dk, dv, args.causal)
                do = torch.randn_like(o)
                return lambda: attention_backward(dq, dk, dv, o, do, lse, args.causal)
        elif name == "sdpa" and args.backward:
            supported = True

            def mk(dq, dk, dv):
                qq, kk, vv = (t.detach().requires_grad_(True) for t in (dq, dk, dv))
                out = F.scaled_dot_product_attention(qq, kk, vv, is_causal=args.causal)
                do = torch.randn_like(out)
                return lambda: torch.autograd.grad(out, (qq, kk, vv), do, retain_graph=True)
        elif name == "sm100":
            supported = dtype == torch.float16 and args.head_dim == 64
            mk = lambda dq, dk, dv: (lambda: attention_forward(dq, dk, dv, args.causal))
        elif name == "sdpa":
            supported = True
            mk = lambda dq, dk, dv: (lambda: F.scaled_dot_product_attention(
                dq, dk, dv, is_causal=args.causal))
        else:
            raise SystemExit(f"unknown kernel {name!r} (choose from sm100, sdpa)")
        if not supported:
            print(f"{name:10s} unsupported for this dtype / head dimension")
            continue
        ops = [(dev, mk(dq, dk, dv)) for dev, dq, dk, dv in shards]
        if args.backward and args.sustained > 0:
            # autograd needs grad mode: no inference_mode here
            ms, mhz, watts, reasons = sustained(ops, args.sustained)
            tf = flops / (ms / 1e3) / 1e12
            per_ghz = tf / (mhz / 1e3) if mhz else float("nan")
            print(f"{name:10s} sustained {args.sustained:.0f} s (backward): {ms:.4f} ms/call, "
                  f"{tf:.1f} TFLOPS, SM {mhz} MHz (median), {watts} W (median), "
                  f"{per_ghz:.1f} TFLOPS/GHz, clock event reasons {reasons}")
            continue
        if args.backward:
            # autograd needs grad mode; time the ops outside inference_mode
            ms = time_on_devices(ops, args.samples, args.iterations, args.warmup)
            med = statistics.median(ms)
            tf = flops / (med / 1e3) / 1e12
            results[name] = med
            print(f"{name:10s} {med:10.4f} {percentile(ms, 0.1):9.4f} "
                  f"{percentile(ms, 0.9):9.4f} {tf:9.1f} {100 * tf / (peak * args.gpus):6.1f}%  "
                  f"(backward)")
            continue
        if args.sustained > 0:
            with torch.inference_mode():
                ms, mhz, watts, reasons = sustained(ops, args.sustained)
            tf = flops / (ms / 1e3) / 1e12
            per_ghz = tf / (mhz / 1e3) if mhz else float("nan")
            print(f"{name:10s} sustained {args.sustained:.0f} s: {ms:.4f} ms/call, {tf:.1f} TFLOPS, "
                  f"SM {mhz} MHz (median), {watts} W (median), {per_ghz:.1f} TFLOPS/GHz, "
                  f"clock event reasons {reasons}")
            continue
        with torch.inference_mode():
            ms = time_on_devices(ops, args.samples, args.iterations, args.warmup)
        med = statistics.median(ms)
        tf = flops / (med / 1e3) / 1e12
        results[name] = med
        print(f"{name:10s} {med:10.4f} {percentile(ms, 0.1):9.4f} {percentile(ms, 0.9):9.4f} "
              f"{tf:9.1f} {100 * tf / (peak * args.gpus):6.1f}%")
    if "sm100" in results and "sdpa" in results:
        print(f"sdpa / sm100 time ratio: {results['sdpa'] / results['sm100']:.2f}x")


if __name__ == "__main__":
    main()
