"""Seeded synthetic attention inputs for the benchmark configurations.

Mirrors the reference's ``benchmarks/workloads.py:56-89`` (seeded
``torch.randn`` for q, k, v in that order, fp16, [B, H, N, D]) with one
change: every batch element ``b`` draws from its own generator seeded with
``seed * 1_000_003 + b``.  The bytes of batch element ``b`` therefore do not
depend on how the batch is split over GPUs, so a 1-GPU run and an 8-GPU run
see identical inputs and any shard can be regenerated on its own device.

Configurations (all D = 64):

* ``c1``  B=1,  H=8,  N=1024
* ``c2``  B=1,  H=8,  N in {128, 256, 512, 1024}
* ``c3``  B=4,  H=32, N=8192
* ``c4``  B=32, H=32, N=8192, causal, sharded over GPUs along B
* ``c5``  B=2,  H=16, N=16384, stress: q, k ~ 8*N(0,1); v ~ N(0,1); in every
  (b, h) slice round(0.01*N) key rows (a seeded randperm) set to +-30 per
  element, sign drawn from the same generator; cast to fp16 after scaling.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

HEAD_DIM = 64


@dataclass(frozen=True)
class Config:
    name: str
    batch: int
    heads: int
    seq_len: int
    stress: bool = False


CONFIGS = {
    "c1": Config("c1", 1, 8, 1024),
    "c2_128": Config("c2_128", 1, 8, 128),
    "c2_256": Config("c2_256", 1, 8, 256),
    "c2_512": Config("c2_512", 1, 8, 512),
    "c2_1024": Config("c2_1024", 1, 8, 1024),
    "c3": Config("c3", 4, 32, 8192),
    "c4": Config("c4", 32, 32, 8192),
    "c5": Config("c5", 2, 16, 16384, stress=True),
}


def _gen(device, seed: int, b: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1_000_003 + b)
    return g


def _one_batch(cfg: Config, b: int, seed: int, device) -> tuple[torch.Tensor, ...]:
    shape = (cfg.heads, cfg.seq_len, HEAD_DIM)
    g = _gen(device, seed, b)
    if not cfg.stress:
        q = torch.randn(shape, generator=g, device=device, dtype=torch.float16)
        k = torch.randn(shape, generator=g, device=device, dtype=torch.float16)
        v = torch.randn(shape, generator=g, device=device, dtype=torch.float16)
        return q, k, v
    q = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * 8
    k = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * 8
    v = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    n_out = round(0.01 * cfg.seq_len)
    for h in range(cfg.heads):
        rows = torch.randperm(cfg.seq_len, generator=g, device=device)[:n_out]
        sign = torch.randint(0, 2, (n_out, HEAD_DIM), generator=g, device=device) * 2 - 1
        k[h, rows] = 30.0 * sign.to(torch.float32)
    return q.half(), k.half(), v.half()


def make_inputs(cfg: Config | str, seed: int = 0, device="cpu",
                batches: range | None = None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """q, k, v of shape [len(batches), H, N, 64] fp16 for the selected batch elements."""
    if isinstance(cfg, str):
        cfg = CONFIGS[cfg]
    batches = batches if batches is not None else range(cfg.batch)
    parts = [_one_batch(cfg, b, seed, device) for b in batches]
    if not parts:
        empty = torch.empty((0, cfg.heads, cfg.seq_len, HEAD_DIM), dtype=torch.float16,
                            device=device)
        return empty, empty.clone(), empty.clone()
    q, k, v = (torch.stack([p[i] for p in parts]).contiguous() for i in range(3))
    return q, k, v


def attention_flops(batch: int, heads: int, n_q: int, n_k: int, causal: bool,
                    d: int = HEAD_DIM) -> float:
    """The metric's algorithmic FLOPs: 4*B*H*Nq*Nk*D, halved for causal."""
    f = 4.0 * batch * heads * n_q * n_k * d
    return f / 2 if causal else f


def attention_bytes(batch: int, heads: int, n_q: int, n_k: int, d: int = HEAD_DIM) -> float:
    """Algorithmic HBM bytes: read q, k, v once and write o, fp16."""
    return 2.0 * batch * heads * d * (2 * n_q + 2 * n_k)
