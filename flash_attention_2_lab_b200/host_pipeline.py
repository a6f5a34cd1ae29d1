"""Attention forward for inputs that live in host memory.

``attention_forward_host`` streams the batch through the GPU in chunks of
batch elements on three CUDA streams -- host-to-device copies, the kernel, and
device-to-host copies -- so the PCIe transfers of one chunk overlap the
compute of another and the copies of the two directions overlap each other.
Device memory is a ring of a few chunk-sized slots, independent of the batch.

The inputs should be pinned (``tensor.pin_memory()``) for the copies to be
asynchronous; the output is returned in pinned host memory (or written to the
given ``out``).  The call returns after the last chunk has been copied back.
"""

from __future__ import annotations

import torch

from ._native import check, lib


def attention_forward_host(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                           causal: bool = False, scale: float | None = None,
                           out: torch.Tensor | None = None, device=None,
                           chunk_batches: int = 1, slots: int = 3) -> torch.Tensor:
    if query.is_cuda or key.is_cuda or value.is_cuda:
        raise ValueError("attention_forward_host expects host tensors")
    if query.dim() != 4 or key.dim() != 4 or value.dim() != 4:
        raise ValueError("query, key and value must have shape [B, H, N, D]")
    if chunk_batches < 1 or slots < 2:
        raise ValueError("chunk_batches must be >= 1 and slots >= 2")
    for name, t in (("query", query), ("key", key), ("value", value)):
        if t.dtype != torch.float16 or t.shape[-1] != 64 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous float16 tensor with head dimension 64")
    if (query.shape[:2] != key.shape[:2] or key.shape != value.shape):
        raise ValueError("query, key and value must agree in batch and heads; key and value "
                         "must have identical shapes")
    sc = scale if scale is not None else 1.0 / 8.0
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    b = query.shape[0]
    if out is None:
        out = torch.empty(query.shape, dtype=query.dtype, pin_memory=True)
    if b == 0:
        return out
    cb = min(chunk_batches, b)
    n_slots = min(slots, (b + cb - 1) // cb)
    with torch.cuda.device(dev):
        compute = torch.cuda.current_stream(dev)
        h2d = torch.cuda.Stream(dev)
        d2h = torch.cuda.Stream(dev)
        bufs = [tuple(torch.empty((cb, *t.shape[1:]), dtype=t.dtype, device=dev)
                      for t in (query, key, value, query)) for _ in range(n_slots)]
        freed = [None] * n_slots  # event: slot's previous output copied back
        for i, b0 in enumerate(range(0, b, cb)):
            b1 = min(b, b0 + cb)
            n = b1 - b0
            s = i % n_slots
            dq, dk, dv, do = (t[:n] for t in bufs[s])
            if freed[s] is not None:
                h2d.wait_event(freed[s])
            with torch.cuda.stream(h2d):
                dq.copy_(query[b0:b1], non_blocking=True)
                dk.copy_(key[b0:b1], non_blocking=True)
                dv.copy_(value[b0:b1], non_blocking=True)
                loaded = torch.cuda.Event()
                loaded.record(h2d)
            compute.wait_event(loaded)
            check(lib().fa_fwd_sm100_varlen(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                                            do.data_ptr(), n, query.shape[1], query.shape[2],
                                            key.shape[2], int(causal), sc,
                                            compute.cuda_stream))
            done = torch.cuda.Event()
            done.record(compute)
            d2h.wait_event(done)
            with torch.cuda.stream(d2h):
                out[b0:b1].copy_(do, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(d2h)
            freed[s] = ev
        d2h.synchronize()
    return out
