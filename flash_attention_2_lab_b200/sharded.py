"""(batch, head) sharding of one attention forward over the GPUs of a node.

The (b, h) slices of attention are independent, so the forward shards with
no collective on the data path: every GPU runs the kernel on its own
contiguous block of batch elements.  The reference has no multi-GPU code;
this is the launcher the multi-GPU configuration asks for.

Two ways to use it:

* one process driving several devices -- ``attention_forward_sharded``
  (copies each shard to its device, launches on each device's current
  stream, optionally gathers the result);
* one process per GPU (torchrun) -- every rank takes ``shard_range`` of the
  batch and reduces its timing with ``max_over_ranks``; no data moves
  between ranks.
"""

from __future__ import annotations

from typing import Sequence

import torch


def shard_range(total: int, world: int, rank: int) -> range:
    """Contiguous, balanced split of ``range(total)``: the first ``total % world``
    ranks get one extra element."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def split_dim(total_b: int, total_h: int, world: int) -> str:
    """Shard along the batch axis when every rank gets at least one batch
    element (each shard is then a contiguous slice), otherwise along the
    flattened batch*head axis."""
    return "batch" if total_b >= world else "batch_head"


def attention_forward_sharded(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                              causal: bool = False, devices: Sequence[int | str] | None = None,
                              gather_to: int | str | None = None, scale: float | None = None):
    """Run one forward split over ``devices``.

    Inputs may live on any device (or the host); each shard is copied to its
    device.  Returns the list of per-device outputs, or, with ``gather_to``,
    one tensor on that device (peer copies over NVLink between GPUs).
    """
    from . import attention_forward

    if devices is None:
        devices = list(range(torch.cuda.device_count()))
    devs = [torch.device("cuda", d) if isinstance(d, int) else torch.device(d) for d in devices]
    if not devs:
        raise RuntimeError("no CUDA devices to shard over")
    b, h = query.shape[0], query.shape[1]
    flat = split_dim(b, h, len(devs)) == "batch_head"
    if flat:
        query = query.reshape(1, b * h, *query.shape[2:])
        key = key.reshape(1, b * h, *key.shape[2:])
        value = value.reshape(1, b * h, *value.shape[2:])
    axis = 1 if flat else 0
    total = query.shape[axis]
    outs = []
    for rank, dev in enumerate(devs):
        r = shard_range(total, len(devs), rank)
        if len(r) == 0:
            continue
        sl = [slice(None)] * 4
        sl[axis] = slice(r.start, r.stop)
        qs, ks, vs = (t[tuple(sl)].to(dev, non_blocking=True).contiguous()
                      for t in (query, key, value))
        with torch.cuda.device(dev):
            outs.append(attention_forward(qs, ks, vs, causal, scale))
    if gather_to is None:
        return outs
    tgt = torch.device("cuda", gather_to) if isinstance(gather_to, int) else torch.device(gather_to)
    out = torch.cat([o.to(tgt, non_blocking=True) for o in outs], dim=axis)
    if flat:
        out = out.reshape(b, h, *out.shape[2:])
    return out


def max_over_ranks(value: float, device: torch.device | str | None = None) -> float:
    """Max of a per-rank float over the default process group (identity when
    torch.distributed is not initialised)."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64,
                     device=device if device is not None else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
