"""Differentiable attention on the sm_100a kernels, for training callers.

``attention(q, k, v, causal=False, scale=None)`` runs the forward that also
returns the row log-sum-exp (``fa_fwd_sm100_lse``) and, on backward, the
backward kernel (``fa_bwd_sm100_varlen``): dQ, dK, dV in fp16 from one pass
over the key tiles with P recomputed from the saved statistics.  q: contiguous
fp16 CUDA tensor [B, H, Nq, 64]; k, v: [B, H, Nk, 64] (Nk may differ from Nq;
the causal mask is top-left, key j hidden from query i < j, as in the
forward).

The reference has no backward (its kernels are forward only); this is the
training half of the same operator.
"""

from __future__ import annotations

import torch

from ._native import ext


class _AttentionSm100(torch.autograd.Function):
    @staticmethod
    def forward(ctx, query, key, value, causal, scale):
        output, lse = ext().attention_forward_lse(query, key, value, causal, scale)
        ctx.save_for_backward(query, key, value, output, lse)
        ctx.causal = causal
        ctx.scale = scale
        return output

    @staticmethod
    def backward(ctx, grad_output):
        query, key, value, output, lse = ctx.saved_tensors
        dq, dk, dv = ext().attention_backward(query, key, value, output,
                                              grad_output.contiguous(), lse, ctx.causal,
                                              ctx.scale)
        return dq, dk, dv, None, None


def attention(query, key, value, causal: bool = False, scale: float | None = None):
    """softmax(q k^T * scale [+ causal mask]) v with a backward pass."""
    return _AttentionSm100.apply(query, key, value, causal, scale)


def attention_forward_lse(query, key, value, causal: bool = False, scale: float | None = None):
    """(output, row log-sum-exp [B, H, Nq] fp32)."""
    return tuple(ext().attention_forward_lse(query, key, value, causal, scale))


def attention_backward(query, key, value, output, grad_output, lse, causal: bool = False,
                       scale: float | None = None):
    """(dq, dk, dv) for the output of attention_forward_lse."""
    return tuple(ext().attention_backward(query, key, value, output, grad_output, lse, causal,
                                          scale))
