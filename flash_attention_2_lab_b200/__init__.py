"""B200 (sm_100a) FlashAttention forward: drop-in for the production attention
forward of flash_attention_2_lab.

Public calls (all run the sm_100a kernel; there is no CPU or eager fallback):

* ``tensorcore_attention_forward_production_128x128(q, k, v, causal)`` --
  the reference's production entry point (csrc/bindings.cpp:136-140), same
  checks, messages and output contract.
* ``attention_forward(q, k, v, causal=False, scale=None)`` -- general form:
  any sequence length, different query/key lengths, optional scale.
* ``attention_forward_causal(q, k, v)`` -- the causal call.
* ``sharded`` -- (batch, head) sharding of one forward over several GPUs.
* ``attention(q, k, v, causal=False, scale=None)`` -- differentiable form
  (forward with log-sum-exp, backward kernel); see ``autograd``.
"""

from __future__ import annotations

from ._native import ext, lib
from .autograd import attention, attention_backward, attention_forward_lse

__all__ = [
    "attention",
    "attention_backward",
    "attention_forward",
    "attention_forward_lse",
    "attention_forward_causal",
    "tensorcore_attention_forward_production_128x128",
    "ext",
    "lib",
]


def tensorcore_attention_forward_production_128x128(query, key, value, causal):
    return ext().tensorcore_attention_forward_production_128x128(query, key, value, causal)


def attention_forward(query, key, value, causal: bool = False, scale: float | None = None):
    return ext().attention_forward(query, key, value, causal, scale)


def attention_forward_causal(query, key, value, scale: float | None = None):
    return ext().attention_forward(query, key, value, True, scale)
