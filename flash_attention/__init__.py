"""Forward calls of the ``flash_attention`` package on the B200 kernel.

The reference package (flash_attention/__init__.py:1-3) exports only its
FP32 oracle, ``attention_reference``; its production forward is reached
through the ``flash_attention_cuda`` extension with ``causal=False/True``
(csrc/bindings.cpp:136-140).  This package gives that forward its package
names, backed by the sm_100a kernel through the in-tree extension:

* ``attention_forward(query, key, value, causal=False, scale=None)``
* ``attention_forward_causal(query, key, value, scale=None)``

Same layout as the reference: fp16 CUDA tensors [B, H, N, 64], contiguous;
fp16 output of the same shape; default scale 1/sqrt(64).  There is no CPU
path: CPU tensors raise the reference's "query must be a CUDA tensor".
"""

from flash_attention_2_lab_b200 import attention_forward, attention_forward_causal

__all__ = ["attention_forward", "attention_forward_causal"]
