"""Drop-in module name of the reference's extension (``import
flash_attention_cuda``, reference setup.py:5-33 / csrc/bindings.cpp:70).

Re-exports the in-tree sm_100a extension built by
``python -m flash_attention_2_lab_b200.build``; there is no fallback.
"""

from flash_attention_2_lab_b200._native import ext as _ext

_mod = _ext()
tensorcore_attention_forward_production_128x128 = _mod.tensorcore_attention_forward_production_128x128
tensorcore_attention_forward = _mod.tensorcore_attention_forward
tensorcore_attention_forward_bc32 = _mod.tensorcore_attention_forward_bc32
tensorcore_attention_forward_bc32_raw_pv = _mod.tensorcore_attention_forward_bc32_raw_pv
tensorcore_attention_forward_bc32_raw_qk_raw_pv = _mod.tensorcore_attention_forward_bc32_raw_qk_raw_pv
attention_forward = _mod.attention_forward
