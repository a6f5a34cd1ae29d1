"""CPU tests of the ``flash_attention`` package names: the noncausal and
causal forward calls exist, route to the sm_100a extension (no CPU fallback:
CPU tensors raise the reference's message), and do not import the oracle."""

import importlib
import sys

import pytest
import torch


def test_package_exports_forward_calls():
    fa = importlib.import_module("flash_attention")
    assert callable(fa.attention_forward)
    assert callable(fa.attention_forward_causal)
    assert set(fa.__all__) == {"attention_forward", "attention_forward_causal"}


def test_package_forward_has_no_cpu_path():
    import flash_attention

    x = torch.zeros(1, 1, 128, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="query must be a CUDA tensor"):
        flash_attention.attention_forward(x, x, x)
    with pytest.raises(RuntimeError, match="query must be a CUDA tensor"):
        flash_attention.attention_forward_causal(x, x, x)


def test_package_does_not_load_the_oracle():
    for name in [m for m in sys.modules if m.startswith("oracle")]:
        del sys.modules[name]
    sys.modules.pop("flash_attention", None)
    importlib.import_module("flash_attention")
    assert not any(m.startswith("oracle") for m in sys.modules)
