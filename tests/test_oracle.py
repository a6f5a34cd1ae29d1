"""CPU tests of the numpy oracle: pinned to the reference's own output
(golden fixtures from flash_attention/reference.py) and to PyTorch SDPA in
FP32, mirroring the reference's tests/test_reference.py."""

import math
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle.attention_oracle import attention_oracle, flops

GOLDEN = Path(__file__).resolve().parent / "golden" / "attention_golden.npz"


def golden_cases():
    data = np.load(GOLDEN)
    names = sorted({k.split("/")[0] for k in data.files})
    return data, names


def test_golden_file_present():
    _, names = golden_cases()
    assert len(names) >= 15


@pytest.mark.parametrize("name", golden_cases()[1])
def test_oracle_matches_reference_golden(name):
    data, _ = golden_cases()
    q, k, v = (data[f"{name}/{t}"] for t in "qkv")
    meta = data[f"{name}/meta"]
    causal = bool(meta[5])
    scale = None if meta[6] < 0 else float(meta[6])
    out = attention_oracle(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32),
                           causal=causal, scale=scale)
    ref = data[f"{name}/out"]
    assert out.shape == ref.shape
    np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-5)


# reference tests/test_reference.py:10-52
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize(("batch", "heads", "sequence", "head_dimension"),
                         [(1, 1, 1, 16), (1, 2, 17, 32), (2, 4, 64, 64), (1, 8, 65, 128)])
def test_oracle_matches_sdpa(batch, heads, sequence, head_dimension, causal):
    torch.manual_seed(0)
    q = torch.randn(batch, heads, sequence, head_dimension)
    k = torch.randn(batch, heads, sequence, head_dimension)
    v = torch.randn(batch, heads, sequence, head_dimension)
    out = attention_oracle(q.numpy(), k.numpy(), v.numpy(), causal=causal)
    exp = F.scaled_dot_product_attention(q, k, v, is_causal=causal)
    np.testing.assert_allclose(out, exp.numpy(), rtol=1e-5, atol=1e-5)


# reference tests/test_reference.py:55-64
def test_oracle_supports_different_query_and_key_lengths():
    torch.manual_seed(0)
    q = torch.randn(2, 4, 7, 32)
    k = torch.randn(2, 4, 11, 32)
    v = torch.randn(2, 4, 11, 32)
    out = attention_oracle(q.numpy(), k.numpy(), v.numpy())
    exp = F.scaled_dot_product_attention(q, k, v)
    assert out.shape == (2, 4, 7, 32)
    np.testing.assert_allclose(out, exp.numpy(), rtol=1e-5, atol=1e-5)


# reference tests/test_reference.py:67-103
def test_oracle_custom_and_default_scale():
    torch.manual_seed(0)
    q, k, v = (torch.randn(1, 2, 9, 16) for _ in range(3))
    out = attention_oracle(q.numpy(), k.numpy(), v.numpy(), scale=0.3)
    exp = F.scaled_dot_product_attention(q, k, v, scale=0.3)
    np.testing.assert_allclose(out, exp.numpy(), rtol=1e-5, atol=1e-5)
    out_d = attention_oracle(q.numpy(), k.numpy(), v.numpy())
    out_e = attention_oracle(q.numpy(), k.numpy(), v.numpy(), scale=1 / math.sqrt(16))
    np.testing.assert_array_equal(out_d, out_e)


def test_oracle_block_rows_do_not_change_result():
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((1, 1, 300, 64)).astype(np.float32) for _ in range(3))
    a = attention_oracle(q, k, v, causal=True, block_rows=1024)
    b = attention_oracle(q, k, v, causal=True, block_rows=37)
    np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-6)


def test_oracle_causal_with_fewer_keys_than_queries():
    torch.manual_seed(3)
    q = torch.randn(1, 2, 9, 16)
    k = torch.randn(1, 2, 4, 16)
    v = torch.randn(1, 2, 4, 16)
    mask = torch.ones(9, 4, dtype=torch.bool).triu(1)
    exp = F.scaled_dot_product_attention(q, k, v, attn_mask=~mask)
    out = attention_oracle(q.numpy(), k.numpy(), v.numpy(), causal=True)
    np.testing.assert_allclose(out, exp.numpy(), rtol=1e-5, atol=1e-5)


def test_oracle_heads_subset():
    rng = np.random.default_rng(1)
    q, k, v = (rng.standard_normal((2, 3, 40, 64)).astype(np.float32) for _ in range(3))
    full = attention_oracle(q, k, v, causal=True)
    part = attention_oracle(q, k, v, causal=True, heads=slice(2, 5))
    np.testing.assert_array_equal(part, full.reshape(6, 40, 64)[2:5])


# reference tests/test_reference.py:106-121
def test_oracle_rejects_bad_rank():
    x = np.zeros((2, 3, 4), np.float32)
    with pytest.raises(ValueError, match="must have shape"):
        attention_oracle(x, x, x)


def test_oracle_rejects_mismatched_kv_length():
    q = np.zeros((1, 1, 4, 8), np.float32)
    k = np.zeros((1, 1, 5, 8), np.float32)
    v = np.zeros((1, 1, 6, 8), np.float32)
    with pytest.raises(ValueError, match="same sequence length"):
        attention_oracle(q, k, v)


def test_oracle_rejects_integer_dtype():
    x = np.zeros((1, 1, 4, 8), np.int32)
    with pytest.raises(TypeError, match="floating-point"):
        attention_oracle(x, x, x)


def test_flops_formula():
    assert flops(4, 32, 8192, 8192, 64, False) == pytest.approx(2.199e12, rel=1e-3)
    assert flops(4, 32, 8192, 8192, 64, True) == pytest.approx(1.0995e12, rel=1e-3)
