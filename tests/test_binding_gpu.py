"""GPU tests of the torch extension boundary, mirroring the reference's
tests/test_tensorcore_attention.py:301-372 (production kernel vs SDPA, fp16,
rtol/atol 3e-2) plus its error contract and the legacy entry points."""

import pytest
import torch
import torch.nn.functional as F

import flash_attention_2_lab_b200 as fa
from flash_attention_2_lab_b200 import _native
from oracle.attention_oracle import attention_oracle
from parity_utils import assert_parity

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize(("batch", "heads", "sequence_length"),
                         [(1, 2, 128), (1, 4, 256), (1, 8, 512), (1, 8, 1024)])
def test_production_128x128_matches_sdpa(batch, heads, sequence_length, causal):
    torch.manual_seed(0)
    shape = (batch, heads, sequence_length, 64)
    query = torch.randn(shape, device="cuda", dtype=torch.float16).contiguous()
    key = torch.randn(shape, device="cuda", dtype=torch.float16).contiguous()
    value = torch.randn(shape, device="cuda", dtype=torch.float16).contiguous()
    expected = F.scaled_dot_product_attention(query, key, value, attn_mask=None, dropout_p=0.0,
                                              is_causal=causal)
    ext = _native.ext()
    actual = ext.tensorcore_attention_forward_production_128x128(query, key, value, causal)
    assert actual.shape == expected.shape
    assert actual.dtype == torch.float16
    assert actual.is_cuda
    torch.testing.assert_close(actual, expected, rtol=3e-2, atol=3e-2)
    # and the tighter bound against the FP32 oracle
    ref = attention_oracle(query.float().cpu().numpy(), key.float().cpu().numpy(),
                           value.float().cpu().numpy(), causal=causal)
    assert_parity(actual, ref)


# The reference's own shapes for its earlier entry points
# (tests/test_tensorcore_attention.py:15-24 for the Bc16 kernel, :81-90,
# :182-191 and :240-249 for the three Bc32 variants); all route to the sm_100a
# kernel here and are checked against SDPA at the reference's 3e-2 and against
# the FP32 oracle at the north-star bound.
BC16_SHAPES = [(1, 1, 16), (1, 2, 64), (1, 4, 80), (1, 8, 128), (2, 3, 256)]
BC32_SHAPES = [(1, 1, 32), (1, 2, 64), (1, 4, 96), (1, 8, 128), (1, 8, 512)]
BC32_NAMES = ["tensorcore_attention_forward_bc32", "tensorcore_attention_forward_bc32_raw_pv",
              "tensorcore_attention_forward_bc32_raw_qk_raw_pv"]
LEGACY_CASES = ([("tensorcore_attention_forward", *s) for s in BC16_SHAPES]
                + [(n, *s) for n in BC32_NAMES for s in BC32_SHAPES])


@pytest.mark.parametrize(("name", "batch", "heads", "n"), LEGACY_CASES)
def test_legacy_entry_points_match_sdpa_and_oracle(name, batch, heads, n):
    torch.manual_seed(n + heads)
    q, k, v = (torch.randn(batch, heads, n, 64, device="cuda", dtype=torch.float16)
               for _ in range(3))
    out = getattr(_native.ext(), name)(q, k, v)
    assert out.shape == q.shape and out.dtype == torch.float16
    exp = F.scaled_dot_product_attention(q, k, v)
    torch.testing.assert_close(out, exp, rtol=3e-2, atol=3e-2)
    ref = attention_oracle(q.float().cpu().numpy(), k.float().cpu().numpy(),
                           v.float().cpu().numpy(), causal=False)
    assert_parity(out, ref, what=f"{name} N={n}")


@pytest.mark.parametrize("name", BC32_NAMES)
def test_bc32_entry_points_reject_partial_key_tile(name):
    # reference tests/test_tensorcore_attention.py:155-179
    q = torch.randn(1, 1, 48, 64, device="cuda", dtype=torch.float16)
    with pytest.raises(RuntimeError, match="divisible by 32"):
        getattr(_native.ext(), name)(q, torch.randn_like(q), torch.randn_like(q))


def test_flash_attention_package_forward_calls():
    import flash_attention

    torch.manual_seed(3)
    q, k, v = (torch.randn(2, 4, 384, 64, device="cuda", dtype=torch.float16) for _ in range(3))
    for causal, fn in ((False, flash_attention.attention_forward),
                       (True, flash_attention.attention_forward_causal)):
        out = fn(q, k, v)
        ref = attention_oracle(q.float().cpu().numpy(), k.float().cpu().numpy(),
                               v.float().cpu().numpy(), causal=causal)
        assert_parity(out, ref, what=f"flash_attention causal={causal}")


def test_package_calls():
    torch.manual_seed(2)
    q = torch.randn(1, 2, 300, 64, device="cuda", dtype=torch.float16)
    k = torch.randn(1, 2, 500, 64, device="cuda", dtype=torch.float16)
    v = torch.randn(1, 2, 500, 64, device="cuda", dtype=torch.float16)
    for causal, fn in ((False, lambda: fa.attention_forward(q, k, v)),
                       (True, lambda: fa.attention_forward_causal(q, k, v))):
        ref = attention_oracle(q.float().cpu().numpy(), k.float().cpu().numpy(),
                               v.float().cpu().numpy(), causal=causal)
        assert_parity(fn(), ref)


def test_empty_input_returns_empty_output():
    q = torch.empty(0, 8, 128, 64, device="cuda", dtype=torch.float16)
    out = fa.tensorcore_attention_forward_production_128x128(q, q, q, True)
    assert out.shape == q.shape and out.dtype == torch.float16


def _qkv(shape=(1, 2, 128, 64), dtype=torch.float16):
    return [torch.randn(shape, device="cuda").to(dtype) for _ in range(3)]


@pytest.mark.parametrize(("mutate", "message"), [
    (lambda q, k, v: (q.float(), k, v), "query must have dtype torch.float16"),
    (lambda q, k, v: (q, k.float(), v), "key must have dtype torch.float16"),
    (lambda q, k, v: (q[0], k, v), r"query must have shape \[B, H, N, D\]"),
    (lambda q, k, v: (q, k[:, :1], v), "query and key must have identical shapes"),
    (lambda q, k, v: (q, k, v[:, :1]), "query and value must have identical shapes"),
    (lambda q, k, v: (q.transpose(2, 3).contiguous().transpose(2, 3), k, v),
     "query must be contiguous"),
    (lambda q, k, v: (q[..., :32].contiguous(), k[..., :32].contiguous(),
                      v[..., :32].contiguous()), "head dimension must equal 64"),
    (lambda q, k, v: (q[:, :, :96].contiguous(), k[:, :, :96].contiguous(),
                      v[:, :, :96].contiguous()), "sequence length must be divisible by 128"),
    (lambda q, k, v: (q, k.cpu(), v), "key must be a CUDA tensor"),
])
def test_production_input_errors(mutate, message):
    q, k, v = mutate(*_qkv())
    with pytest.raises(RuntimeError, match=message):
        fa.tensorcore_attention_forward_production_128x128(q, k, v, False)


def test_grid_limit_message_kept():
    q = torch.empty(1, 65536, 128, 64, device="cuda", dtype=torch.float16)
    with pytest.raises(RuntimeError, match="batch \\* heads exceeds CUDA grid.y limit"):
        fa.tensorcore_attention_forward_production_128x128(q, q, q, False)


def test_output_on_query_device_and_current_stream():
    q, k, v = _qkv((1, 4, 256, 64))
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        out = fa.tensorcore_attention_forward_production_128x128(q, k, v, True)
    s.synchronize()
    assert out.device == q.device
    exp = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    torch.testing.assert_close(out, exp, rtol=3e-2, atol=3e-2)
