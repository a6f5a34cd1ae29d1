"""GPU tests of the logsumexp output and the backward pass.

No counterpart in the reference (its kernels are forward only).  The
reference for both is PyTorch autograd in FP32 on the same fp16 inputs,
restating flash_attention/reference.py:9-61 (scores * scale, top-left causal
mask, softmax, @ V).  Bounds: the log-sum-exp within 1e-3 absolute; the
forward output within the north-star bound; the gradients within
|err| <= 2e-2 * max|ref| + 2e-2 * |ref| + 1e-4 (the backward rounds P and dS
to fp16 before its products, as the forward rounds P; the absolute 1e-4 floor
covers gradients that are exactly zero, e.g. dK with a single key)."""

import pytest
import torch

from flash_attention_2_lab_b200 import _native
from parity_utils import ATOL, RTOL, read_status

pytestmark = pytest.mark.gpu


def lse_forward(q, k, v, causal, scale):
    lib = _native.lib()
    o = torch.empty_like(q)
    b, h, n, _ = q.shape
    lse = torch.empty(b, h, n, device=q.device, dtype=torch.float32)
    _native.check(lib.fa_fwd_sm100_lse(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                       lse.data_ptr(), b, h, n, k.shape[2], int(causal), scale,
                                       torch.cuda.current_stream().cuda_stream))
    return o, lse


def backward(q, k, v, o, do, lse, causal, scale):
    lib = _native.lib()
    dq, dk, dv = (torch.empty_like(t) for t in (q, k, v))
    b, h, n, _ = q.shape
    _native.check(lib.fa_bwd_sm100(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                   do.data_ptr(), lse.data_ptr(), dq.data_ptr(), dk.data_ptr(),
                                   dv.data_ptr(), b, h, n, int(causal), scale,
                                   torch.cuda.current_stream().cuda_stream))
    return dq, dk, dv


def reference(q, k, v, do, causal, scale):
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    s = torch.matmul(qf, kf.transpose(-1, -2)) * scale
    if causal:
        n, m = q.shape[2], k.shape[2]
        s = s.masked_fill(torch.ones(n, m, dtype=torch.bool, device=q.device).triu(1),
                          float("-inf"))
    lse = torch.logsumexp(s, -1)
    out = torch.softmax(s, -1) @ vf
    out.backward(do.float())
    return out.detach(), lse.detach(), qf.grad, kf.grad, vf.grad


def grad_close(got, ref, what):
    got = got.float()
    err = (got - ref).abs()
    bound = 2e-2 * ref.abs().max() + 2e-2 * ref.abs() + 1e-4
    assert torch.isfinite(got).all(), f"{what}: non-finite"
    worst = (err / bound).max().item()
    assert worst <= 1.0, f"{what}: max err {err.max().item():.3e}, worst err/bound {worst:.3f}"
    return worst


CASES = [(1, 2, 128), (1, 2, 256), (2, 3, 384), (1, 4, 1024), (1, 2, 200), (2, 2, 1000),
         (1, 2, 4096)]


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize(("b", "h", "n"), CASES)
def test_lse_and_backward_match_autograd(b, h, n, causal):
    g = torch.Generator(device="cuda").manual_seed(n * 3 + h)
    q, k, v, do = (torch.randn(b, h, n, 64, device="cuda", generator=g).half() for _ in range(4))
    scale = 0.125
    o, lse = lse_forward(q, k, v, causal, scale)
    dq, dk, dv = backward(q, k, v, o, do, lse, causal, scale)
    torch.cuda.synchronize()
    assert read_status() == 0
    o_ref, lse_ref, dq_ref, dk_ref, dv_ref = reference(q, k, v, do, causal, scale)
    assert ((o.float() - o_ref).abs() <= ATOL + RTOL * o_ref.abs()).all()
    assert (lse - lse_ref).abs().max().item() < 1e-3
    grad_close(dv, dv_ref, "dv")
    grad_close(dk, dk_ref, "dk")
    grad_close(dq, dq_ref, "dq")


def test_lse_forward_output_equals_plain_forward():
    g = torch.Generator(device="cuda").manual_seed(7)
    q, k, v = (torch.randn(2, 8, 2048, 64, device="cuda", generator=g).half() for _ in range(3))
    for causal in (False, True):
        o, _ = lse_forward(q, k, v, causal, 0.125)
        plain = torch.empty_like(q)
        _native.check(_native.lib().fa_fwd_sm100_varlen(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), plain.data_ptr(), 2, 8, 2048, 2048,
            int(causal), 0.125, torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        assert torch.equal(o, plain)


@pytest.mark.parametrize("causal", [False, True])
def test_autograd_function_matches_autograd_reference(causal):
    import flash_attention_2_lab_b200 as fa

    g = torch.Generator(device="cuda").manual_seed(11)
    q, k, v, do = (torch.randn(2, 4, 512, 64, device="cuda", generator=g).half()
                   for _ in range(4))
    qs, ks, vs = (t.clone().requires_grad_(True) for t in (q, k, v))
    out = fa.attention(qs, ks, vs, causal=causal)
    out.backward(do)
    o_ref, _, dq_ref, dk_ref, dv_ref = reference(q, k, v, do, causal, 0.125)
    assert ((out.detach().float() - o_ref).abs() <= ATOL + RTOL * o_ref.abs()).all()
    grad_close(qs.grad, dq_ref, "dq")
    grad_close(ks.grad, dk_ref, "dk")
    grad_close(vs.grad, dv_ref, "dv")


def backward_varlen(q, k, v, o, do, lse, causal, scale):
    lib = _native.lib()
    dq, dk, dv = (torch.empty_like(t) for t in (q, k, v))
    b, h, nq, _ = q.shape
    _native.check(lib.fa_bwd_sm100_varlen(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                          do.data_ptr(), lse.data_ptr(), dq.data_ptr(),
                                          dk.data_ptr(), dv.data_ptr(), b, h, nq, k.shape[2],
                                          int(causal), scale,
                                          torch.cuda.current_stream().cuda_stream))
    return dq, dk, dv


# (nq, nk): more keys than queries (causal: keys past the last query get no
# gradient, whole key tiles included), fewer keys, ragged both ways, one key.
VARLEN = [(128, 384), (384, 128), (200, 520), (1000, 300), (130, 1), (64, 700)]


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize(("nq", "nk"), VARLEN)
def test_backward_unequal_lengths_match_autograd(nq, nk, causal):
    g = torch.Generator(device="cuda").manual_seed(nq * 7 + nk)
    q, do = (torch.randn(2, 2, nq, 64, device="cuda", generator=g).half() for _ in range(2))
    k, v = (torch.randn(2, 2, nk, 64, device="cuda", generator=g).half() for _ in range(2))
    scale = 0.125
    o, lse = lse_forward(q, k, v, causal, scale)
    dq, dk, dv = backward_varlen(q, k, v, o, do, lse, causal, scale)
    torch.cuda.synchronize()
    assert read_status() == 0
    o_ref, lse_ref, dq_ref, dk_ref, dv_ref = reference(q, k, v, do, causal, scale)
    assert ((o.float() - o_ref).abs() <= ATOL + RTOL * o_ref.abs()).all()
    assert (lse - lse_ref).abs().max().item() < 1e-3
    grad_close(dv, dv_ref, "dv")
    grad_close(dk, dk_ref, "dk")
    grad_close(dq, dq_ref, "dq")
    if causal and nk > nq:
        assert not dk[:, :, nq:].any() and not dv[:, :, nq:].any()


def test_backward_without_queries_zeroes_key_gradients():
    k, v = (torch.randn(1, 2, 300, 64, device="cuda").half() for _ in range(2))
    q = torch.empty(1, 2, 0, 64, device="cuda", dtype=torch.float16)
    lse = torch.empty(1, 2, 0, device="cuda")
    dq, dk, dv = (torch.full_like(t, 7.0) for t in (q, k, v))
    _native.check(_native.lib().fa_bwd_sm100_varlen(
        q.data_ptr() or k.data_ptr(), k.data_ptr(), v.data_ptr(), q.data_ptr() or k.data_ptr(),
        q.data_ptr() or k.data_ptr(), lse.data_ptr() or k.data_ptr(),
        dq.data_ptr() or k.data_ptr(), dk.data_ptr(), dv.data_ptr(), 1, 2, 0, 300, 0, 0.125,
        torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert not dk.any() and not dv.any()


def test_autograd_function_unequal_lengths():
    import flash_attention_2_lab_b200 as fa

    g = torch.Generator(device="cuda").manual_seed(13)
    q, do = (torch.randn(1, 4, 300, 64, device="cuda", generator=g).half() for _ in range(2))
    k, v = (torch.randn(1, 4, 700, 64, device="cuda", generator=g).half() for _ in range(2))
    for causal in (False, True):
        qs, ks, vs = (t.clone().requires_grad_(True) for t in (q, k, v))
        out = fa.attention(qs, ks, vs, causal=causal)
        out.backward(do)
        o_ref, _, dq_ref, dk_ref, dv_ref = reference(q, k, v, do, causal, 0.125)
        assert ((out.detach().float() - o_ref).abs() <= ATOL + RTOL * o_ref.abs()).all()
        grad_close(qs.grad, dq_ref, "dq")
        grad_close(ks.grad, dk_ref, "dk")
        grad_close(vs.grad, dv_ref, "dv")


def test_training_binding_shape_checks():
    ext = _native.ext()
    q = torch.randn(1, 2, 128, 64, device="cuda").half()
    k = torch.randn(1, 2, 256, 64, device="cuda").half()
    o, lse = ext.attention_forward_lse(q, k, k, False, None)
    assert o.shape == q.shape and lse.shape == (1, 2, 128)
    with pytest.raises(RuntimeError, match="key must have shape"):
        ext.attention_forward_lse(q, torch.randn(2, 2, 256, 64, device="cuda").half(), k, False,
                                  None)
    with pytest.raises(RuntimeError, match="value must have the shape of key"):
        ext.attention_forward_lse(q, k, torch.randn(1, 2, 128, 64, device="cuda").half(), False,
                                  None)
    with pytest.raises(RuntimeError, match="grad_output must have the shape of query"):
        ext.attention_backward(q, k, k, o, torch.randn(1, 2, 256, 64, device="cuda").half(), lse,
                               False, None)
    with pytest.raises(RuntimeError, match="lse must be"):
        ext.attention_backward(q, k, k, o, o, lse[:, :, :64].contiguous(), False, None)
