"""Shared helpers of the GPU parity tests: C-ABI calls on torch-owned device
memory, the parity bound, and a GPU fp32 restatement for full-size checks."""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from flash_attention_2_lab_b200 import _native

# North-star tolerance against the FP32 reference: |out - ref| <= ATOL + RTOL*|ref|
ATOL = 2e-3
RTOL = 1e-2


def abi_forward(q, k, v, causal, scale=None, out=None, stream=None):
    """Call fa_fwd_sm100_varlen through the C ABI; returns the output tensor."""
    lib = _native.lib()
    if out is None:
        out = torch.empty_like(q)
    b, h, nq, d = q.shape
    nk = k.shape[2]
    sc = scale if scale is not None else 1.0 / d ** 0.5
    st = (stream or torch.cuda.current_stream()).cuda_stream
    rc = lib.fa_fwd_sm100_varlen(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                 b, h, nq, nk, int(causal), sc, st)
    _native.check(rc)
    return out


def read_status(clear=True) -> int:
    v = ctypes.c_uint(0)
    _native.check(_native.lib().fa_read_status(torch.cuda.current_stream().cuda_stream,
                                               ctypes.byref(v), int(clear)))
    return v.value


def parity_report(out: np.ndarray, ref: np.ndarray, atol=ATOL, rtol=RTOL):
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(out - ref)
    bound = atol + rtol * np.abs(ref)
    return float(err.max(initial=0.0)), float((err / bound).max(initial=0.0))


def assert_parity(out, ref, atol=ATOL, rtol=RTOL, what=""):
    if isinstance(out, torch.Tensor):
        out = out.detach().float().cpu().numpy()
    if isinstance(ref, torch.Tensor):
        ref = ref.detach().float().cpu().numpy()
    assert out.shape == ref.shape, (out.shape, ref.shape)
    assert np.isfinite(out).all(), f"{what}: non-finite output"
    max_abs, worst = parity_report(out, ref, atol, rtol)
    assert worst <= 1.0, f"{what}: max abs err {max_abs:.3e}, worst err/bound {worst:.3f}"
    return max_abs


def torch_fp32_reference(q, k, v, causal, scale=None, heads_per_chunk=4):
    """FP32 attention on the GPU, chunked over (batch*head) slices; the same
    math as the oracle, used where the CPU would take minutes."""
    b, h, nq, d = q.shape
    nk = k.shape[2]
    sc = scale if scale is not None else 1.0 / d ** 0.5
    qf, kf, vf = (t.reshape(b * h, t.shape[2], d) for t in (q, k, v))
    out = torch.empty((b * h, nq, d), device=q.device, dtype=torch.float32)
    mask = None
    if causal:
        mask = torch.ones(nq, nk, dtype=torch.bool, device=q.device).triu(1)
    for i in range(0, b * h, heads_per_chunk):
        s = torch.matmul(qf[i:i + heads_per_chunk].float(),
                         kf[i:i + heads_per_chunk].float().transpose(-1, -2))
        s *= sc
        if mask is not None:
            s.masked_fill_(mask, float("-inf"))
        out[i:i + heads_per_chunk] = torch.softmax(s, -1) @ vf[i:i + heads_per_chunk].float()
        del s
    return out.reshape(b, h, nq, d)
