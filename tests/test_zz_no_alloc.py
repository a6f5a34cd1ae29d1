"""GPU test of fa_fwd_sm100_noalloc, the entry point for callers that must not
allocate device memory during the call (code running under CUDA graph
capture, serving paths with a memory budget fixed at start-up, code called
from an allocator callback).  It must give the same results as the regular
entry point, including in the key-range split mode whose scratch lives in a
fixed array inside the library, on consecutive calls (the array keeps the
previous call's contents).

Named so that pytest collects it last."""

import pytest
import torch

from flash_attention_2_lab_b200 import _native
from parity_utils import ATOL, RTOL, abi_forward, read_status

pytestmark = pytest.mark.gpu


def noalloc_forward(q, k, v, causal, scale=None):
    out = torch.empty_like(q)
    b, h, nq, d = q.shape
    sc = scale if scale is not None else 1.0 / d ** 0.5
    rc = _native.lib().fa_fwd_sm100_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                            out.data_ptr(), b, h, nq, k.shape[2], int(causal),
                                            sc, torch.cuda.current_stream().cuda_stream)
    _native.check(rc)
    return out


# the first three use the key-range split mode (scratch), the last does not
CASES = [(1, 8, 2048, 2048), (1, 1, 8192, 8192), (1, 2, 1000, 6000), (2, 4, 1024, 1024)]


@pytest.fixture
def split_across_blocks():
    # An explicit split limit: the first three cases use the cross-block split
    # and its scratch (the automatic policy keeps one-wave problems in-block).
    # The teardown restores the process-wide policy even when a check fails.
    _native.lib().fa_set_max_splits(16)
    yield
    _native.lib().fa_set_max_splits(0)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize(("b", "h", "nq", "nk"), CASES)
def test_noalloc_matches_regular_entry_point_twice(split_across_blocks, b, h, nq, nk, causal):
    g = torch.Generator().manual_seed(nq + nk + b)
    q = torch.randn(b, h, nq, 64, generator=g).half().cuda()
    k = torch.randn(b, h, nk, 64, generator=g).half().cuda()
    v = torch.randn(b, h, nk, 64, generator=g).half().cuda()
    expected = abi_forward(q, k, v, causal).float()
    for _ in range(2):
        got = noalloc_forward(q, k, v, causal).float()
        torch.cuda.synchronize()
        bound = ATOL + RTOL * expected.abs()
        assert ((got - expected).abs() <= bound).all()
    assert read_status() == 0


def test_noalloc_takes_no_device_memory(split_across_blocks):
    # On a stream that has never run a split launch, the regular entry point
    # would allocate its scratch buffer (several MiB here); the no-alloc entry
    # point must leave the device's free memory unchanged.
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(1, 1, 8192, 64, generator=g).half().cuda() for _ in range(3))
    out = torch.empty_like(q)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    free_before, _ = torch.cuda.mem_get_info()
    with torch.cuda.stream(side):
        for _ in range(2):
            rc = _native.lib().fa_fwd_sm100_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                                    out.data_ptr(), 1, 1, 8192, 8192, 0, 0.125,
                                                    side.cuda_stream)
            _native.check(rc)
    side.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before
    expected = abi_forward(q, k, v, False)
    torch.cuda.synchronize()
    bound = ATOL + RTOL * expected.float().abs()
    assert ((out.float() - expected.float()).abs() <= bound).all()
    assert read_status() == 0
