"""attention_forward_host: host-resident inputs streamed through the GPU in
batch chunks (H2D, kernel and D2H on separate streams)."""

import pytest
import torch

import flash_attention_2_lab_b200 as fa
from flash_attention_2_lab_b200.host_pipeline import attention_forward_host
from parity_utils import assert_parity


def test_rejects_device_tensors_and_bad_shapes():
    x = torch.zeros(1, 2, 128, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="contiguous float16"):
        attention_forward_host(x.float(), x, x)
    with pytest.raises(ValueError, match="chunk_batches"):
        attention_forward_host(x, x, x, chunk_batches=0)
    with pytest.raises(ValueError, match="shape"):
        attention_forward_host(x[0], x, x)


@pytest.mark.gpu
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize(("b", "h", "nq", "nk", "chunk"),
                         [(5, 4, 1024, 1024, 2), (3, 2, 300, 700, 1), (2, 8, 2048, 2048, 4)])
def test_matches_device_call(b, h, nq, nk, chunk, causal):
    g = torch.Generator().manual_seed(b * 100 + nq)
    q = torch.randn(b, h, nq, 64, generator=g).half().pin_memory()
    k = torch.randn(b, h, nk, 64, generator=g).half().pin_memory()
    v = torch.randn(b, h, nk, 64, generator=g).half().pin_memory()
    out = attention_forward_host(q, k, v, causal, chunk_batches=chunk)
    assert out.device.type == "cpu" and out.shape == q.shape
    ref = fa.attention_forward(q.cuda(), k.cuda(), v.cuda(), causal).float().cpu()
    assert_parity(out.float(), ref, atol=4e-3, rtol=1e-2, what="host pipeline vs device call")
