"""GPU tests of the (batch, head) sharded launcher over every visible device
(run on 1 GPU by the default suite and on 2-8 GPUs by a multi-GPU call): the
gathered result must match the FP32 oracle at the north-star bound and the
single-device result closely.  A shard may take a different kernel variant
than the whole problem (fewer heads per device can make its query tiles fit
one wave, which selects the in-block key-range halves), so the comparison
with the single-device result is by tolerance, not bit for bit."""

import pytest
import torch

import flash_attention_2_lab_b200 as fa
from flash_attention_2_lab_b200.sharded import attention_forward_sharded
from oracle.attention_oracle import attention_oracle
from parity_utils import assert_parity

pytestmark = pytest.mark.gpu


def _check(q, k, v, causal, devices):
    single = fa.attention_forward(q.cuda(0), k.cuda(0), v.cuda(0), causal)
    sharded = attention_forward_sharded(q, k, v, causal, devices=devices, gather_to=0)
    torch.cuda.synchronize()
    assert sharded.shape == q.shape and sharded.device == torch.device("cuda", 0)
    ref = attention_oracle(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                           causal=causal)
    assert_parity(sharded, ref, what=f"sharded over {len(devices)} devices")
    assert (sharded.float() - single.float()).abs().max().item() < 4e-3


@pytest.mark.parametrize("causal", [False, True])
def test_sharded_matches_oracle_and_single_device(causal):
    n_dev = torch.cuda.device_count()
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(8, 4, 1024, 64, generator=g).half() for _ in range(3))
    _check(q, k, v, causal, list(range(n_dev)))


def test_sharded_flattened_heads_when_batch_small():
    n_dev = torch.cuda.device_count()
    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(1, 16, 512, 64, generator=g).half() for _ in range(3))
    _check(q, k, v, True, list(range(n_dev)) * 2)


def test_device_count_reported():
    # Records how many devices the sharded tests above spanned in this run.
    print(f"sharded tests ran over {torch.cuda.device_count()} device(s)")
    assert torch.cuda.device_count() >= 1
