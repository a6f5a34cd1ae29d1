"""GPU test of the (batch, head) sharded launcher over every visible device:
the sharded result must be bit-identical to the single-device result (each
head is computed by the same kernel code on the same bytes)."""

import pytest
import torch

import flash_attention_2_lab_b200 as fa
from flash_attention_2_lab_b200.sharded import attention_forward_sharded

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("causal", [False, True])
def test_sharded_equals_single_device(causal):
    n_dev = torch.cuda.device_count()
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(8, 4, 1024, 64, generator=g).half() for _ in range(3))
    single = fa.attention_forward(q.cuda(0), k.cuda(0), v.cuda(0), causal)
    sharded = attention_forward_sharded(q, k, v, causal, devices=list(range(n_dev)), gather_to=0)
    torch.cuda.synchronize()
    assert torch.equal(sharded, single)


def test_sharded_flattened_heads_when_batch_small():
    n_dev = torch.cuda.device_count()
    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(1, 16, 512, 64, generator=g).half() for _ in range(3))
    single = fa.attention_forward(q.cuda(0), k.cuda(0), v.cuda(0), True)
    sharded = attention_forward_sharded(q, k, v, True, devices=list(range(n_dev)) * 2,
                                        gather_to=0)
    torch.cuda.synchronize()
    assert torch.equal(sharded, single)
