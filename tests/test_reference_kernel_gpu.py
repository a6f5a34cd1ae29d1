"""Second parity witness: the reference's own production kernel
(tensorcore_attention_forward_production_128x128, csrc/tensorcore_attention.cu:
2019-2727), built for sm_100a from the reference sources by oracle/build_ref.py
into oracle/_ref/.  Skipped where that build is absent."""

import importlib.util
from pathlib import Path

import pytest
import torch

import flash_attention_2_lab_b200 as fa
from oracle.attention_oracle import attention_oracle
from parity_utils import assert_parity

pytestmark = pytest.mark.gpu

REF_SO = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "flash_attention_cuda_ref.so"


@pytest.fixture(scope="module")
def ref_ext():
    if not REF_SO.exists():
        pytest.skip("reference kernel not built (oracle/build_ref.py)")
    spec = importlib.util.spec_from_file_location("flash_attention_cuda_ref", REF_SO)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize(("b", "h", "n"), [(1, 2, 128), (1, 4, 256), (1, 8, 512), (1, 8, 1024),
                                           (2, 4, 2048)])
def test_matches_reference_kernel(ref_ext, b, h, n, causal):
    g = torch.Generator().manual_seed(n + b)
    q, k, v = (torch.randn(b, h, n, 64, generator=g).half().cuda() for _ in range(3))
    ours = fa.tensorcore_attention_forward_production_128x128(q, k, v, causal)
    theirs = ref_ext.tensorcore_attention_forward_production_128x128(q, k, v, causal)
    torch.cuda.synchronize()
    torch.testing.assert_close(ours, theirs, rtol=3e-2, atol=3e-2)
    ref = attention_oracle(q.float().cpu().numpy(), k.float().cpu().numpy(),
                           v.float().cpu().numpy(), causal=causal)
    assert_parity(ours, ref, what="ours")
    assert_parity(theirs, ref, what="reference kernel")
