"""GPU tests of the key-range split mode (problems with fewer query pairs than
SMs): results against the oracle and against the unsplit kernel, repeated
calls (the arrival counters must reset themselves), and concurrent streams
(each stream has its own scratch buffer)."""

import pytest
import torch

from flash_attention_2_lab_b200 import _native
from oracle.attention_oracle import attention_oracle
from parity_utils import abi_forward, assert_parity, read_status

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _split_across_blocks():
    # An explicit limit selects the cross-block split; the automatic policy
    # keeps one-wave problems in one block per query tile instead.
    _native.lib().fa_set_max_splits(16)
    yield
    _native.lib().fa_set_max_splits(0)
    assert read_status() == 0


def seeded(b, h, nq, nk, seed):
    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(b, h, n, 64, generator=g).half().cuda() for n in (nq, nk, nk))


# (splits need >= 8 key tiles each, i.e. >= 2048 keys for two splits)
CASES = [(1, 8, 2048, 2048), (1, 2, 4096, 4096), (1, 1, 8192, 8192), (2, 1, 640, 3000),
         (1, 3, 300, 2500), (1, 1, 128, 9000), (1, 1, 1000, 5000)]


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize(("b", "h", "nq", "nk"), CASES)
def test_split_matches_oracle_and_unsplit(b, h, nq, nk, causal):
    q, k, v = seeded(b, h, nq, nk, seed=nq * 7 + nk)
    split = abi_forward(q, k, v, causal)
    torch.cuda.synchronize()
    ref = attention_oracle(q.float().cpu().numpy(), k.float().cpu().numpy(),
                           v.float().cpu().numpy(), causal=causal)
    assert_parity(split, ref, what="split")
    _native.lib().fa_set_max_splits(1)
    whole = abi_forward(q, k, v, causal)
    torch.cuda.synchronize()
    assert_parity(whole, ref, what="unsplit")
    assert (split.float() - whole.float()).abs().max().item() < 4e-3
    _native.lib().fa_set_max_splits(0)
    auto = abi_forward(q, k, v, causal)
    torch.cuda.synchronize()
    assert_parity(auto, ref, what="automatic (in-block key halves)")


def test_split_repeated_calls_and_sizes():
    # counters reset themselves: many calls, alternating shapes, same answers
    ref = {}
    for rep in range(3):
        for (nq, nk) in ((2048, 2048), (2048, 512), (512, 4096)):
            q, k, v = seeded(1, 4, nq, nk, seed=nq + nk)
            out = abi_forward(q, k, v, True)
            torch.cuda.synchronize()
            if rep == 0:
                ref[(nq, nk)] = out.clone()
            else:
                assert torch.equal(out, ref[(nq, nk)])


def test_split_two_streams():
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    qa, ka, va = seeded(1, 8, 2048, 2048, seed=1)
    qb, kb, vb = seeded(1, 2, 1024, 4000, seed=2)
    ea = abi_forward(qa, ka, va, False)
    eb = abi_forward(qb, kb, vb, True)
    torch.cuda.synchronize()
    for _ in range(5):
        s1.wait_stream(torch.cuda.current_stream())
        s2.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s1):
            oa = abi_forward(qa, ka, va, False, stream=s1)
        with torch.cuda.stream(s2):
            ob = abi_forward(qb, kb, vb, True, stream=s2)
        torch.cuda.synchronize()
        assert torch.equal(oa, ea) and torch.equal(ob, eb)


def test_release_workspaces():
    q, k, v = seeded(1, 2, 2048, 2048, seed=3)
    a = abi_forward(q, k, v, False)
    torch.cuda.synchronize()
    assert _native.lib().fa_release_workspaces() == 0
    b = abi_forward(q, k, v, False)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_split_layouts_in_sequence():
    # A small split problem followed by a larger one: the scratch buffer's
    # counter prefix must stay zero whatever the previous launch stored.
    seq = [((1, 1, 1000, 5000), False), ((1, 8, 2048, 2048), True),
           ((1, 2, 4096, 4096), False), ((1, 8, 2048, 2048), False)]
    for _ in range(2):
        for (b, h, nq, nk), causal in seq:
            q, k, v = seeded(b, h, nq, nk, seed=nq * 7 + nk)
            out = abi_forward(q, k, v, causal)
            torch.cuda.synchronize()
            ref = attention_oracle(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                   v.float().cpu().numpy(), causal=causal)
            assert_parity(out, ref, what=f"{(b, h, nq, nk, causal)}")


def test_split_recovers_after_a_timed_out_launch():
    # A split launch whose waits run out of time returns early, possibly after
    # some splits have counted themselves finished.  The counters are cleared
    # before every split launch, so the next launch on the stream is correct.
    q, k, v = seeded(1, 2, 4096, 4096, seed=11)
    lib = _native.lib()
    try:
        lib.fa_set_wait_limit_ns(1000)  # 1 us: the pipeline's first waits give up
        abi_forward(q, k, v, False)
        torch.cuda.synchronize()
    finally:
        lib.fa_set_wait_limit_ns(0)
    read_status(clear=True)  # may or may not report the time-outs
    ref = attention_oracle(q.float().cpu().numpy(), k.float().cpu().numpy(),
                           v.float().cpu().numpy(), causal=False)
    for _ in range(2):
        out = abi_forward(q, k, v, False)
        torch.cuda.synchronize()
        assert_parity(out, ref, what="split after a timed-out launch")
