"""CPU tests of the (batch, head) sharding host logic, including a
world-size-2 gloo run of the per-rank path the benchmark uses."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flash_attention_2_lab_b200 import workloads
from flash_attention_2_lab_b200.sharded import max_over_ranks, shard_range, split_dim
from oracle.attention_oracle import attention_oracle


@pytest.mark.parametrize("total", [0, 1, 7, 32, 1024])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_range_partitions(total, world):
    parts = [shard_range(total, world, r) for r in range(world)]
    flat = [i for p in parts for i in p]
    assert flat == list(range(total))
    sizes = [len(p) for p in parts]
    assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_split_dim():
    assert split_dim(32, 32, 8) == "batch"
    assert split_dim(2, 16, 8) == "batch_head"


def test_workload_bytes_independent_of_sharding():
    cfg = workloads.Config("tiny", 4, 2, 16)
    q, k, v = workloads.make_inputs(cfg, seed=3)
    q2, k2, v2 = workloads.make_inputs(cfg, seed=3, batches=range(2, 4))
    assert torch.equal(q[2:], q2) and torch.equal(k[2:], k2) and torch.equal(v[2:], v2)


def test_stress_workload_has_outliers():
    cfg = workloads.Config("tiny_stress", 1, 2, 200, stress=True)
    q, k, v = workloads.make_inputs(cfg, seed=0)
    rows = (k.float().abs() == 30).all(dim=-1)
    assert rows.sum(dim=-1).tolist() == [[2, 2]]
    assert q.float().std() > 4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = workloads.Config("tiny", 5, 2, 40)
    mine = shard_range(cfg.batch, world, rank)
    q, k, v = workloads.make_inputs(cfg, seed=1, batches=mine)
    out = attention_oracle(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=True)
    # the optional final gather of the launcher
    buf = [None] * world
    dist.all_gather_object(buf, out)
    t = max_over_ranks(1.0 + rank)
    if rank == 0:
        np.save(os.path.join(result_dir, "gathered.npy"), np.concatenate(buf))
        np.save(os.path.join(result_dir, "tmax.npy"), np.array([t]))
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_world2_sharded_equals_full(tmp_path):
    port = _free_port()
    mp.spawn(_rank_main, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    gathered = np.load(tmp_path / "gathered.npy")
    cfg = workloads.Config("tiny", 5, 2, 40)
    q, k, v = workloads.make_inputs(cfg, seed=1)
    full = attention_oracle(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=True)
    np.testing.assert_allclose(gathered, full, rtol=1e-6, atol=1e-6)
    assert float(np.load(tmp_path / "tmax.npy")[0]) == 2.0


def test_max_over_ranks_without_process_group():
    assert max_over_ranks(3.5) == 3.5


def _rank_dies(rank, world, port, result_dir):
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        os._exit(0)  # a rank that leaves between steps, before the timing reduction
    try:
        max_over_ranks(1.0)
        outcome = "returned"
    except Exception as e:  # the surviving rank must get an error, not hang
        outcome = "error: " + type(e).__name__
    with open(os.path.join(result_dir, "outcome.txt"), "w") as f:
        f.write(outcome)
    os._exit(0)


def test_lost_rank_is_detected_not_hung(tmp_path):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_dies, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
        assert not p.is_alive()
    assert (tmp_path / "outcome.txt").read_text().startswith("error")
