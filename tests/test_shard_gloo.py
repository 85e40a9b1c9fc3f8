"""
KV-head sharding logic on CPU with world_size-2 gloo process groups.

Each rank computes attention for its own kv heads with the CPU oracle (the GPU
kernels are exercised by tests/test_gpu_shard.py); what is tested here is the
head partition, the replicated block tables, and the all-gather + permute that
reassembles ``[B, Hq, D]`` exactly as the unsharded computation lays it out.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from memforge_b200.kv_shard import HeadShard, gather_heads
from tests import cases


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = cases.small_decode_case("shard", 21, "f32", 16, 8, 32, [5, 70, 130])
        shard = HeadShard(world, rank, 16, 8)
        a, b = shard.kv_range
        qa, qb = shard.q_range
        # this rank's slice of the pool and queries; tables replicated unchanged
        local = cases.DecodeCase(**{**c.__dict__, "num_q_heads": qb - qa, "num_kv_heads": b - a,
                                    "q": np.ascontiguousarray(c.q[:, qa:qb]),
                                    "k_pool": np.ascontiguousarray(c.k_pool[:, :, a:b]),
                                    "v_pool": np.ascontiguousarray(c.v_pool[:, :, a:b])})
        out_local = torch.from_numpy(cases.oracle_decode(local))
        # views, not copies
        qt = torch.from_numpy(c.q)
        assert shard.local_q(qt).data_ptr() == qt[:, qa:qb].data_ptr()
        full = gather_heads(out_local)
        result_q.put((rank, full.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_sharded_decode_reassembles_the_unsharded_result(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    c = cases.small_decode_case("shard", 21, "f32", 16, 8, 32, [5, 70, 130])
    want = cases.oracle_decode(c)
    for r in range(world):
        assert np.allclose(results[r], want, atol=1e-6), r


def test_head_shard_ranges():
    shards = [HeadShard(4, r, 64, 8) for r in range(4)]
    assert [s.kv_range for s in shards] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    assert [s.q_range for s in shards] == [(0, 16), (16, 32), (32, 48), (48, 64)]
    with pytest.raises(ValueError, match="do not split"):
        HeadShard(3, 0, 64, 8)
    with pytest.raises(ValueError, match="outside world"):
        HeadShard(2, 2, 64, 8)


def _failing_worker(rank, world, port, result_q):
    """Rank 1 never joins the collective: rank 0's short timeout must end it."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    try:
        if rank == 1:
            result_q.put((rank, "left"))
            return                 # leaves between steps, no collective in flight
        try:
            gather_heads(torch.zeros(2, 4, 8))
            result_q.put((rank, "completed"))
        except Exception as e:     # the host learns of the missing rank
            result_q.put((rank, type(e).__name__))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_missing_rank_is_reported_on_the_host():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "left"
    assert res[0] != "completed"
