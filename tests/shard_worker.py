"""
Worker for tests/test_gpu_shard.py, launched with torch.distributed.run:
each rank holds its kv-head shard of a config-5-shaped pool (a subsample of the
sequences), runs the sharded KV write + decode, all-gathers over NCCL, and rank 0
checks the gathered output against the unsharded single-GPU kernel result and
the torch fp32 reference.
"""

import json
import math
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from memforge_b200 import _kernels as K  # noqa: E402
from memforge_b200.kv_shard import HeadShard, PeerOutput, ShardedPagedDecode  # noqa: E402
from tests import cases  # noqa: E402
from tests.gpu_util import torch_reference  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from datetime import timedelta
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    meta = cases.config5_meta(0, batch=int(os.environ.get("SHARD_BATCH", "16")))
    Hq, Hkv, D, NB = 64, 8, 128, meta["num_blocks"]
    B = meta["ctx"].shape[0]
    # identical full pool on every rank (same seed); each keeps its heads
    g = torch.Generator(device=dev).manual_seed(5)
    kfull = torch.randn((NB, 16, Hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
    vfull = torch.randn((NB, 16, Hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
    q = torch.randn((B, Hq, D), generator=g, device=dev, dtype=torch.bfloat16)
    new_k = torch.randn((B, Hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
    new_v = torch.randn((B, Hkv, D), generator=g, device=dev, dtype=torch.bfloat16)
    tables = torch.from_numpy(meta["tables"].clip(min=0)).to(dev)
    ctx = torch.from_numpy(meta["ctx"]).to(dev)
    pos = meta["ctx"].astype(np.int64) - 1
    slots = torch.from_numpy((meta["tables"][np.arange(B), pos // 16].astype(np.int64) * 16
                              + pos % 16).astype(np.int32)).to(dev)
    shard = HeadShard(world, rank, Hq, Hkv)
    a, b = shard.kv_range
    step = ShardedPagedDecode(shard, NB, D, device=dev)
    step.key_pool.copy_(kfull[:, :, a:b])
    step.value_pool.copy_(vfull[:, :, a:b])
    out = step.step(q, new_k, new_v, slots, tables, ctx)
    torch.cuda.synchronize()
    K.check_device_errors(dev)
    # The same step with the output assembled over peer memory (stores into every
    # GPU's buffer + flag barrier), three steps so both buffers are reused: bit-identical.
    peer = PeerOutput(B, Hq, D, torch.bfloat16, dev)
    peer_equal = True
    for _ in range(3):
        full = step.step_peer(peer, q, new_k, new_v, slots, tables, ctx)
        torch.cuda.synchronize()
        K.check_device_errors(dev)
        peer_equal = peer_equal and bool(torch.equal(full, out))
    ok = torch.tensor([1 if peer_equal else 0], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    peer.close()
    res = {"peer_equal_nccl_all_ranks": bool(ok.item() == 1)}
    if rank == 0:
        # unsharded: same kernels on the full pool
        K.reshape_and_cache(new_k, new_v, kfull, vfull, slots)
        single = torch.empty_like(q)
        K.paged_attention(q, single, kfull, vfull, tables, ctx, scale=1 / math.sqrt(D))
        ref = torch_reference(q, kfull, vfull, tables, meta["ctx"], [1] * B, 1 / math.sqrt(D))
        res["max_vs_single"] = float((out.float() - single.float()).abs().max())
        err = (out.float() - ref).abs()
        res["max_vs_ref"] = float(err.max())
        res["within_tol"] = bool((err <= 2e-2 + 1e-2 * ref.abs()).all())
        res["pool_bit_exact"] = bool(torch.equal(step.key_pool, kfull[:, :, a:b]))
        print("SHARD_RESULT " + json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
