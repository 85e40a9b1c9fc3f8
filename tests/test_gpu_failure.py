"""
Failure detection on the GPU without a fault: a bounded wait that runs out.

``mf_peer_barrier`` completes a head-sharded step by waiting for every other
rank's epoch flag.  Here one GPU plays rank 0 of a world of two, with both
ranks' flag arrays in its own memory, and rank 1 never publishes.  The wait is
bounded (2 s of ``%globaltimer``): the kernel must give up, set
``MF_ERR_TIMEOUT`` in the error word and return, leaving the context usable, so
that a decode launched afterwards on the same context still matches the
oracle.  Nothing here traps, faults or waits without a bound.
"""

import time

import numpy as np
import pytest
import torch

from tests import cases
from tests.gpu_util import assert_close, to_dev, to_np32

pytestmark = pytest.mark.gpu

K = pytest.importorskip("memforge_b200._kernels")
L = pytest.importorskip("memforge_b200._lib")


def test_peer_barrier_times_out_when_a_rank_never_arrives():
    dev = torch.device("cuda", torch.cuda.current_device())
    K.check_device_errors(dev)
    flags = [torch.zeros(2, dtype=torch.int32, device=dev) for _ in range(2)]
    t0 = time.perf_counter()
    K.peer_barrier([f.data_ptr() for f in flags], rank=0, epoch=1, device=dev)
    torch.cuda.synchronize(dev)
    waited = time.perf_counter() - t0
    word = int(K.err_word(dev).item())
    assert word & L.MF_ERR_TIMEOUT, f"error word 0x{word:x} lacks MF_ERR_TIMEOUT"
    assert 1.5 < waited < 10.0, f"the bounded wait took {waited:.2f} s (limit 2 s)"
    # rank 0 published its epoch into both ranks' flags before waiting
    assert flags[0][0].item() == 1 and flags[1][0].item() == 1
    assert flags[0][1].item() == 0
    with pytest.raises(IndexError, match="bounded pipeline wait gave up"):
        K.check_device_errors(dev)
    assert int(K.err_word(dev).item()) == 0


def test_barrier_completes_when_every_rank_has_arrived():
    dev = torch.device("cuda", torch.cuda.current_device())
    K.check_device_errors(dev)
    flags = [torch.zeros(2, dtype=torch.int32, device=dev) for _ in range(2)]
    flags[0][1] = 1          # rank 1 has already published epoch 1 to rank 0
    t0 = time.perf_counter()
    K.peer_barrier([f.data_ptr() for f in flags], rank=0, epoch=1, device=dev)
    torch.cuda.synchronize(dev)
    assert time.perf_counter() - t0 < 1.0
    assert int(K.err_word(dev).item()) == 0


def test_context_is_usable_after_a_timeout():
    dev = torch.device("cuda", torch.cuda.current_device())
    flags = [torch.zeros(2, dtype=torch.int32, device=dev) for _ in range(2)]
    K.peer_barrier([f.data_ptr() for f in flags], rank=0, epoch=1, device=dev)
    torch.cuda.synchronize(dev)
    with pytest.raises(IndexError):
        K.check_device_errors(dev)
    c = cases.small_decode_case("after-timeout", 61, "bf16", 32, 8, 128, [1, 300, 2500])
    q = to_dev(c.q, "bf16")
    out = torch.empty_like(q)
    K.paged_attention(q, out, to_dev(c.k_pool, "bf16"), to_dev(c.v_pool, "bf16"),
                      torch.from_numpy(c.tables.clip(min=0)).cuda(),
                      torch.from_numpy(c.ctx_lens).cuda(), q_per_seq=1, scale=c.scale)
    torch.cuda.synchronize(dev)
    K.check_device_errors(dev)
    assert_close(to_np32(out), cases.oracle_decode(c), "bf16", "decode after a timeout")
    assert np.isfinite(to_np32(out)).all()
