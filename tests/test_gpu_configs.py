"""
GPU parity at the BASELINE configurations' stated sizes.

* Config 2: the KV write of 64 new tokens into the 16384-block pool, then the
  decode output of all 64 sequences, with exactly the stream-K plan the bench
  times (same lengths, tables and batch).
* Config 4: speculative verify of 32 five-token windows over contexts up to
  8192 (Hq 40), then the commit of the confirmed prefixes, the pool checked
  bit for bit against the oracle's commit (``scatter_accepted_kv`` semantics).
* Config 5: the 256-sequence, 14.5 GB pool on one GPU; the KV write is checked
  bit for bit and the decode output of a seeded subset of 16 sequences (plus
  the shortest and the longest) against the fp32 reference.

Attention is compared with ``tests.gpu_util.torch_reference`` (fp32 on the
device, itself checked against the numpy oracle in ``test_torch_reference.py``)
at the bf16 tolerance 2e-2 abs + 1e-2 rel.  KV writes and commits are bit-exact.
"""

import math

import numpy as np
import pytest
import torch

from oracle import paged_oracle as O
from tests import cases
from tests.gpu_util import TOL, torch_reference

pytestmark = pytest.mark.gpu

K = pytest.importorskip("memforge_b200._kernels")


def _close(got: torch.Tensor, want: torch.Tensor, what: str):
    tol = TOL["bf16"]
    g, w = got.float(), want.float()
    assert torch.isfinite(g).all(), f"{what}: non-finite output"
    err = (g - w).abs()
    bad = err > tol["atol"] + tol["rtol"] * w.abs()
    assert not bool(bad.any()), (f"{what}: {int(bad.sum())} elements out of tolerance, "
                                 f"max |err| {float(err.max()):.3e}")


def _pool(NB, H, D, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    kp = torch.randn((NB, 16, H, D), generator=g, device="cuda", dtype=torch.bfloat16)
    vp = torch.randn((NB, 16, H, D), generator=g, device="cuda", dtype=torch.bfloat16)
    return kp, vp, g


def _write_then_decode(meta, Hq, Hkv, D, seed):
    """The bench step: the new token's K/V at position ctx-1, then decode."""
    B = len(meta["ctx"])
    kp, vp, g = _pool(meta["num_blocks"], Hkv, D, seed)
    q = torch.randn((B, Hq, D), generator=g, device="cuda", dtype=torch.bfloat16)
    nk = torch.randn((B, Hkv, D), generator=g, device="cuda", dtype=torch.bfloat16)
    nv = torch.randn((B, Hkv, D), generator=g, device="cuda", dtype=torch.bfloat16)
    pos = meta["ctx"].astype(np.int64) - 1
    slots_np = meta["tables"][np.arange(B), pos // 16].astype(np.int64) * 16 + pos % 16
    slots = torch.from_numpy(slots_np.astype(np.int32)).cuda()
    tables = torch.from_numpy(meta["tables"].clip(min=0).astype(np.int32)).cuda()
    ctx = torch.from_numpy(meta["ctx"].astype(np.int32)).cuda()
    K.reshape_and_cache(nk, nv, kp, vp, slots)
    out = torch.empty_like(q)
    K.paged_attention(q, out, kp, vp, tables, ctx, q_per_seq=1, scale=1 / math.sqrt(D))
    torch.cuda.synchronize()
    K.check_device_errors(q.device)
    # the written slots hold the new rows bit for bit
    sl = slots.long()
    assert torch.equal(kp.view(-1, Hkv, D)[sl], nk)
    assert torch.equal(vp.view(-1, Hkv, D)[sl], nv)
    return q, out, kp, vp, tables, ctx


def test_config2_decode_output_full_batch():
    meta = cases.config2_meta(0)
    q, out, kp, vp, tables, ctx = _write_then_decode(meta, 32, 8, 128, seed=21)
    want = torch_reference(q, kp, vp, tables, meta["ctx"], [1] * len(meta["ctx"]),
                           1 / math.sqrt(128))
    _close(out, want, "config 2 decode (64 sequences)")


def test_config2_decode_is_deterministic_across_launches():
    """Stream-K partials merge in a fixed range order: repeated launches agree bit for bit."""
    meta = cases.config2_meta(0)
    q, out, kp, vp, tables, ctx = _write_then_decode(meta, 32, 8, 128, seed=22)
    again = torch.empty_like(out)
    for _ in range(3):
        K.paged_attention(q, again, kp, vp, tables, ctx, q_per_seq=1, scale=1 / math.sqrt(128))
        torch.cuda.synchronize()
        assert torch.equal(again, out)


def test_config4_verify_and_commit_full_size():
    from memforge_b200.speculative import commit_accepted, verify_attention
    meta = cases.config4_meta(0)
    B, Hq, Hkv, D, W = 32, 40, 8, 128, meta["window"]
    kp, vp, g = _pool(meta["num_blocks"], Hkv, D, 41)
    q = torch.randn((B * W, Hq, D), generator=g, device="cuda", dtype=torch.bfloat16)
    wk = torch.randn((B * W, Hkv, D), generator=g, device="cuda", dtype=torch.bfloat16)
    wv = torch.randn((B * W, Hkv, D), generator=g, device="cuda", dtype=torch.bfloat16)
    tables = torch.from_numpy(meta["tables"].clip(min=0).astype(np.int32)).cuda()
    ctx_np = meta["ctx"].astype(np.int64)
    ctx = torch.from_numpy(meta["ctx"].astype(np.int32)).cuda()
    before_k, before_v = kp.clone(), vp.clone()
    out = verify_attention(q, wk, wv, kp, vp, tables, ctx)
    torch.cuda.synchronize()
    K.check_device_errors(q.device)
    assert torch.equal(kp, before_k) and torch.equal(vp, before_v), "verify wrote the pool"
    want = torch_reference(q, kp, vp, tables, ctx_np + W, [W] * B, 1 / math.sqrt(D),
                           win_k=wk, win_v=wv)
    _close(out, want, "config 4 verify (32 x 5 rows)")

    accepted = meta["accepted"].astype(np.int32)
    commit_accepted(kp, vp, wk, wv, tables, ctx, torch.from_numpy(accepted + 1).cuda())
    torch.cuda.synchronize()
    K.check_device_errors(q.device)
    # oracle commit on the host, per sequence, on the bf16 bit patterns
    want_k = before_k.cpu().view(torch.int16).numpy().view(np.uint16)[None].copy()
    want_v = before_v.cpu().view(torch.int16).numpy().view(np.uint16)[None].copy()
    wk_bits = wk.cpu().view(torch.int16).numpy().view(np.uint16)
    wv_bits = wv.cpu().view(torch.int16).numpy().view(np.uint16)
    for s in range(B):
        t = meta["tables"][s][meta["tables"][s] >= 0]
        O.commit_accepted(want_k, want_v, 0, t, int(ctx_np[s]),
                          np.transpose(wk_bits[s * W:(s + 1) * W], (1, 0, 2))[None],
                          np.transpose(wv_bits[s * W:(s + 1) * W], (1, 0, 2))[None],
                          int(accepted[s]) + 1, 16, "bf16")
    got_k = kp.cpu().view(torch.int16).numpy().view(np.uint16)
    got_v = vp.cpu().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got_k, want_k[0]), "config 4 commit: key pool differs from the oracle"
    assert np.array_equal(got_v, want_v[0]), "config 4 commit: value pool differs from the oracle"


def test_config5_decode_single_gpu_subset():
    """256 sequences, contexts log-uniform in [4096, 32768], 14.5 GB of K/V on one GPU."""
    meta = cases.config5_meta(0)
    free, _ = torch.cuda.mem_get_info()
    need = meta["num_blocks"] * 16 * 8 * 128 * 2 * 2
    if free < need + (8 << 30):
        pytest.skip(f"needs {need / 2**30:.1f} GiB of free device memory")
    q, out, kp, vp, tables, ctx = _write_then_decode(meta, 64, 8, 128, seed=51)
    B = len(meta["ctx"])
    g = np.random.default_rng(5)
    pick = set(g.choice(B, size=16, replace=False).tolist())
    pick |= {int(np.argmin(meta["ctx"])), int(np.argmax(meta["ctx"]))}
    for s in sorted(pick):
        want = torch_reference(q[s:s + 1], kp, vp, tables[s:s + 1], meta["ctx"][s:s + 1], [1],
                               1 / math.sqrt(128))
        _close(out[s:s + 1], want, f"config 5 decode, sequence {s} (ctx {int(meta['ctx'][s])})")
