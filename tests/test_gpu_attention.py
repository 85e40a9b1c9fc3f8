"""
GPU parity of the paged attention kernels against the numpy oracle (small,
seeded cases) across dtypes, head geometries, ragged lengths, stream-K splits,
speculative windows and error paths.  Tolerances: fp32 1e-5; bf16/fp16
2e-2 abs + 1e-2 rel (the stated tolerance for this path).
"""

import math

import numpy as np
import pytest
import torch

from tests import cases
from tests.gpu_util import assert_close, to_dev, to_np32

pytestmark = pytest.mark.gpu

K = pytest.importorskip("memforge_b200._kernels")


def run_case(case, window=None, causal=True, check=True):
    q = to_dev(case.q, case.dtype)
    kp = to_dev(case.k_pool, case.dtype)
    vp = to_dev(case.v_pool, case.dtype)
    tables = torch.from_numpy(case.tables.clip(min=0)).cuda()
    kv = torch.from_numpy(case.ctx_lens).cuda()
    out = torch.empty_like(q)
    wk = wv = None
    if window is not None:
        wk = to_dev(np.concatenate([np.transpose(window[s][1], (1, 0, 2)) for s in range(case.batch)]), case.dtype)
        wv = to_dev(np.concatenate([np.transpose(window[s][2], (1, 0, 2)) for s in range(case.batch)]), case.dtype)
    K.paged_attention(q, out, kp, vp, tables, kv, q_per_seq=case.q_per_seq, scale=case.scale,
                      causal=causal, win_k=wk, win_v=wv)
    torch.cuda.synchronize()
    if check:
        K.check_device_errors(q.device)
    return to_np32(out)


def check(case, window=None):
    got = run_case(case, window)
    want = cases.oracle_decode(case, window=window)
    assert_close(got, want, case.dtype, case.name)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("hq,hkv", [(8, 8), (16, 4), (28, 4), (32, 8), (64, 8), (8, 1), (16, 2)])
def test_decode_matches_oracle(hq, hkv, dtype):
    c = cases.small_decode_case(f"dec{hq}x{hkv}", 100 + hq, dtype, hq, hkv, 128, [1, 77, 300])
    check(c)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("ctx", [[1], [15, 16, 17], [63, 64, 65], [2048, 5], [129, 128, 127, 16]])
def test_ragged_lengths_and_page_boundaries(ctx, D):
    c = cases.small_decode_case(f"rag{D}", 7, "bf16", 16, 4, D, ctx)
    check(c)


def test_many_way_split_merges_exactly():
    """Few long sequences over 148 SMs: each is cut into ~50-150 ranges."""
    c = cases.small_decode_case("split", 8, "bf16", 32, 8, 128, [4000, 3000, 1, 17])
    check(c)


@pytest.mark.parametrize("hq,hkv", [(8, 1), (16, 2)])
def test_one_or_two_kv_heads_many_ranges(hq, hkv):
    """The per-GPU shapes of an 8- or 4-way kv-head shard of a GQA-8 model: the
    SM runs 8 or 4 independent page ranges, so long sequences are cut into
    many pieces that merge."""
    c = cases.small_decode_case(f"few{hkv}", 22, "bf16", hq, hkv, 128, [6000, 2500, 1, 700, 33])
    check(c)


def test_many_short_sequences():
    g = cases.rng(9)
    ctx = g.integers(1, 80, size=300).tolist()
    c = cases.small_decode_case("short", 9, "bf16", 32, 8, 128, ctx)
    check(c)


@pytest.mark.parametrize("hq,hkv,D", [(15, 5, 64), (4, 4, 32), (6, 2, 80)])
def test_fp32_generic_path_matches_oracle(hq, hkv, D):
    c = cases.small_decode_case("f32", 11, "f32", hq, hkv, D, [1, 33, 513])
    check(c)


def test_config1_fp32():
    c = cases.config1(0)
    check(c)


@pytest.mark.parametrize("hq,hkv,W", [(40, 8, 5), (64, 8, 5), (32, 8, 4), (16, 2, 3), (32, 2, 16)])
def test_verify_window_matches_oracle(hq, hkv, W):
    c = cases.small_decode_case("verify", 12, "bf16", hq, hkv, 128, [max(5, W), 200, 1000, 33],
                                q_per_seq=W)
    g = cases.rng(12)
    window = {s: (int(c.ctx_lens[s]) - W, cases.bf16_round(cases.normal(g, (hkv, W, 128))),
                  cases.bf16_round(cases.normal(g, (hkv, W, 128)))) for s in range(c.batch)}
    check(c, window)


def test_verify_long_windows_repeat_bit_for_bit():
    """A 16-row verify window over long contexts (GQA 8, so one 128-row tile
    holds every row of a kv head): the output matches the oracle, and repeated
    launches give the same bits."""
    W = 16
    c = cases.small_decode_case("vsplit", 21, "bf16", 16, 2, 128, [8000 + W, 3000 + W, W],
                                q_per_seq=W)
    g = cases.rng(21)
    window = {s: (int(c.ctx_lens[s]) - W, cases.bf16_round(cases.normal(g, (2, W, 128))),
                  cases.bf16_round(cases.normal(g, (2, W, 128)))) for s in range(c.batch)}
    first = run_case(c, window)
    assert_close(first, cases.oracle_decode(c, window=window), "bf16", "vsplit")
    for _ in range(2):
        assert np.array_equal(run_case(c, window), first)


def test_uniform_long_runs_need_no_decode_launch():
    """A verify batch with one q_per_seq (every run longer than 8 rows per kv
    head) is served by the tcgen05 kernel alone, so it needs no workspace; a
    varlen batch that mixes one-row and long runs also launches the decode
    kernel, which does."""
    from memforge_b200._lib import MF_EWORKSPACE, MemforgeError
    W = 5
    c = cases.small_decode_case("uni", 23, "bf16", 40, 8, 128, [W + 300, W + 40], q_per_seq=W)
    g = cases.rng(23)
    window = {s: (int(c.ctx_lens[s]) - W, cases.bf16_round(cases.normal(g, (8, W, 128))),
                  cases.bf16_round(cases.normal(g, (8, W, 128)))) for s in range(c.batch)}
    empty = torch.empty(0, dtype=torch.uint8, device="cuda")
    q = to_dev(c.q, "bf16")
    out = torch.empty_like(q)
    kp, vp = to_dev(c.k_pool, "bf16"), to_dev(c.v_pool, "bf16")
    tables = torch.from_numpy(c.tables.clip(min=0)).cuda()
    kv = torch.from_numpy(c.ctx_lens).cuda()
    wk = to_dev(np.concatenate([np.transpose(window[s][1], (1, 0, 2)) for s in range(c.batch)]), "bf16")
    wv = to_dev(np.concatenate([np.transpose(window[s][2], (1, 0, 2)) for s in range(c.batch)]), "bf16")
    K.paged_attention(q, out, kp, vp, tables, kv, q_per_seq=W, scale=c.scale, win_k=wk, win_v=wv,
                      workspace_tensor=empty)
    torch.cuda.synchronize()
    K.check_device_errors(q.device)
    assert_close(to_np32(out), cases.oracle_decode(c, window=window), "bf16", "uniform verify")
    # the same pool as a varlen batch: a one-row run beside a 40-row run
    cu = torch.tensor([0, 1, 41], dtype=torch.int32, device="cuda")
    qv = torch.empty((41, 40, 128), dtype=torch.bfloat16, device="cuda").normal_()
    with pytest.raises(MemforgeError) as e:
        K.paged_attention(qv, torch.empty_like(qv), kp, vp, tables, kv, cu_seqlens_q=cu,
                          max_q_len=40, scale=c.scale, workspace_tensor=empty)
    assert e.value.code == MF_EWORKSPACE


def test_verify_window_ignores_stale_pool_slots():
    """With a side window the pool holds only the context: NaN in its unwritten
    slots (where the window's positions would go) must not leak."""
    W = 5
    c = cases.small_decode_case("wstale", 19, "bf16", 40, 8, 128, [W + 37, W + 128, W + 300],
                                q_per_seq=W)
    g = cases.rng(19)
    window = {s: (int(c.ctx_lens[s]) - W, cases.bf16_round(cases.normal(g, (8, W, 128))),
                  cases.bf16_round(cases.normal(g, (8, W, 128)))) for s in range(c.batch)}
    a = run_case(c, window)
    for s in range(c.batch):
        n = int(c.ctx_lens[s]) - W  # pool positions 0 .. n-1 are written
        for pos in range(n, n + W):
            blk = c.tables[s][pos // 16]
            if blk >= 0:
                c.k_pool[blk, pos % 16] = np.nan
                c.v_pool[blk, pos % 16] = np.nan
    b = run_case(c, window)
    assert np.isfinite(b).all()
    assert np.array_equal(a, b)
    check(c, window)


@pytest.mark.parametrize("W", [2, 5, 16])
def test_multi_row_causal_from_pool(W):
    """Verify-style rows whose keys are already in the pool (no side window)."""
    c = cases.small_decode_case("mrow", 13, "bf16", 32, 8, 128, [W, 64, 301], q_per_seq=W)
    check(c)


def test_long_bf16_rows_take_the_prefill_kernel():
    """160 rows per kv head (G 4 x 40 positions): dispatched to the tcgen05 prefill kernel."""
    c = cases.small_decode_case("long", 14, "bf16", 32, 8, 128, [70, 300], q_per_seq=40)
    check(c)


@pytest.mark.parametrize("q_per_seq", [1, 3, 40])
def test_bf16_head_dim_80_takes_the_generic_kernel(q_per_seq):
    """head_dim 80 is served by neither tensor-core kernel: the generic CUDA-core kernel, bf16."""
    c = cases.small_decode_case("gen80", 15, "bf16", 12, 4, 80, [40, 50, 333], q_per_seq=q_per_seq)
    check(c)


def test_noncausal_rows_see_the_whole_context():
    c = cases.small_decode_case("nc", 15, "f32", 4, 4, 64, [20, 50], q_per_seq=3)
    got = run_case(c, causal=False)
    c2 = cases.DecodeCase(**{**c.__dict__})
    # every row sees kv_len keys: the oracle with all positions = kv_len - 1
    from oracle.paged_oracle import varlen_attention
    seq_ids = [s for s in range(c.batch) for _ in range(3)]
    positions = [int(c.ctx_lens[s]) - 1 for s in range(c.batch) for _ in range(3)]
    tables = [c.tables[s][c.tables[s] >= 0] for s in range(c.batch)]
    want = varlen_attention(np.transpose(c.q, (1, 0, 2)), c.k_pool[None], c.v_pool[None], 0,
                            tables, seq_ids, positions, 16, scale=c.scale)
    assert_close(got, np.transpose(want, (1, 0, 2)), "f32", "noncausal")


def test_stale_slots_past_the_context_are_never_read():
    """NaN in unwritten slots of the last page must not leak (test_varlen_attention.py:299-322)."""
    c = cases.small_decode_case("stale", 16, "bf16", 16, 4, 128, [40, 7])
    a = run_case(c)
    for s in range(c.batch):
        n = int(c.ctx_lens[s])
        last = c.tables[s][(n - 1) // 16]
        c.k_pool[last, n % 16 or 16:] = np.nan
        c.v_pool[last, n % 16 or 16:] = np.nan
    b = run_case(c)
    assert np.isfinite(b).all()
    assert np.array_equal(a, b)


def test_large_scores_stay_finite():
    c = cases.small_decode_case("big", 17, "bf16", 8, 2, 128, [11, 300], q_std=8.0, kv_std=8.0)
    check(c)


def test_bad_block_id_is_reported_not_faulted():
    c = cases.small_decode_case("bad", 18, "bf16", 8, 2, 128, [40])
    c.tables[0, 1] = c.num_blocks + 5
    run_case(c, check=False)
    with pytest.raises(IndexError, match="block table entry"):
        K.check_device_errors(torch.device("cuda"))


def test_workspace_is_reusable_back_to_back():
    """Split-K arrival counters are left zeroed: repeated launches stay correct."""
    c = cases.small_decode_case("ws", 19, "bf16", 32, 8, 128, [4000, 30, 900])
    want = cases.oracle_decode(c)
    for _ in range(3):
        assert_close(run_case(c), want, "bf16", "repeat")
