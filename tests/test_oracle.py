"""
Pin the CPU oracle to the reference before trusting it.

Two kinds of evidence:
* known-answer vectors written in the reference's own test files (cited by
  file:line), restated here as constants;
* golden fixtures produced by running the reference's functions
  (``tests/golden/make_golden.py``).

Integer and byte results must be identical; fp32 attention within the
reference's own tolerance (``ATOL = 1e-5``, ``tests/python/test_varlen_attention.py:36``).
"""

from __future__ import annotations

import glob
import math
import os

import numpy as np
import pytest

from oracle import paged_oracle as O
from tests import cases
from tests.conftest import GOLDEN

ATOL = 1e-5


def load(name):
    return np.load(os.path.join(GOLDEN, name))


# ------------------------------------------------------------------ slot math

def test_slot_indices_known_answer():
    # tests/python/test_kv_pool.py:20-28
    phys, slots = O.slot_indices(np.array([5, 2, 7]), 0, 10, 4)
    assert phys.tolist() == [5, 5, 5, 5, 2, 2, 2, 2, 7, 7]
    assert slots.tolist() == [0, 1, 2, 3, 0, 1, 2, 3, 0, 1]


def test_slot_indices_mid_range_known_answer():
    # tests/python/test_kv_pool.py:31-38
    phys, slots = O.slot_indices(np.array([5, 2, 7]), 6, 9, 4)
    assert phys.tolist() == [2, 2, 7]
    assert slots.tolist() == [2, 3, 0]


def test_slot_indices_rejects_past_table():
    # tests/python/test_kv_pool.py:41-46
    with pytest.raises(IndexError, match="outside a block table"):
        O.slot_indices(np.array([5, 2]), 0, 12, 4)


def test_flat_slot_index_known_answer():
    # tests/python/test_kernels.py:38-42
    flat = O.flat_slot_index(np.array([3, 1, 0, 2]), np.array([0, 2, 3, 1]), 4)
    assert flat.tolist() == [12, 6, 3, 9]
    assert flat.tolist() == load("flat_slot_index.npz")["flat"].tolist()


def test_group_by_sequence_known_answer():
    # tests/python/test_varlen_attention.py:89-94
    assert O.group_by_sequence([2, 0, 2, 1, 0]) == [(2, [0, 2]), (0, [1, 4]), (1, [3])]
    assert O.group_by_sequence([7]) == [(7, [0])]


# ------------------------------------------------------------- bf16 rounding

def test_bf16_rounding_is_round_to_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, 1e-40, 0.0, -0.0],
                 dtype=np.float32)
    b = O.f32_to_bf16(x)
    back = O.bf16_to_f32(b)
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7: even mantissa (1.0) wins.
    assert back[1] == 1.0
    # 1 + 3*2^-8 ties between 1+2^-7 and 1+2^-6: even is 1+2^-6.
    assert back[2] == np.float32(1.015625)
    assert back[3] == -2.5
    assert np.isinf(back[4]) or back[4] > 3e38


def test_bf16_rounding_matches_torch():
    torch = pytest.importorskip("torch")
    g = cases.rng(7)
    x = np.concatenate([cases.normal(g, (4096,), 10.0),
                        np.array([np.inf, -np.inf, 65504.0, 1e-38], np.float32)])
    ours = O.f32_to_bf16(x)
    theirs = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, theirs)


# --------------------------------------------------------------- scatter_kv

@pytest.mark.parametrize("name", ["scatter_f32_to_f32", "scatter_f32_to_bf16",
                                  "scatter_bf16_to_bf16"])
def test_scatter_matches_reference_bit_exact(name):
    f = load(name + ".npz")
    src, pool = name.split("_")[1], name.split("_")[3]
    k = O.from_f32(f["k0"], pool)
    v = O.from_f32(f["v0"], pool)
    flat = O.flat_indices(f["table"], int(f["start"]), int(f["end"]), int(f["block_size"]))
    assert flat.tolist() == f["flat"].tolist()
    keys = O.from_f32(f["keys"], src)
    values = O.from_f32(f["values"], src)
    O.scatter_kv(k, v, int(f["layer"]), flat, keys, values, pool, src)
    assert np.array_equal(k, f["k_after"]), "key pool bytes differ from the reference"
    assert np.array_equal(v, f["v_after"])


def test_commit_matches_scatter_accepted_kv():
    f = load("commit.npz")
    for confirmed in (0, 1, 3, 5):
        k = f["k0"].copy()
        v = f["v0"].copy()
        for layer in range(k.shape[0]):
            row = int(f["row"])
            O.commit_accepted(k, v, layer, f["table"], int(f["ctx"]),
                              f[f"new_k_{layer}"][row:row + 1],
                              f[f"new_v_{layer}"][row:row + 1],
                              confirmed, int(f["block_size"]), "f32")
        assert np.array_equal(k, f[f"k_after_{confirmed}"])
        assert np.array_equal(v, f[f"v_after_{confirmed}"])


# ---------------------------------------------------------------- attention

VARLEN = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "varlen_*.npz")))


@pytest.mark.parametrize("name", VARLEN)
def test_varlen_matches_reference(name):
    f = load(name + ".npz")
    bs = int(f["block_size"])
    tables = [t[t >= 0] for t in f["tables"]]
    q = f["q"][0]
    got = O.varlen_attention(q, f["k0"], f["v0"], int(f["layer"]), tables,
                             f["seq_ids"].tolist(), f["positions"].tolist(), bs)
    for key in ("out_materialised", "out_blockwise", "out_reference"):
        want = f[key][0]
        assert np.allclose(got, want, atol=ATOL), (key, float(np.abs(got - want).max()))


@pytest.mark.parametrize("name", VARLEN)
def test_varlen_bf16_matches_reference(name):
    """bf16 storage, fp32 arithmetic on the rounded values, bf16 output."""
    f = load(name + ".npz")
    bs = int(f["block_size"])
    tables = [t[t >= 0] for t in f["tables"]]
    q = O.bf16_to_f32(O.f32_to_bf16(f["q"][0]))
    k = O.bf16_to_f32(O.f32_to_bf16(f["k0"]))
    v = O.bf16_to_f32(O.f32_to_bf16(f["v0"]))
    got = O.varlen_attention(q, k, v, int(f["layer"]), tables,
                             f["seq_ids"].tolist(), f["positions"].tolist(), bs)
    got_bf16 = O.f32_to_bf16(got)
    want = f["out_bf16"][0]
    # Same fp32 value rounded once: at most one bf16 ulp apart.
    diff = np.abs(O.bf16_to_f32(got_bf16) - O.bf16_to_f32(want))
    assert diff.max() <= 2 ** -7 * np.abs(O.bf16_to_f32(want)).max() + 1e-6


def test_blockwise_decode_matches_reference():
    f = load("blockwise.npz")
    bs = int(f["block_size"])
    for hq in (2, 4, 8):
        for ctx in (1, 5, 18, 20):
            q = f[f"q_{hq}_{ctx}"][0, :, 0, :]          # (H, D)
            got = O.varlen_attention(q[:, None, :], f["k0"], f["v0"], 0, [f["table"]],
                                     [0], [ctx - 1], bs)
            want = f[f"o_{hq}_{ctx}"][0, :, 0, :]
            assert np.allclose(got[:, 0, :], want, atol=ATOL), (hq, ctx)
    q = f["q_big"][0, :, 0, :]
    got = O.varlen_attention(q[:, None, :], f["k0"] * 50.0, f["v0"], 0, [f["table"]],
                             [0], [10], bs)
    assert np.isfinite(got).all()
    assert np.allclose(got[:, 0, :], f["o_big"][0, :, 0, :], atol=1e-4)


def test_config1_matches_reference():
    f = load("config1.npz")
    c = cases.config1(0)
    assert cases.checksum(c.q, c.k_pool, c.v_pool, c.tables, c.ctx_lens) == str(f["checksum"]), \
        "the seeded generator no longer reproduces the fixture's inputs"
    got = cases.oracle_decode(c)                           # (B, H, D)
    want = np.transpose(f["out_materialised"][0], (1, 0, 2))
    assert np.allclose(got, want, atol=ATOL)
    assert np.allclose(got, f["out_blockwise"], atol=ATOL)


def test_decode_attention_matches_varlen():
    c = cases.small_decode_case("x", 3, "f32", 8, 2, 32, [1, 17, 40])
    flat_k = c.k_pool.reshape(-1, c.num_kv_heads, c.head_dim)
    flat_v = c.v_pool.reshape(-1, c.num_kv_heads, c.head_dim)
    a = O.decode_attention(c.q, flat_k, flat_v, c.tables, c.ctx_lens, 16, c.scale)
    b = cases.oracle_decode(c)
    assert np.allclose(a, b, atol=ATOL)


def test_standalone_paged_attention_matches_reference():
    f = load("standalone.npz")
    for name in ("decode", "multi_query", "long"):
        got = O.standalone_paged_attention(
            f[f"{name}_q"], f[f"{name}_kcache"], f[f"{name}_vcache"],
            f[f"{name}_table"].tolist(), int(f[f"{name}_ctx"]))
        assert np.allclose(got, f[f"{name}_out"], atol=ATOL), name


def test_window_equals_writing_the_window_first():
    """The verify side buffer is equivalent to writing those keys into the pool."""
    c = cases.small_decode_case("w", 5, "f32", 10, 2, 32, [40, 70], q_per_seq=5)
    g = cases.rng(9)
    window = {}
    k_written = c.k_pool.copy()
    v_written = c.v_pool.copy()
    for s in range(c.batch):
        start = int(c.ctx_lens[s]) - 5
        kw = cases.normal(g, (2, 5, 32))
        vw = cases.normal(g, (2, 5, 32))
        window[s] = (start, kw, vw)
        flat = O.flat_indices(c.tables[s][c.tables[s] >= 0], start, start + 5, 16)
        kf = k_written.reshape(-1, 2, 32)
        vf = v_written.reshape(-1, 2, 32)
        kf[flat] = np.transpose(kw, (1, 0, 2))
        vf[flat] = np.transpose(vw, (1, 0, 2))
    a = cases.oracle_decode(c, window=window)
    c2 = cases.DecodeCase(**{**c.__dict__, "k_pool": k_written, "v_pool": v_written})
    b = cases.oracle_decode(c2)
    assert np.array_equal(a, b)


def test_oracle_rejects_like_the_reference():
    c = cases.small_decode_case("r", 1, "f32", 4, 2, 8, [8])
    q = np.zeros((4, 3, 8), np.float32)
    with pytest.raises(ValueError, match="query tokens but"):
        O.varlen_attention(q, c.k_pool[None], c.v_pool[None], 0, [c.tables[0]], [0, 0], [5, 6, 7], 16)
    with pytest.raises(ValueError, match="negative query position"):
        O.varlen_attention(q[:, :2], c.k_pool[None], c.v_pool[None], 0, [c.tables[0]], [0, 0], [3, -1], 16)
    with pytest.raises(IndexError, match="no block table"):
        O.varlen_attention(q[:, :2], c.k_pool[None], c.v_pool[None], 0, [c.tables[0]], [0, 3], [3, 3], 16)
    with pytest.raises(IndexError, match="block table has"):
        O.varlen_attention(q[:, :1], c.k_pool[None], c.v_pool[None], 0, [c.tables[0][:1]], [0], [40], 16)
    with pytest.raises(ValueError, match="not a multiple of"):
        O.varlen_attention(np.zeros((3, 1, 8), np.float32), c.k_pool[None], c.v_pool[None], 0,
                           [c.tables[0]], [0], [7], 16)


def test_acceptance_rule_matches_reference_verify_tokens(golden_dir):
    """accepted_drafts reproduces RejectionSampler.verify_tokens's accepted count from
    the uniforms it drew, and the token it drew afterwards has positive weight under
    the distribution next_token_after draws from."""
    f = np.load(os.path.join(golden_dir, "accept.npz"))
    K = f["draft"].shape[1]
    seen = set()
    for c in range(f["draft"].shape[0]):
        p, q = f["p"][c].astype(np.float64), f["q"][c].astype(np.float64)
        n = O.accepted_drafts(f["draft"][c], f["p"][c], f["q"][c], f["uniforms"][c])
        assert n == int(f["accepted"][c]), c
        seen.add(n)
        if n < K:
            w = np.maximum(p[n] - q[n], 0.0)
            if w.sum() == 0:
                w = p[n]
        else:
            w = p[K]
        assert w[int(f["last_token"][c])] > 0, c
        assert not bool(f["last_is_draft"][c])
    assert seen == set(range(K + 1))     # every outcome 0..K occurs


def test_greedy_acceptance_and_inverse_cdf_draw():
    assert O.accepted_drafts([3, 4, 9], target_tokens=[3, 4, 1, 7]) == 2
    assert O.accepted_drafts([3, 4], target_tokens=[3, 4, 8]) == 2
    assert O.accepted_drafts([5], target_tokens=[3, 1]) == 0
    w = np.array([0.0, 1.0, 0.0, 3.0])
    assert O.inverse_cdf_draw(w, 0.0) == 1
    assert O.inverse_cdf_draw(w, 0.24) == 1
    assert O.inverse_cdf_draw(w, 0.26) == 3
    assert O.inverse_cdf_draw(np.zeros(4), 0.5) is None
    p = np.array([[0.5, 0.5, 0.0], [0.0, 0.0, 1.0]])
    q = np.array([[0.5, 0.5, 0.0]])
    # rejection at 0 with p == q: the difference is all zero, so the draw is from p
    assert O.next_token_after(0, 1, p, q, 0.75) == 1
    assert O.next_token_after(1, 1, p, q, 0.1) == 2
