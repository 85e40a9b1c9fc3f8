"""
Speculative verify + commit (BASELINE config 4 semantics) on the GPU:
* the commit writes only the confirmed prefix, bit-exact against the
  reference's scatter_accepted_kv (golden pools) and the oracle;
* verify over a side window equals attention over the pool with the window
  written into it, and rejected drafts never reach the pool.
"""

import os

import numpy as np
import pytest
import torch

from oracle import paged_oracle as O
from tests import cases
from tests.conftest import GOLDEN
from tests.gpu_util import assert_close, to_dev, to_np32

pytestmark = pytest.mark.gpu


def test_scatter_accepted_kv_matches_reference_golden():
    from memforge_b200.kv_pool import ModelKVSpec, PagedKVPool
    from memforge_b200.speculative import scatter_accepted_kv
    f = np.load(os.path.join(GOLDEN, "commit.npz"))
    L, NB, BS, H, D = f["k0"].shape
    spec = ModelKVSpec(num_layers=L, num_kv_heads=H, head_dim=D, dtype=torch.float32, device="cuda")
    for confirmed in (0, 1, 3, 5):
        pool = PagedKVPool(spec, num_blocks=NB, block_size=BS)
        pool.key_pool.copy_(torch.from_numpy(f["k0"]))
        pool.value_pool.copy_(torch.from_numpy(f["v0"]))
        new_kv = [(torch.from_numpy(f[f"new_k_{l}"]).cuda(), torch.from_numpy(f[f"new_v_{l}"]).cuda())
                  for l in range(L)]
        scatter_accepted_kv(pool, torch.from_numpy(f["table"]).cuda(), int(f["ctx"]), new_kv,
                            int(f["row"]), confirmed)
        torch.cuda.synchronize()
        assert np.array_equal(pool.key_pool.cpu().numpy(), f[f"k_after_{confirmed}"]), confirmed
        assert np.array_equal(pool.value_pool.cpu().numpy(), f[f"v_after_{confirmed}"]), confirmed


def test_verify_then_commit_round_trip():
    from memforge_b200.speculative import commit_accepted, verify_attention
    W, Hq, Hkv, D = 5, 40, 8, 128
    ctx = [700, 33, 2048, 16, 5000]
    c = cases.small_decode_case("spec", 31, "bf16", Hq, Hkv, D, [n + W for n in ctx], q_per_seq=W)
    g = cases.rng(32)
    B = len(ctx)
    win_k = cases.bf16_round(cases.normal(g, (B * W, Hkv, D)))
    win_v = cases.bf16_round(cases.normal(g, (B * W, Hkv, D)))
    accepted = np.array([0, 4, 2, 3, 1], np.int32)
    kp, vp = to_dev(c.k_pool, "bf16"), to_dev(c.v_pool, "bf16")
    before_k = kp.clone()
    tables = torch.from_numpy(c.tables.clip(min=0)).cuda()
    ctx_t = torch.tensor(ctx, dtype=torch.int32, device="cuda")
    out = verify_attention(to_dev(c.q, "bf16"), to_dev(win_k, "bf16"), to_dev(win_v, "bf16"), kp, vp,
                           tables, ctx_t)
    torch.cuda.synchronize()
    # verify must not have touched the pool
    assert torch.equal(kp, before_k)
    window = {s: (ctx[s], np.transpose(win_k[s * W:(s + 1) * W], (1, 0, 2)),
                  np.transpose(win_v[s * W:(s + 1) * W], (1, 0, 2))) for s in range(B)}
    assert_close(to_np32(out), cases.oracle_decode(c, window=window), "bf16", "verify")
    # commit the confirmed prefix (accepted + 1 tokens)
    commit_accepted(kp, vp, to_dev(win_k, "bf16"), to_dev(win_v, "bf16"), tables, ctx_t,
                    torch.from_numpy(accepted + 1).cuda())
    torch.cuda.synchronize()
    want_k = O.f32_to_bf16(c.k_pool)[None]
    want_v = O.f32_to_bf16(c.v_pool)[None]
    for s in range(B):
        t = c.tables[s][c.tables[s] >= 0]
        O.commit_accepted(want_k, want_v, 0, t, ctx[s],
                          O.f32_to_bf16(np.transpose(win_k[s * W:(s + 1) * W], (1, 0, 2)))[None],
                          O.f32_to_bf16(np.transpose(win_v[s * W:(s + 1) * W], (1, 0, 2)))[None],
                          int(accepted[s]) + 1, 16, "bf16")
    got_k = kp.cpu().view(torch.int16).numpy().view(np.uint16)
    got_v = vp.cpu().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got_k, want_k[0]), "pool after commit differs from the reference commit"
    assert np.array_equal(got_v, want_v[0])


def _commit_case(seed, ctx, W, H=2, D=64, width=6):
    """Pool, disjoint block tables (no slot is named twice) and fp32 windows."""
    g = np.random.default_rng(seed)
    B = len(ctx)
    NB = B * width + 4
    kp0 = g.standard_normal((NB, 16, H, D)).astype(np.float32)
    vp0 = g.standard_normal((NB, 16, H, D)).astype(np.float32)
    tables = g.permutation(NB)[:B * width].reshape(B, width).astype(np.int32)
    wk = g.standard_normal((B * W, H, D)).astype(np.float32)
    wv = g.standard_normal((B * W, H, D)).astype(np.float32)
    return kp0, vp0, tables, wk, wv


def _oracle_commit(kp0, vp0, tables, ctx, wk, wv, conf, W, src, pool):
    want_k = O.from_f32(kp0, pool)[None].copy()
    want_v = O.from_f32(vp0, pool)[None].copy()
    for s, n in enumerate(conf):
        k = O.from_f32(np.transpose(wk[s * W:(s + 1) * W], (1, 0, 2)), src)[None]
        v = O.from_f32(np.transpose(wv[s * W:(s + 1) * W], (1, 0, 2)), src)[None]
        if n <= 0:
            continue
        flat = O.flat_indices(tables[s], ctx[s], ctx[s] + n, 16)
        O.scatter_kv(want_k, want_v, 0, flat, k[:, :, :n], v[:, :, :n], pool, src)
    return want_k[0], want_v[0]


def _bits(t):
    if t.dtype == torch.float32:
        return t.cpu().view(torch.int32).numpy()
    return t.cpu().view(torch.int16).numpy()


def _want_bits(a, dt):
    return a.view(np.int32) if dt == "f32" else a.view(np.int16)


@pytest.mark.parametrize("src,pool", [("bf16", "bf16"), ("f16", "f16"), ("f32", "f32"),
                                      ("f32", "bf16")])
def test_commit_window_bit_exact_with_page_crossings(src, pool):
    """One launch commits each window's confirmed prefix (0..W rows, across page
    boundaries); the rejected rows' slots keep their old bytes."""
    from memforge_b200 import _kernels as K
    W = 5
    ctx = [0, 13, 15, 16, 30, 47, 60]
    conf = [1, 5, 3, 0, 4, 5, 2]
    kp0, vp0, tables, wk, wv = _commit_case(40, ctx, W)
    # torch's fp32 -> bf16/f16 casts round to nearest even, like the oracle's
    kp, vp = to_dev(kp0, pool), to_dev(vp0, pool)
    dk, dv = to_dev(wk, src), to_dev(wv, src)
    K.commit_window(dk, dv, kp, vp, torch.from_numpy(tables).cuda(),
                    torch.tensor(ctx, dtype=torch.int32, device="cuda"),
                    torch.tensor(conf, dtype=torch.int32, device="cuda"))
    K.check_device_errors(kp.device)
    want_k, want_v = _oracle_commit(kp0, vp0, tables, ctx, wk, wv, conf, W, src, pool)
    assert np.array_equal(_bits(kp), _want_bits(want_k, pool))
    assert np.array_equal(_bits(vp), _want_bits(want_v, pool))


def test_commit_window_errors_skip_whole_sequences_and_set_bits():
    """A sequence the reference would reject (IndexError from slot_indices before
    the first write) writes nothing; a confirmed count <= 0 is a silent no-op."""
    from memforge_b200 import _kernels as K
    W, width = 4, 2
    ctx = [30, 5, 5, 5, 5, 5]
    # seq 0 crosses past its 2-page table; seq 1 confirms more than W; seq 3
    # names a block outside the pool; seqs 4 and 5 confirm nothing
    conf = [4, 5, 2, 1, 0, -2]
    kp0, vp0, tables, wk, wv = _commit_case(41, ctx, W, width=width)
    tables[3, 0] = 999
    kp, vp = to_dev(kp0, "bf16"), to_dev(vp0, "bf16")
    dk, dv = to_dev(wk, "bf16"), to_dev(wv, "bf16")
    K.commit_window(dk, dv, kp, vp, torch.from_numpy(tables).cuda(),
                    torch.tensor(ctx, dtype=torch.int32, device="cuda"),
                    torch.tensor(conf, dtype=torch.int32, device="cuda"))
    bits = int(K.err_word(kp.device).item())
    with pytest.raises(IndexError):
        K.check_device_errors(kp.device)
    assert bits == 0x1 | 0x4 | 0x8, hex(bits)
    # Only seq 2's confirmed rows land; seq 0's in-table positions 30, 31 stay untouched.
    want_k, want_v = _oracle_commit(kp0, vp0, tables, ctx, wk, wv, [0, 0, 2, 0, 0, 0], W,
                                    "bf16", "bf16")
    assert np.array_equal(_bits(kp), _want_bits(want_k, "bf16"))
    assert np.array_equal(_bits(vp), _want_bits(want_v, "bf16"))


def test_commit_window_nothing_confirmed_is_silent():
    from memforge_b200 import _kernels as K
    W = 5
    ctx = [7, 40]
    kp0, vp0, tables, wk, wv = _commit_case(42, ctx, W)
    kp, vp = to_dev(kp0, "bf16"), to_dev(vp0, "bf16")
    before = kp.clone()
    K.commit_window(to_dev(wk, "bf16"), to_dev(wv, "bf16"), kp, vp,
                    torch.from_numpy(tables).cuda(),
                    torch.tensor(ctx, dtype=torch.int32, device="cuda"),
                    torch.tensor([0, -1], dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    assert int(K.err_word(kp.device).item()) == 0
    assert torch.equal(kp, before)


def test_commit_window_all_layers_in_one_launch():
    """(L, B*W, H, D) windows into an (L, blocks, 16, H, D) pool: every layer's
    confirmed rows land, bit-exact, with one launch."""
    from memforge_b200 import _kernels as K
    from memforge_b200.speculative import commit_accepted
    W, L_ = 5, 3
    ctx = [7, 16, 40, 63]
    conf = [5, 0, 2, 1]
    layers = [_commit_case(50 + l, ctx, W) for l in range(L_)]
    tables = layers[0][2]
    kp = torch.stack([to_dev(c[0], "bf16") for c in layers])
    vp = torch.stack([to_dev(c[1], "bf16") for c in layers])
    wk = torch.stack([to_dev(c[3], "bf16") for c in layers])
    wv = torch.stack([to_dev(c[4], "bf16") for c in layers])
    before = K.launch_counter["commit_window"]
    commit_accepted(kp, vp, wk, wv, torch.from_numpy(tables).cuda(),
                    torch.tensor(ctx, dtype=torch.int32, device="cuda"),
                    torch.tensor(conf, dtype=torch.int32, device="cuda"))
    K.check_device_errors(kp.device)
    assert K.launch_counter["commit_window"] == before + 1
    for l, c in enumerate(layers):
        want_k, want_v = _oracle_commit(c[0], c[1], tables, ctx, c[3], c[4], conf, W, "bf16",
                                        "bf16")
        assert np.array_equal(_bits(kp[l]), _want_bits(want_k, "bf16")), l
        assert np.array_equal(_bits(vp[l]), _want_bits(want_v, "bf16")), l
