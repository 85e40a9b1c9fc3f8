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
