"""
Fused speculative accept + commit (``mf_accept_commit``) against the oracle's
restatement of ``RejectionSampler.verify_tokens`` (pinned to the reference's
own draws in ``tests/golden/accept.npz``) and of ``scatter_accepted_kv``:

* the accepted counts are exact (integer decisions given the uniforms);
* the next token is the oracle's inverse-CDF draw (a draw that lands within
  float rounding of a CDF step may pick the neighbour; the test then checks the
  step instead);
* the pool after the commit is bit-exact, rejected slots untouched, in every
  layer; a sequence whose prefix leaves its table writes nothing.
"""

import os

import numpy as np
import pytest
import torch

from oracle import paged_oracle as O
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

SP = pytest.importorskip("memforge_b200.speculative")
K_ = pytest.importorskip("memforge_b200._kernels")


def _draw_ok(weights, u, tok, want):
    """tok equals the oracle's draw, or sits at a CDF step within rounding of u."""
    if tok == want:
        return True
    w = np.maximum(np.asarray(weights, np.float64), 0)
    c = np.cumsum(w)
    t = u * c[-1]
    lo = c[tok - 1] if tok > 0 else 0.0
    return w[tok] > 0 and lo - 1e-5 * c[-1] <= t <= c[tok] + 1e-5 * c[-1]


def test_sampling_decision_matches_the_reference_sampler():
    f = np.load(os.path.join(GOLDEN, "accept.npz"))
    B, K = f["draft"].shape
    g = np.random.default_rng(3)
    ru = g.random(B).astype(np.float32)
    dev = "cuda"
    n, nxt = SP.accept_and_commit(torch.from_numpy(f["draft"]).to(dev),
                                  target_probs=torch.from_numpy(f["p"]).to(dev),
                                  draft_probs=torch.from_numpy(f["q"]).to(dev),
                                  uniforms=torch.from_numpy(f["uniforms"]).to(dev),
                                  resample_uniform=torch.from_numpy(ru).to(dev))
    torch.cuda.synchronize()
    n, nxt = n.cpu().numpy(), nxt.cpu().numpy()
    assert np.array_equal(n, f["accepted"]), "accepted counts differ from the reference's"
    for b in range(B):
        want = O.next_token_after(int(n[b]), K, f["p"][b], f["q"][b], float(ru[b]))
        if n[b] < K:
            w = np.maximum(f["p"][b][n[b]].astype(np.float64) - f["q"][b][n[b]], 0)
            if w.sum() == 0:
                w = f["p"][b][n[b]]
        else:
            w = f["p"][b][K]
        assert _draw_ok(w, float(ru[b]), int(nxt[b]), want), b


def test_large_vocabulary_draw():
    """Qwen2.5's 152064-token vocabulary: the block-wide inverse CDF."""
    g = np.random.default_rng(8)
    B, K, V = 6, 4, 152064
    p = g.dirichlet(np.ones(V) * 0.05, size=(B, K + 1)).astype(np.float32)
    q = g.dirichlet(np.ones(V) * 0.05, size=(B, K)).astype(np.float32)
    draft = np.array([[g.choice(V, p=q[b, i] / q[b, i].sum()) for i in range(K)]
                      for b in range(B)], np.int32)
    un = g.random((B, K)).astype(np.float32)
    un[0] = 0.0                    # sequence 0 accepts every draft: the bonus draw
    ru = g.random(B).astype(np.float32)
    t = lambda x: torch.from_numpy(x).cuda()
    n, nxt = SP.accept_and_commit(t(draft), target_probs=t(p), draft_probs=t(q), uniforms=t(un),
                                  resample_uniform=t(ru))
    n, nxt = n.cpu().numpy(), nxt.cpu().numpy()
    assert n[0] == K
    for b in range(B):
        want_n = O.accepted_drafts(draft[b], p[b], q[b], un[b])
        assert n[b] == want_n
        want = O.next_token_after(want_n, K, p[b], q[b], float(ru[b]))
        w = p[b][K] if want_n == K else np.maximum(p[b][want_n].astype(np.float64) - q[b][want_n], 0)
        assert _draw_ok(w, float(ru[b]), int(nxt[b]), want), b


def _pool_case(seed, B, W, L, H=2, D=128, width=6, dtype=torch.bfloat16):
    g = torch.Generator(device="cuda").manual_seed(seed)
    NB = B * width + 3
    kp = torch.randn((L, NB, 16, H, D), generator=g, device="cuda").to(dtype)
    vp = torch.randn_like(kp)
    wk = torch.randn((L, B * W, H, D), generator=g, device="cuda").to(dtype)
    wv = torch.randn_like(wk)
    perm = np.random.default_rng(seed).permutation(NB)[:B * width].reshape(B, width)
    return kp, vp, wk, wv, perm.astype(np.int32)


def _bits(t):
    return t.cpu().view(torch.int16 if t.element_size() == 2 else torch.int32).numpy()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_greedy_round_commits_the_confirmed_prefix_bit_exact(dtype):
    B, K, L = 9, 4, 3
    W = K + 1
    g = np.random.default_rng(4)
    target = g.integers(0, 50, size=(B, W)).astype(np.int32)
    draft = target[:, :K].copy()
    for b in range(B):           # sequence b disagrees at slot b % (K+1) (K+1: all agree)
        if b % W < K:
            draft[b, b % W] = (draft[b, b % W] + 1) % 50
    ctx = np.array([0, 15, 16, 30, 47, 60, 5, 31, 64], np.int32)
    kp, vp, wk, wv, tables = _pool_case(11, B, W, L, dtype=dtype)
    want_k, want_v = _bits(kp)[None].copy(), _bits(vp)[None].copy()
    n, nxt = SP.accept_and_commit(torch.from_numpy(draft).cuda(),
                                  target_tokens=torch.from_numpy(target).cuda(),
                                  win_k=wk, win_v=wv, key_pool=kp, value_pool=vp,
                                  block_tables=torch.from_numpy(tables).cuda(),
                                  ctx_lens=torch.from_numpy(ctx).cuda())
    torch.cuda.synchronize()
    K_.check_device_errors(kp.device)
    n, nxt = n.cpu().numpy(), nxt.cpu().numpy()
    wkb, wvb = _bits(wk), _bits(wv)
    st = "bf16" if dtype == torch.bfloat16 else "f32"
    for b in range(B):
        a = O.accepted_drafts(draft[b], target_tokens=target[b])
        assert n[b] == a == (b % W)
        assert nxt[b] == target[b, a]
        for l in range(L):
            wl_k = np.transpose(wkb[l, b * W:(b + 1) * W], (1, 0, 2))[None]
            wl_v = np.transpose(wvb[l, b * W:(b + 1) * W], (1, 0, 2))[None]
            O.commit_accepted(want_k[0], want_v[0], l, tables[b], int(ctx[b]), wl_k, wl_v,
                              a + 1, 16, st)
    assert np.array_equal(_bits(kp), want_k[0])
    assert np.array_equal(_bits(vp), want_v[0])


def test_decision_only_and_bad_table_writes_nothing():
    B, K, L = 3, 4, 2
    W = K + 1
    target = np.tile(np.arange(W, dtype=np.int32), (B, 1))
    draft = target[:, :K].copy()
    kp, vp, wk, wv, tables = _pool_case(12, B, W, L, width=2)
    ctx = np.array([3, 29, 10], np.int32)          # sequence 1: 29 + 4 > 2 pages
    before_k = kp.clone()
    tt = torch.from_numpy(target).cuda()
    n, nxt = SP.accept_and_commit(torch.from_numpy(draft).cuda(), target_tokens=tt)
    assert n.tolist() == [K] * B and nxt.tolist() == [K] * B
    assert torch.equal(kp, before_k)
    SP.accept_and_commit(torch.from_numpy(draft).cuda(), target_tokens=tt, win_k=wk, win_v=wv,
                         key_pool=kp, value_pool=vp, block_tables=torch.from_numpy(tables).cuda(),
                         ctx_lens=torch.from_numpy(ctx).cuda())
    with pytest.raises(IndexError, match="block table"):
        K_.check_device_errors(kp.device)
    # sequence 1 wrote nothing; 0 and 2 wrote their 5 rows
    want = before_k.clone()
    for b in (0, 2):
        for j in range(W):
            pos = int(ctx[b]) + j
            want[:, tables[b][pos // 16], pos % 16] = wk[:, b * W + j]
    assert torch.equal(kp, want)
