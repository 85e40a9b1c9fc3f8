"""
The reference's operator seams, served by the sm_100a kernels, checked against
the reference's golden outputs and its own test cases (ported from
tests/python/test_varlen_attention.py, test_block_attention.py,
test_triton_paged_decode.py, test_paged_attention.py in MemForge).
"""

import glob
import math
import os
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import paged_oracle as O
from tests.conftest import GOLDEN
from tests.gpu_util import assert_close

pytestmark = pytest.mark.gpu

ATOL = 1e-5
VARLEN = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "varlen_*.npz")))


def load(name):
    return np.load(os.path.join(GOLDEN, name))


def golden_pool(f, dtype=torch.float32):
    from memforge_b200.kv_pool import ModelKVSpec, PagedKVPool
    L, NB, BS, H, D = f["k0"].shape
    spec = ModelKVSpec(num_layers=L, num_kv_heads=H, head_dim=D, dtype=dtype, device="cuda")
    pool = PagedKVPool(spec, num_blocks=NB, block_size=BS)
    pool.key_pool.copy_(torch.from_numpy(f["k0"]))
    pool.value_pool.copy_(torch.from_numpy(f["v0"]))
    return pool


# ------------------------------------------------------------ varlen seam

@pytest.mark.parametrize("name", VARLEN)
def test_varlen_matches_reference_golden(name):
    from memforge_b200.varlen_attention import (paged_attention_varlen,
                                                paged_attention_varlen_materialised)
    f = load(name + ".npz")
    pool = golden_pool(f)
    tables = [torch.from_numpy(t[t >= 0].astype(np.int64)) for t in f["tables"]]
    q = torch.from_numpy(f["q"]).cuda()
    sid, pos = f["seq_ids"].tolist(), f["positions"].tolist()
    a = paged_attention_varlen(q, pool.key_pool, pool.value_pool, int(f["layer"]), tables, sid,
                               pos, int(f["block_size"]))
    b = paged_attention_varlen_materialised(q, pool, int(f["layer"]), tables, sid, pos)
    for got in (a, b):
        assert got.shape == q.shape and got.dtype == q.dtype
        assert np.allclose(got.cpu().numpy(), f["out_materialised"], atol=ATOL)
        assert np.allclose(got.cpu().numpy(), f["out_reference"], atol=ATOL)


@pytest.mark.parametrize("name", VARLEN)
def test_varlen_bf16_matches_reference_golden(name):
    from memforge_b200.varlen_attention import paged_attention_varlen_materialised
    f = load(name + ".npz")
    pool = golden_pool(f, torch.bfloat16)
    tables = [torch.from_numpy(t[t >= 0].astype(np.int64)) for t in f["tables"]]
    q = torch.from_numpy(f["q"]).to(torch.bfloat16).cuda()
    got = paged_attention_varlen_materialised(q, pool, int(f["layer"]), tables,
                                              f["seq_ids"].tolist(), f["positions"].tolist())
    want = O.bf16_to_f32(f["out_bf16"])
    assert_close(got.float().cpu().numpy(), want, "bf16", name)


def _small_pool(num_blocks=96, layers=2, kv_heads=2, head_dim=8, seed=0, block=4):
    from memforge_b200.kv_pool import ModelKVSpec, PagedKVPool
    spec = ModelKVSpec(num_layers=layers, num_kv_heads=kv_heads, head_dim=head_dim,
                       dtype=torch.float32, device="cuda")
    pool = PagedKVPool(spec, num_blocks=num_blocks, block_size=block)
    g = torch.Generator(device="cuda").manual_seed(seed)
    pool.key_pool.normal_(generator=g)
    pool.value_pool.normal_(generator=g)
    return pool


def _tables(lengths, block=4):
    out, nxt = [], 0
    for n in lengths:
        k = (n + block - 1) // block
        out.append(torch.arange(nxt, nxt + k))
        nxt += k
    return out


def test_a_token_cannot_see_later_positions():
    """test_varlen_attention.py:236-274, by perturbation."""
    from memforge_b200.varlen_attention import paged_attention_varlen
    pool = _small_pool()
    tables = _tables([10])
    q = torch.randn(1, 4, 10, 8, device="cuda")
    sid, pos = [0] * 10, list(range(10))
    before = paged_attention_varlen(q, pool.key_pool, pool.value_pool, 0, tables, sid, pos, 4)
    phys = int(tables[0][7 // 4])
    pool.key_pool[0, phys, 7 % 4] += 5.0
    pool.value_pool[0, phys, 7 % 4] += 5.0
    after = paged_attention_varlen(q, pool.key_pool, pool.value_pool, 0, tables, sid, pos, 4)
    for row in range(7):
        assert torch.equal(before[:, :, row], after[:, :, row]), row
    for row in range(7, 10):
        assert not torch.equal(before[:, :, row], after[:, :, row]), row


def test_one_sequence_cannot_see_another():
    from memforge_b200.varlen_attention import paged_attention_varlen
    pool = _small_pool()
    tables = _tables([8, 8])
    q = torch.randn(1, 4, 2, 8, device="cuda")
    before = paged_attention_varlen(q, pool.key_pool, pool.value_pool, 0, tables, [0, 1], [7, 7], 4)
    for b in tables[1].tolist():
        pool.key_pool[0, b] += 3.0
        pool.value_pool[0, b] += 3.0
    after = paged_attention_varlen(q, pool.key_pool, pool.value_pool, 0, tables, [0, 1], [7, 7], 4)
    assert torch.equal(before[:, :, 0], after[:, :, 0])
    assert not torch.equal(before[:, :, 1], after[:, :, 1])


def test_interleaved_packing_order_does_not_matter():
    from memforge_b200.varlen_attention import paged_attention_varlen
    pool = _small_pool()
    tables = _tables([12, 6, 20])
    sid, pos = [0, 0, 0, 1, 2], [9, 10, 11, 5, 19]
    q = torch.randn(1, 4, 5, 8, device="cuda")
    straight = paged_attention_varlen(q, pool.key_pool, pool.value_pool, 0, tables, sid, pos, 4)
    order = [3, 0, 4, 2, 1]
    shuffled = paged_attention_varlen(q[:, :, order].contiguous(), pool.key_pool, pool.value_pool,
                                      0, tables, [sid[i] for i in order], [pos[i] for i in order], 4)
    for new, old in enumerate(order):
        assert torch.allclose(shuffled[:, :, new], straight[:, :, old], atol=ATOL)


def test_each_layer_reads_its_own_slice():
    from memforge_b200.varlen_attention import paged_attention_varlen
    pool = _small_pool(layers=3)
    tables = _tables([9])
    q = torch.randn(1, 4, 2, 8, device="cuda")
    outs = [paged_attention_varlen(q, pool.key_pool, pool.value_pool, l, tables, [0, 0], [7, 8], 4)
            for l in range(3)]
    assert not torch.allclose(outs[0], outs[1], atol=1e-4)
    assert not torch.allclose(outs[1], outs[2], atol=1e-4)


def test_varlen_with_device_tables_is_graph_capturable():
    """The seam reads device tables on the device: after one warm-up call a CUDA
    graph of it replays with new table contents, pool values and queries."""
    from memforge_b200.varlen_attention import paged_attention_varlen
    pool = _small_pool(block=16, head_dim=64, num_blocks=64, kv_heads=2)
    tabs = [t.cuda() for t in _tables([70, 33, 120], block=16)]
    sid = [0, 0, 0, 1, 2, 2]
    pos = [66, 67, 68, 32, 100, 101]
    q = torch.randn(1, 4, 6, 64, device="cuda")
    paged_attention_varlen(q, pool.key_pool, pool.value_pool, 1, tabs, sid, pos, 16)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            out = paged_attention_varlen(q, pool.key_pool, pool.value_pool, 1, tabs, sid, pos, 16)
    torch.cuda.current_stream().wait_stream(s)
    for trial in range(3):
        q.normal_()
        pool.key_pool[1].normal_()
        tabs[1].copy_(torch.randperm(64, device="cuda")[:tabs[1].numel()])
        g.replay()
        want = paged_attention_varlen(q, pool.key_pool, pool.value_pool, 1, tabs, sid, pos, 16)
        torch.cuda.synchronize()
        assert torch.allclose(out, want, atol=ATOL), trial


def test_varlen_metadata_is_uploaded_once_per_pass():
    """Every layer of a pass reuses the plan: no host work beyond the first layer's."""
    from memforge_b200 import varlen_attention as V
    pool = _small_pool(block=4)
    tabs = [t.cuda() for t in _tables([13, 6, 20])]
    sid, pos = [0, 0, 1, 2], [11, 12, 5, 19]
    q = torch.randn(1, 4, 4, 8, device="cuda")
    V._memo.clear()
    for layer in range(2):
        V.paged_attention_varlen(q, pool.key_pool, pool.value_pool, layer, tabs, sid, pos, 4)
    assert len(V._memo) == 1


def test_varlen_validation_matches_reference():
    from memforge_b200.varlen_attention import paged_attention_varlen
    pool = _small_pool()
    tables = _tables([8])
    kp, vp = pool.key_pool, pool.value_pool
    with pytest.raises(ValueError, match="query tokens but"):
        paged_attention_varlen(torch.zeros(1, 4, 3, 8, device="cuda"), kp, vp, 0, tables, [0, 0], [5, 6, 7], 4)
    with pytest.raises(ValueError, match="at least one query token"):
        paged_attention_varlen(torch.zeros(1, 4, 0, 8, device="cuda"), kp, vp, 0, tables, [], [], 4)
    with pytest.raises(ValueError, match="negative query position"):
        paged_attention_varlen(torch.zeros(1, 4, 2, 8, device="cuda"), kp, vp, 0, tables, [0, 0], [3, -1], 4)
    with pytest.raises(IndexError, match="no block table"):
        paged_attention_varlen(torch.zeros(1, 4, 2, 8, device="cuda"), kp, vp, 0, tables, [0, 3], [3, 3], 4)
    with pytest.raises(IndexError, match="block table has"):
        paged_attention_varlen(torch.zeros(1, 4, 1, 8, device="cuda"), kp, vp, 0, tables, [0], [40], 4)
    with pytest.raises(ValueError, match="not a multiple of"):
        paged_attention_varlen(torch.zeros(1, 3, 1, 8, device="cuda"), kp, vp, 0, tables, [0], [7], 4)


# --------------------------------------------------------- blockwise seam

def test_blockwise_matches_reference_golden():
    from memforge_b200.block_attention import paged_attention_blockwise
    f = load("blockwise.npz")
    pool = golden_pool(f)
    table = torch.from_numpy(f["table"])
    for hq in (2, 4, 8):
        for ctx in (1, 5, 18, 20):
            q = torch.from_numpy(f[f"q_{hq}_{ctx}"]).cuda()
            got = paged_attention_blockwise(q, pool.key_pool, pool.value_pool, 0, table, ctx, 4)
            assert np.allclose(got.cpu().numpy(), f[f"o_{hq}_{ctx}"], atol=ATOL), (hq, ctx)
    q = torch.from_numpy(f["q_big"]).cuda()
    got = paged_attention_blockwise(q, pool.key_pool * 50.0, pool.value_pool, 0, table, 11, 4)
    assert torch.isfinite(got).all()
    assert np.allclose(got.cpu().numpy(), f["o_big"], atol=1e-4)


def test_blockwise_rejects_bad_inputs():
    from memforge_b200.block_attention import paged_attention_blockwise
    pool = _small_pool()
    table = torch.tensor([0, 1])
    q = torch.randn(1, 2, 1, 8, device="cuda")
    kp, vp = pool.key_pool, pool.value_pool
    with pytest.raises(ValueError, match="single query position"):
        paged_attention_blockwise(torch.randn(1, 2, 3, 8, device="cuda"), kp, vp, 0, table, 5, 4)
    with pytest.raises(ValueError, match="context_length must be positive"):
        paged_attention_blockwise(q, kp, vp, 0, table, 0, 4)
    with pytest.raises(ValueError, match="not a multiple"):
        paged_attention_blockwise(torch.randn(1, 5, 1, 8, device="cuda"), kp, vp, 0, table, 5, 4)
    with pytest.raises(IndexError, match="block table has"):
        paged_attention_blockwise(q, kp, vp, 0, torch.tensor([0]), 20, 4)


# ---------------------------------------------- Triton-signature decode seam

def _decode_reference(q, kflat, vflat, tables, ctx, bs, scale):
    """tests/python/test_triton_paged_decode.py:10-25."""
    B, Hq, D = q.shape
    Hkv = kflat.shape[1]
    G = Hq // Hkv
    outs = []
    for b in range(B):
        n = int(ctx[b])
        pos = torch.arange(n, device=q.device)
        slots = tables[b][pos // bs] * bs + pos % bs
        k = kflat[slots].float()
        v = vflat[slots].float()
        qb = q[b].float().view(Hkv, G, D)
        p = torch.softmax(torch.einsum("hgd,nhd->hgn", qb, k) * scale, -1)
        outs.append(torch.einsum("hgn,nhd->hgd", p, v).reshape(Hq, D))
    return torch.stack(outs)


def _decode_case(B, Hq, Hkv, D, bs, ctxs, dtype, seed=0):
    from memforge_b200.paged_decode import paged_decode_attention
    g = torch.Generator(device="cuda").manual_seed(seed)
    nblocks = 4 + sum((c + bs - 1) // bs for c in ctxs) + 8
    kflat = torch.randn(nblocks * bs, Hkv, D, device="cuda", dtype=dtype, generator=g)
    vflat = torch.randn_like(kflat)
    q = torch.randn(B, Hq, D, device="cuda", dtype=dtype, generator=g)
    maxb = max((c + bs - 1) // bs for c in ctxs) + 2
    perm = torch.randperm(nblocks, device="cuda", generator=g)
    tables = torch.zeros(B, maxb, dtype=torch.long, device="cuda")
    i = 0
    for b, c in enumerate(ctxs):
        n = (c + bs - 1) // bs
        tables[b, :n] = perm[i:i + n]
        i += n
    ctx = torch.tensor(ctxs, device="cuda", dtype=torch.long)
    scale = D ** -0.5
    out = paged_decode_attention(q, kflat, vflat, tables, ctx, bs, max(ctxs), scale)
    return out.float(), _decode_reference(q, kflat, vflat, tables, ctx, bs, scale)


@pytest.mark.parametrize("dtype,tol", [(torch.float16, 2e-3), (torch.bfloat16, 2e-2)])
@pytest.mark.parametrize("Hq,Hkv", [(8, 8), (16, 4), (28, 4), (32, 8)])
def test_decode_matches_triton_reference(Hq, Hkv, dtype, tol):
    out, ref = _decode_case(3, Hq, Hkv, 128, 16, [1, 77, 300], dtype)
    assert (out - ref).abs().max().item() < tol


def test_decode_ragged_lengths_and_tile_boundaries():
    for ctxs in ([1], [63, 64, 65], [2048, 5], [129, 128, 127, 16]):
        out, ref = _decode_case(len(ctxs), 16, 4, 128, 16, ctxs, torch.float16)
        assert (out - ref).abs().max().item() < 2e-3, ctxs


def test_decode_ignores_garbage_beyond_context():
    from memforge_b200.paged_decode import paged_decode_attention
    torch.manual_seed(1)
    bs = 16
    kflat = torch.randn(64 * bs, 4, 128, device="cuda", dtype=torch.float16)
    vflat = torch.randn_like(kflat)
    q = torch.randn(1, 16, 128, device="cuda", dtype=torch.float16)
    tbl = torch.arange(8, device="cuda").view(1, 8)
    ctx = torch.tensor([40], device="cuda")
    a = paged_decode_attention(q, kflat, vflat, tbl, ctx, bs, 128, 128 ** -0.5)
    kflat[40:128] = 1e4
    vflat[40:128] = -1e4
    b = paged_decode_attention(q, kflat, vflat, tbl, ctx, bs, 128, 128 ** -0.5)
    assert torch.equal(a, b)


def test_decode_context_length_is_a_runtime_value_in_a_cuda_graph():
    from memforge_b200.paged_decode import paged_decode_attention
    bs, D = 16, 128
    kflat = torch.randn(64 * bs, 4, D, device="cuda", dtype=torch.float16)
    vflat = torch.randn_like(kflat)
    q = torch.randn(2, 16, D, device="cuda", dtype=torch.float16)
    tbl = torch.arange(16, device="cuda").repeat(2, 1)
    ctx = torch.tensor([10, 200], device="cuda")
    out = torch.empty(2, 16, D, device="cuda", dtype=torch.float16)
    paged_decode_attention(q, kflat, vflat, tbl, ctx, bs, 256, D ** -0.5, out=out)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        paged_decode_attention(q, kflat, vflat, tbl, ctx, bs, 256, D ** -0.5, out=out)
    for lens in ([10, 200], [255, 1], [64, 64]):
        ctx.copy_(torch.tensor(lens))
        g.replay()
        ref = _decode_reference(q, kflat, vflat, tbl, ctx, bs, D ** -0.5)
        assert (out.float() - ref).abs().max().item() < 2e-3, lens


# ------------------------------------------------------ standalone operator

def test_standalone_paged_attention_matches_reference_golden():
    from memforge_b200.paged_attention import PagedAttention, PagedKVCache
    f = load("standalone.npz")
    for name in ("decode", "multi_query", "long"):
        kc = f[f"{name}_kcache"]
        NB, H, BS, D = kc.shape
        cache = PagedKVCache(num_blocks=NB, block_size=BS, num_heads=H, head_dim=D, device="cuda")
        cache.write_kv(torch.from_numpy(f[f"{name}_keys"]).cuda(),
                       torch.from_numpy(f[f"{name}_values"]).cuda(),
                       f[f"{name}_table"].tolist(), start_pos=0)
        assert np.array_equal(cache.key_cache.cpu().numpy(), kc), name
        assert np.array_equal(cache.value_cache.cpu().numpy(), f[f"{name}_vcache"]), name
        out = PagedAttention()(torch.from_numpy(f[f"{name}_q"]).cuda(), cache,
                               f[f"{name}_table"].tolist(), int(f[f"{name}_ctx"]))
        assert out.shape == f[f"{name}_out"].shape
        assert np.allclose(out.cpu().numpy(), f[f"{name}_out"], atol=ATOL), name


def test_standalone_write_rejects_positions_past_the_table():
    from memforge_b200.paged_attention import PagedKVCache
    cache = PagedKVCache(num_blocks=4, block_size=16, num_heads=2, head_dim=16, device="cuda")
    with pytest.raises(IndexError, match="exceeds allocated block table"):
        cache.write_kv(torch.zeros(1, 2, 20, 16, device="cuda"), torch.zeros(1, 2, 20, 16, device="cuda"),
                       [1], start_pos=0)


# --------------------------------------------------- attention registry seam

def test_registry_function_routes_a_packed_pass_to_the_kernel():
    from memforge_b200 import attention_backend as AB
    from memforge_b200.varlen_attention import paged_attention_varlen
    pool = _small_pool(block=4)
    tables = _tables([13, 6, 20])
    sid, pos = [0, 0, 0, 0, 1, 2], [9, 10, 11, 12, 5, 19]
    q = torch.randn(1, 4, 6, 8, device="cuda")
    module = SimpleNamespace(layer_idx=1)
    with AB.varlen_attention_context(pool, tables, sid, pos) as binding:
        out, _ = AB.paged_attention_forward(module, q, None, None, None)
    assert binding.used == 1
    want = paged_attention_varlen(q, pool.key_pool, pool.value_pool, 1, tables, sid, pos, 4)
    assert out.shape == (1, 6, 4, 8)
    assert torch.allclose(out, want.transpose(1, 2), atol=ATOL)


def test_registry_function_single_query_decode():
    from memforge_b200 import attention_backend as AB
    from memforge_b200.block_attention import paged_attention_blockwise
    pool = _small_pool(block=4)
    table = torch.tensor([5, 2, 9, 1])
    cache = SimpleNamespace(position=14, block_table_tensor_cached=lambda: table)
    q = torch.randn(1, 4, 1, 8, device="cuda")
    with AB.paged_attention_context(pool, cache) as binding:
        out, _ = AB.paged_attention_forward(SimpleNamespace(layer_idx=0), q, None, None, None)
    assert binding.used == 1 and binding.fallbacks == 0
    want = paged_attention_blockwise(q, pool.key_pool, pool.value_pool, 0, table, 14, 4)
    assert torch.allclose(out, want.transpose(1, 2), atol=ATOL)
