"""
Generate the golden fixtures under ``tests/golden`` by running the REFERENCE's
own functions (MemForge, imported from its source tree) on seeded inputs.

Run from the repo root, in a container that has the reference checked out:

    python tests/golden/make_golden.py --reference <path to memforge checkout>

The fixtures (``*.npz``) hold the inputs of each small case and the reference's
outputs; large inputs (BASELINE config 1's pool) are regenerated from their seed
by ``tests/cases.py`` and pinned by a checksum.  Nothing here is needed at test
time: the tests read the committed ``.npz`` files only.

Reference functions exercised (paths inside the reference):
  memforge_ml/kernels/paged_gather.py      flat_slot_index, scatter_kv, gather_kv
  memforge_ml/runtime/kv_pool.py           PagedKVPool.slot_indices/write/write_flat
  memforge_ml/kernels/varlen_attention.py  paged_attention_varlen,
                                           paged_attention_varlen_materialised,
                                           reference_varlen_attention
  memforge_ml/kernels/block_attention.py   paged_attention_blockwise
  memforge_ml/models/paged_attention.py    PagedKVCache, PagedAttention
  memforge_ml/runtime/batched_speculative.py  scatter_accepted_kv
  memforge_ml/speculative/rejection_sampler.py RejectionSampler.verify_tokens
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from tests import cases  # noqa: E402
from oracle.paged_oracle import f32_to_bf16  # noqa: E402


def _t(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x))


def _bf16_tensor(x_f32):
    import torch
    return torch.from_numpy(f32_to_bf16(x_f32).view(np.int16)).view(torch.bfloat16)


def _np(t):
    import torch
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    return t.detach().contiguous().numpy().copy()


def make_pool_np(g, layers, nb, bs, hkv, d):
    k = cases.normal(g, (layers, nb, bs, hkv, d))
    v = cases.normal(g, (layers, nb, bs, hkv, d))
    return k, v


def gen_scatter(out):
    import torch
    from memforge_ml.kernels.paged_gather import flat_slot_index, scatter_kv
    from memforge_ml.runtime.kv_pool import ModelKVSpec, PagedKVPool

    g = cases.rng(101)
    L, NB, BS, H, D = 3, 16, 4, 2, 8
    k0, v0 = make_pool_np(g, L, NB, BS, H, D)
    table = np.array([4, 0, 9, 13], dtype=np.int64)
    start, end = 2, 14
    keys = cases.normal(g, (1, H, end - start, D), 3.0)
    values = cases.normal(g, (1, H, end - start, D), 3.0)
    for pool_dtype in ("f32", "bf16"):
        for src_dtype in ("f32", "bf16"):
            if pool_dtype == "f32" and src_dtype == "bf16":
                continue
            tdt = torch.float32 if pool_dtype == "f32" else torch.bfloat16
            spec = ModelKVSpec(num_layers=L, num_kv_heads=H, head_dim=D, dtype=tdt, device="cpu")
            pool = PagedKVPool(spec, num_blocks=NB, block_size=BS)
            if pool_dtype == "f32":
                pool.key_pool.copy_(_t(k0)); pool.value_pool.copy_(_t(v0))
            else:
                pool.key_pool.copy_(_bf16_tensor(k0)); pool.value_pool.copy_(_bf16_tensor(v0))
            flat = pool.flat_indices(torch.from_numpy(table), start, end)
            kk = _t(keys) if src_dtype == "f32" else _bf16_tensor(keys)
            vv = _t(values) if src_dtype == "f32" else _bf16_tensor(values)
            pool.write_flat(1, flat, kk, vv)
            # The 2-D index path must land the same bytes (test_kernels.py:115-130).
            pool2 = PagedKVPool(spec, num_blocks=NB, block_size=BS)
            pool2.key_pool.copy_(pool.key_pool); pool2.value_pool.copy_(pool.value_pool)
            phys, slots = pool2.slot_indices(torch.from_numpy(table), start, end)
            pool2.write(1, phys, slots, kk, vv)
            assert torch.equal(pool.key_pool, pool2.key_pool)
            np.savez_compressed(
                os.path.join(out, f"scatter_{src_dtype}_to_{pool_dtype}.npz"),
                k0=k0, v0=v0, table=table, start=start, end=end, layer=1,
                keys=keys, values=values, flat=_np(flat),
                k_after=_np(pool.key_pool), v_after=_np(pool.value_pool),
                block_size=BS,
            )
    # flat index KAT straight from the reference function
    flat = flat_slot_index(torch.tensor([3, 1, 0, 2]), torch.tensor([0, 2, 3, 1]), 4)
    np.savez_compressed(os.path.join(out, "flat_slot_index.npz"), flat=_np(flat))


VARLEN_CASES = [
    # name, block, kv_heads, heads, lengths, seq_ids, positions
    ("decode_only", 4, 2, 4, [3, 4, 5, 9], [0, 1, 2, 3], [2, 3, 4, 8]),
    ("full_prefill", 4, 2, 4, [17], [0] * 17, list(range(17))),
    ("chunk_offset", 4, 2, 4, [12], [0] * 7, list(range(5, 12))),
    ("fused", 4, 2, 4, [13, 6, 20], [0, 0, 0, 0, 1, 2], [9, 10, 11, 12, 5, 19]),
    ("interleaved", 4, 2, 8, [11, 6, 20], [1, 0, 2, 0], [5, 9, 19, 10]),
    ("gqa_6_3", 4, 3, 6, [13, 7], [0, 0, 0, 1], [10, 11, 12, 6]),
    ("bs16_mixed", 16, 2, 8, [40, 1, 77], [0] * 5 + [1, 2], [35, 36, 37, 38, 39, 0, 76]),
    ("bs16_gqa5", 16, 5, 15, [150, 33], [0, 1], [149, 32]),
]


def gen_varlen(out):
    import torch
    from memforge_ml.kernels.varlen_attention import (
        paged_attention_varlen, paged_attention_varlen_materialised,
        reference_varlen_attention)
    from memforge_ml.runtime.kv_pool import ModelKVSpec, PagedKVPool

    for idx, (name, bs, hkv, hq, lengths, seq_ids, positions) in enumerate(VARLEN_CASES):
        g = cases.rng(200 + idx)
        D = 8 if bs == 4 else 32
        need = sum((n + bs - 1) // bs for n in lengths)
        NB = need + 6
        L = 2
        k0, v0 = make_pool_np(g, L, NB, bs, hkv, D)
        tables = cases.disjoint_tables(g, lengths, NB, bs)
        q = cases.normal(g, (1, hq, len(seq_ids), D))
        spec = ModelKVSpec(num_layers=L, num_kv_heads=hkv, head_dim=D,
                           dtype=torch.float32, device="cpu")
        pool = PagedKVPool(spec, num_blocks=NB, block_size=bs)
        pool.key_pool.copy_(_t(k0)); pool.value_pool.copy_(_t(v0))
        tt = [torch.from_numpy(tables[i][tables[i] >= 0].astype(np.int64)) for i in range(len(lengths))]
        mat = paged_attention_varlen_materialised(_t(q), pool, 1, tt, seq_ids, positions)
        blk = paged_attention_varlen(_t(q), pool.key_pool, pool.value_pool, 1, tt,
                                     seq_ids, positions, bs)
        ref = reference_varlen_attention(_t(q), pool.key_pool, pool.value_pool, 1, tt,
                                         seq_ids, positions, bs)
        # bf16 variant of the same case: pool + query in bf16.
        spec16 = ModelKVSpec(num_layers=L, num_kv_heads=hkv, head_dim=D,
                             dtype=torch.bfloat16, device="cpu")
        pool16 = PagedKVPool(spec16, num_blocks=NB, block_size=bs)
        pool16.key_pool.copy_(_bf16_tensor(k0)); pool16.value_pool.copy_(_bf16_tensor(v0))
        mat16 = paged_attention_varlen_materialised(_bf16_tensor(q), pool16, 1, tt,
                                                    seq_ids, positions)
        np.savez_compressed(
            os.path.join(out, f"varlen_{name}.npz"),
            k0=k0, v0=v0, tables=tables, q=q, seq_ids=np.array(seq_ids),
            positions=np.array(positions), block_size=bs, layer=1,
            out_materialised=_np(mat), out_blockwise=_np(blk), out_reference=_np(ref),
            out_bf16=_np(mat16),
        )


def gen_blockwise(out):
    import torch
    from memforge_ml.kernels.block_attention import paged_attention_blockwise
    from memforge_ml.runtime.kv_pool import ModelKVSpec, PagedKVPool

    g = cases.rng(300)
    L, NB, BS, hkv, D = 2, 24, 4, 2, 8
    k0, v0 = make_pool_np(g, L, NB, BS, hkv, D)
    spec = ModelKVSpec(num_layers=L, num_kv_heads=hkv, head_dim=D,
                       dtype=torch.float32, device="cpu")
    pool = PagedKVPool(spec, num_blocks=NB, block_size=BS)
    pool.key_pool.copy_(_t(k0)); pool.value_pool.copy_(_t(v0))
    table = np.array([23, 0, 17, 5, 11], dtype=np.int64)
    outs = {}
    for hq in (2, 4, 8):
        for ctx in (1, 5, 18, 20):
            q = cases.normal(g, (1, hq, 1, D))
            o = paged_attention_blockwise(_t(q), pool.key_pool, pool.value_pool, 0,
                                          torch.from_numpy(table), ctx, BS)
            outs[f"q_{hq}_{ctx}"] = q
            outs[f"o_{hq}_{ctx}"] = _np(o)
    # large-score stability case (test_block_attention.py:137-155)
    q = cases.normal(g, (1, 2, 1, D)) * 50.0
    kbig = pool.key_pool.clone() * 50.0
    o = paged_attention_blockwise(_t(q), kbig, pool.value_pool, 0,
                                  torch.from_numpy(table), 11, BS)
    outs["q_big"] = q
    outs["o_big"] = _np(o)
    np.savez_compressed(os.path.join(out, "blockwise.npz"), k0=k0, v0=v0,
                        table=table, block_size=BS, **outs)


def gen_config1(out):
    import torch
    from memforge_ml.kernels.varlen_attention import paged_attention_varlen_materialised
    from memforge_ml.kernels.block_attention import paged_attention_blockwise
    from memforge_ml.runtime.kv_pool import ModelKVSpec, PagedKVPool

    c = cases.config1(0)
    spec = ModelKVSpec(num_layers=1, num_kv_heads=c.num_kv_heads, head_dim=c.head_dim,
                       dtype=torch.float32, device="cpu")
    pool = PagedKVPool(spec, num_blocks=c.num_blocks, block_size=cases.BLOCK)
    pool.key_pool[0].copy_(_t(c.k_pool)); pool.value_pool[0].copy_(_t(c.v_pool))
    seq_ids, positions = cases.rows_of(c)
    tt = [torch.from_numpy(c.tables[s][c.tables[s] >= 0].astype(np.int64)) for s in range(c.batch)]
    q = _t(np.transpose(c.q, (1, 0, 2))[None])
    mat = paged_attention_varlen_materialised(q, pool, 0, tt, seq_ids, positions)
    blk = []
    for s in range(c.batch):
        blk.append(_np(paged_attention_blockwise(
            _t(c.q[s][None, :, None, :]), pool.key_pool, pool.value_pool, 0, tt[s],
            int(c.ctx_lens[s]), cases.BLOCK))[0, :, 0, :])
    np.savez_compressed(os.path.join(out, "config1.npz"),
                        checksum=cases.checksum(c.q, c.k_pool, c.v_pool, c.tables, c.ctx_lens),
                        out_materialised=_np(mat), out_blockwise=np.stack(blk))


def gen_standalone(out):
    import torch
    from memforge_ml.models.paged_attention import PagedAttention, PagedKVCache

    g = cases.rng(400)
    res = {}
    for name, (H, qlen, ctx, D, table) in {
        "decode": (2, 1, 20, 16, [1, 3]),
        "multi_query": (4, 3, 25, 32, [2, 5]),
        "long": (3, 1, 70, 16, [7, 0, 4, 2, 6]),
    }.items():
        cache = PagedKVCache(num_blocks=8, block_size=16, num_heads=H, head_dim=D)
        keys = cases.normal(g, (1, H, ctx, D))
        vals = cases.normal(g, (1, H, ctx, D))
        cache.write_kv(_t(keys), _t(vals), table, start_pos=0)
        q = cases.normal(g, (1, H, qlen, D))
        o = PagedAttention()(_t(q), cache, table, ctx)
        res[f"{name}_keys"] = keys
        res[f"{name}_values"] = vals
        res[f"{name}_kcache"] = _np(cache.key_cache)
        res[f"{name}_vcache"] = _np(cache.value_cache)
        res[f"{name}_q"] = q
        res[f"{name}_table"] = np.array(table)
        res[f"{name}_ctx"] = ctx
        res[f"{name}_out"] = _np(o)
    np.savez_compressed(os.path.join(out, "standalone.npz"), **res)


def gen_commit(out):
    import torch
    from memforge_ml.runtime.batched_speculative import scatter_accepted_kv
    from memforge_ml.runtime.kv_pool import ModelKVSpec, PagedKVPool

    g = cases.rng(500)
    L, NB, BS, H, D, K = 2, 20, 16, 2, 8, 4
    k0, v0 = make_pool_np(g, L, NB, BS, H, D)
    spec = ModelKVSpec(num_layers=L, num_kv_heads=H, head_dim=D,
                       dtype=torch.float32, device="cpu")
    res = {"k0": k0, "v0": v0}
    table = np.array([9, 3, 17, 1], dtype=np.int64)
    new_kv = [(cases.normal(g, (2, H, K + 1, D)), cases.normal(g, (2, H, K + 1, D)))
              for _ in range(L)]
    for confirmed in (0, 1, 3, K + 1):
        pool = PagedKVPool(spec, num_blocks=NB, block_size=BS)
        pool.key_pool.copy_(_t(k0)); pool.value_pool.copy_(_t(v0))
        scatter_accepted_kv(pool, torch.from_numpy(table), 14,
                            [(_t(a), _t(b)) for a, b in new_kv], 1, confirmed)
        res[f"k_after_{confirmed}"] = _np(pool.key_pool)
        res[f"v_after_{confirmed}"] = _np(pool.value_pool)
    for layer, (a, b) in enumerate(new_kv):
        res[f"new_k_{layer}"] = a
        res[f"new_v_{layer}"] = b
    np.savez_compressed(os.path.join(out, "commit.npz"), table=table, ctx=14, row=1,
                        block_size=BS, **res)


def gen_accept(out):
    """
    RejectionSampler.verify_tokens on seeded draft/target distributions.  Its
    uniforms come from torch.rand(1), one per examined draft, after
    torch.manual_seed(seed): the same calls replayed after the same seed give
    the values it compared against (stored as `uniforms`), so the acceptance
    count is reproducible from them.  The draws after the decision
    (torch.multinomial) are recorded to check which distribution they come from.
    """
    import torch
    from memforge_ml.speculative.rejection_sampler import RejectionSampler
    g = cases.rng(70)
    K, V, cases_n = 4, 12, 64
    res = {"draft": [], "p": [], "q": [], "uniforms": [], "accepted": [], "last_token": [],
           "last_is_draft": []}
    for c in range(cases_n):
        q = g.dirichlet(np.ones(V) * 0.5, size=K).astype(np.float32)
        p = g.dirichlet(np.ones(V) * 0.5, size=K + 1).astype(np.float32)
        if c % 4 == 0:   # drafts the target agrees with: long accepted runs
            p[:K] = 0.6 * q + 0.4 * p[:K]
        draft = np.array([g.choice(V, p=q[i] / q[i].sum()) for i in range(K)], np.int32)
        seed = 1000 + c
        torch.manual_seed(seed)
        toks, is_draft, n = RejectionSampler.verify_tokens(
            [int(x) for x in draft], [torch.from_numpy(q[i]) for i in range(K)],
            [torch.from_numpy(p[i]) for i in range(K + 1)])
        torch.manual_seed(seed)
        r = np.array([torch.rand(1).item() for _ in range(K)], np.float32)
        res["draft"].append(draft)
        res["p"].append(p)
        res["q"].append(q)
        res["uniforms"].append(r)
        res["accepted"].append(n)
        res["last_token"].append(toks[-1] if toks else -1)
        res["last_is_draft"].append(bool(is_draft[-1]) if is_draft else True)
    np.savez_compressed(os.path.join(out, "accept.npz"),
                        **{k: np.asarray(v) for k, v in res.items()})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    import torch
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    gen_scatter(HERE)
    gen_varlen(HERE)
    gen_blockwise(HERE)
    gen_config1(HERE)
    gen_standalone(HERE)
    gen_commit(HERE)
    gen_accept(HERE)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
