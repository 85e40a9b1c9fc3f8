"""
mf_paged_decode_noalloc — paged decode for callers that cannot allocate device
memory (their memory belongs to another allocator, or they are handed only
input and output buffers) — against mf_paged_decode with a caller workspace.

Called through the C ABI on raw device pointers, twice in a row: the library's
fixed scratch array is shared by every call and keeps the last call's contents,
so the second call checks that nothing left behind by the first one leaks in.
Collected last on purpose (file name), and self-contained so it also passes on
its own in a fresh process.
"""

import ctypes
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

L = pytest.importorskip("memforge_b200._lib")


def _case(seed, B=24, Hq=32, Hkv=8, D=128, max_ctx=3000):
    g = torch.Generator(device="cuda").manual_seed(seed)
    ctx = torch.randint(1, max_ctx, (B,), generator=g, device="cuda", dtype=torch.int32)
    nblk = ((ctx + 15) // 16).tolist()
    NB = sum(nblk) + 32
    perm = torch.randperm(NB, generator=g, device="cuda").to(torch.int32)
    width = max(nblk)
    tables = torch.zeros((B, width), dtype=torch.int32, device="cuda")
    at = 0
    for b, n in enumerate(nblk):
        tables[b, :n] = perm[at:at + n]
        at += n
    k = torch.randn((NB * 16, Hkv, D), generator=g, device="cuda", dtype=torch.bfloat16)
    v = torch.randn_like(k)
    q = torch.randn((B, Hq, D), generator=g, device="cuda", dtype=torch.bfloat16)
    return q, k, v, tables, ctx


def _call(fn_name, q, k, v, tables, ctx, out, workspace=None):
    lib = L.lib()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    B, Hq, D = q.shape
    Hkv = k.shape[1]
    stream = torch.cuda.current_stream().cuda_stream
    common = [q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), v.data_ptr(), k.stride(0),
              k.stride(1), k.shape[0], tables.data_ptr(), tables.stride(0), ctx.data_ptr(), B,
              Hq, Hkv, D, 16, ctypes.c_float(1 / math.sqrt(D)), L.MF_BF16, out.data_ptr()]
    if fn_name == "mf_paged_decode":
        rc = lib.mf_paged_decode(*common, workspace.data_ptr(), workspace.numel(),
                                 err.data_ptr(), stream)
    else:
        rc = lib.mf_paged_decode_noalloc(*common, err.data_ptr(), stream)
    L.check(rc, fn_name)
    torch.cuda.synchronize()
    assert int(err.item()) == 0, L.describe_err(int(err.item()))
    return out


def _workspace_for(q, k, tables, ctx):
    a = L.AttentionArgs()
    a.struct_size = ctypes.sizeof(a)
    B, Hq, D = q.shape
    a.q, a.q_stride_row, a.q_stride_head = q.data_ptr(), q.stride(0), q.stride(1)
    a.out, a.out_stride_row, a.out_stride_head = q.data_ptr(), Hq * D, D
    a.k_pool = a.v_pool = k.data_ptr()
    a.pool_stride_block, a.pool_stride_slot, a.pool_stride_head = k.stride(0) * 16, k.stride(0), k.stride(1)
    a.num_blocks, a.block_size = k.shape[0] // 16, 16
    a.block_tables, a.table_stride = tables.data_ptr(), tables.stride(0)
    a.q_per_seq, a.kv_lens = 1, ctx.data_ptr()
    a.num_seqs, a.total_q, a.max_q_len = B, B, 1
    a.num_q_heads, a.num_kv_heads, a.head_dim = Hq, k.shape[1], D
    a.scale, a.causal, a.dtype = 1 / math.sqrt(D), 1, L.MF_BF16
    need = L.lib().mf_paged_attention_workspace_size(a, torch.cuda.current_device())
    assert 0 < need <= (16 << 20), need   # fits the library's fixed scratch array
    return torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")


# Two calls whose split-K plans differ (batch, head geometry and context
# lengths), so the second call's ranges and arrival counters are not the
# first call's.  Both entry points run the same kernel with the same plan and
# the same fixed merge order, so their outputs must be bit-identical.
CALLS = [dict(seed=11, B=24, Hq=32, Hkv=8, max_ctx=3000),
         dict(seed=12, B=7, Hq=16, Hkv=2, max_ctx=6000)]


def test_noalloc_decode_matches_the_workspace_entry_point_twice():
    for call, kw in enumerate(CALLS):
        q, k, v, tables, ctx = _case(kw["seed"], B=kw["B"], Hq=kw["Hq"], Hkv=kw["Hkv"],
                                     max_ctx=kw["max_ctx"])
        ws = _workspace_for(q, k, tables, ctx)
        want = _call("mf_paged_decode", q, k, v, tables, ctx, torch.empty_like(q), ws)
        got = _call("mf_paged_decode_noalloc", q, k, v, tables, ctx, torch.empty_like(q))
        assert torch.isfinite(got).all()
        diff = (got.float() - want.float()).abs()
        assert torch.equal(got, want), f"call {call}: max |diff| {float(diff.max()):.3e}"
