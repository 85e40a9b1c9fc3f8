"""
Speculative verify and commit on the paged pool.

MemForge's batched engine verifies K drafts plus one bonus token per sequence
in one target pass and then writes only the confirmed prefix into the pool
(``scatter_accepted_kv``, ``memforge_ml/runtime/batched_speculative.py:780-811``):
rejected slots keep their old contents.  Here the verify kernel reads the K+1
new K/V from a side buffer (the window) instead of the pool, so nothing is
written before acceptance, and ``commit_accepted`` then scatters exactly the
confirmed rows with one reshape_and_cache launch.  The pool afterwards is
byte-identical to the reference's.  ``accept_and_commit`` fuses the round's
acceptance decision (the reference's rejection sampler) with that commit, so
one launch turns the target's probabilities into the updated pool.
"""

from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch

from . import _kernels as K


def verify_attention(q: torch.Tensor, win_k: torch.Tensor, win_v: torch.Tensor,
                     key_layer: torch.Tensor, value_layer: torch.Tensor,
                     block_tables: torch.Tensor, ctx_lens: torch.Tensor,
                     scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                     kv_lens: Optional[torch.Tensor] = None) -> torch.Tensor:
    """
    Attention of W = K+1 window rows per sequence.

    q ``[B*W, Hq, D]`` (sequence-major), win_k/win_v ``[B*W, Hkv, D]`` the new
    keys/values of those rows, key_layer/value_layer one pool layer
    ``(blocks, 16, Hkv, D)``, block_tables int32 ``[B, width]``, ctx_lens int32
    ``[B]`` = tokens already in the pool.  Row j of sequence b sees pool
    positions ``< ctx`` and window rows ``0..j``.
    """
    B = ctx_lens.numel()
    W = q.shape[0] // B
    if W * B != q.shape[0]:
        raise ValueError("q rows are not a whole number of windows")
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if kv_lens is None:
        kv_lens = (ctx_lens + W).to(torch.int32)
    if out is None:
        out = torch.empty_like(q)
    K.paged_attention(q, out, key_layer, value_layer, block_tables, kv_lens, q_per_seq=W,
                      scale=scale, causal=True, win_k=win_k, win_v=win_v)
    return out


def commit_slots(block_tables: torch.Tensor, ctx_lens: torch.Tensor, num_confirmed: torch.Tensor,
                 window: int, block_size: int) -> torch.Tensor:
    """
    Pool slot of every window row: positions ``ctx .. ctx+window-1`` through the
    block table, -1 (skip) from row ``num_confirmed[b]`` on.  Device integer
    arithmetic, CUDA-graph safe.
    """
    j = torch.arange(window, device=ctx_lens.device, dtype=torch.int64)
    pos = ctx_lens.to(torch.int64)[:, None] + j[None, :]
    blk = torch.gather(block_tables.to(torch.int64), 1, pos // block_size)
    slots = blk * block_size + pos % block_size
    keep = j[None, :] < num_confirmed.to(torch.int64)[:, None]
    return torch.where(keep, slots, torch.full_like(slots, -1)).reshape(-1)


def commit_accepted(key_layer: torch.Tensor, value_layer: torch.Tensor, win_k: torch.Tensor,
                    win_v: torch.Tensor, block_tables: torch.Tensor, ctx_lens: torch.Tensor,
                    num_confirmed: torch.Tensor, block_size: int = 16) -> None:
    """
    Write the first ``num_confirmed[b]`` window rows of each sequence into the
    pool: one ``mf_commit_window`` launch (positions ``ctx .. ctx+n-1`` through
    the block table on the device; the rejected rows' slots are left alone).
    ``key_layer`` is one layer ``(blocks, block_size, H, D)`` with ``(B*W, H, D)``
    windows, or the whole pool ``(L, blocks, block_size, H, D)`` with
    ``(L, B*W, H, D)`` windows, which commits every layer in the same launch.
    """
    if key_layer.shape[-3] != block_size:
        raise ValueError(f"pool block size {key_layer.shape[-3]} != {block_size}")
    K.commit_window(win_k, win_v, key_layer, value_layer, block_tables, ctx_lens, num_confirmed)


def scatter_accepted_kv(pool, block_table: torch.Tensor, context_length: int,
                        new_kv: Sequence[Tuple[torch.Tensor, torch.Tensor]], row: int,
                        num_confirmed: int) -> None:
    """The reference's per-sequence commit (``batched_speculative.py:780-811``)."""
    if num_confirmed <= 0:
        return
    physical, slots = pool.slot_indices(block_table, context_length,
                                        context_length + num_confirmed)
    for layer_idx, (keys, values) in enumerate(new_kv):
        pool.write(layer_idx, physical, slots, keys[row:row + 1, :, :num_confirmed, :],
                   values[row:row + 1, :, :num_confirmed, :])


def accept_and_commit(draft_tokens: torch.Tensor, *, target_tokens: Optional[torch.Tensor] = None,
                      target_probs: Optional[torch.Tensor] = None,
                      draft_probs: Optional[torch.Tensor] = None,
                      uniforms: Optional[torch.Tensor] = None,
                      resample_uniform: Optional[torch.Tensor] = None,
                      win_k: Optional[torch.Tensor] = None, win_v: Optional[torch.Tensor] = None,
                      key_pool: Optional[torch.Tensor] = None,
                      value_pool: Optional[torch.Tensor] = None,
                      block_tables: Optional[torch.Tensor] = None,
                      ctx_lens: Optional[torch.Tensor] = None
                      ) -> Tuple[torch.Tensor, torch.Tensor]:
    """
    One launch (``mf_accept_commit``) that decides how many drafts each sequence
    keeps and writes its confirmed prefix into the pool.

    ``draft_tokens`` int ``[B, K]``.  Greedy: ``target_tokens`` int ``[B, K+1]``
    (the target's argmax per slot).  Sampling: ``target_probs`` fp32
    ``[B, K+1, V]``, ``draft_probs`` fp32 ``[B, K, V]``, ``uniforms`` fp32
    ``[B, K]`` (the acceptance draws), ``resample_uniform`` fp32 ``[B]`` (the
    draw of the next token).  With ``win_k``/``win_v`` ``(L, B*(K+1), H, D)``
    (or ``(B*(K+1), H, D)`` for one layer), pools ``(L, blocks, 16, H, D)`` (or
    one layer), int32 ``block_tables [B, width]`` and ``ctx_lens [B]``, rows
    ``0..a`` of each window are committed (``scatter_accepted_kv`` semantics,
    rejected slots untouched).  Returns int32 ``(num_accepted [B], next_token [B])``
    on the device: no host synchronisation.
    """
    from . import _lib as L
    K.require_cuda("accept_and_commit", draft_tokens, target_tokens, target_probs, draft_probs,
                   uniforms, resample_uniform, win_k, win_v, key_pool, value_pool,
                   block_tables, ctx_lens)
    B, nd = draft_tokens.shape
    dev = draft_tokens.device
    a = L.AcceptArgs()
    import ctypes
    a.struct_size = ctypes.sizeof(L.AcceptArgs)
    a.num_seqs, a.num_drafts = B, nd
    keep = []

    def i32(t):
        t = t.to(torch.int32).contiguous()
        keep.append(t)
        return t

    def f32(t):
        t = t.to(torch.float32)
        if t.stride(-1) != 1:
            t = t.contiguous()
        keep.append(t)
        return t
    dt = i32(draft_tokens)
    a.draft_tokens, a.draft_tokens_stride = dt.data_ptr(), dt.stride(0)
    if target_probs is None:
        if target_tokens is None or target_tokens.shape != (B, nd + 1):
            raise ValueError(f"greedy mode needs target_tokens of shape {(B, nd + 1)}")
        tt = i32(target_tokens)
        a.target_tokens, a.target_tokens_stride = tt.data_ptr(), tt.stride(0)
    else:
        V = target_probs.shape[-1]
        if (target_probs.shape != (B, nd + 1, V) or draft_probs is None or
                draft_probs.shape != (B, nd, V) or uniforms is None or
                uniforms.shape != (B, nd) or resample_uniform is None or
                resample_uniform.numel() != B):
            raise ValueError("sampling mode needs target_probs [B, K+1, V], draft_probs "
                             "[B, K, V], uniforms [B, K] and resample_uniform [B]")
        tp, dp, un, ru = f32(target_probs), f32(draft_probs), f32(uniforms), f32(resample_uniform)
        a.target_probs, a.tp_stride_seq, a.tp_stride_slot = tp.data_ptr(), tp.stride(0), tp.stride(1)
        a.draft_probs, a.dp_stride_seq, a.dp_stride_slot = dp.data_ptr(), dp.stride(0), dp.stride(1)
        a.vocab = V
        a.uniforms, a.uniforms_stride = un.data_ptr(), un.stride(0)
        a.resample_uniform = ru.reshape(-1).data_ptr()
    num_accepted = torch.empty(B, dtype=torch.int32, device=dev)
    next_token = torch.empty(B, dtype=torch.int32, device=dev)
    a.num_accepted, a.next_token = num_accepted.data_ptr(), next_token.data_ptr()
    if win_k is not None:
        layered = win_k.dim() == 4
        wk = win_k if layered else win_k.unsqueeze(0)
        wv = win_v if layered else win_v.unsqueeze(0)
        kp = key_pool if layered else key_pool.unsqueeze(0)
        vp = value_pool if layered else value_pool.unsqueeze(0)
        if wv.stride() != wk.stride() or wk.stride(-1) != 1 or wk.shape != wv.shape:
            raise ValueError("window K/V must share shape and strides with a contiguous last dim")
        if vp.stride() != kp.stride() or kp.stride(-1) != 1 or kp.shape != vp.shape:
            raise ValueError("pools must share shape and strides with a contiguous last dim")
        if wk.dtype != kp.dtype:
            raise TypeError("window and pool must share a dtype")
        Lw, R, H, D = wk.shape
        Lp, nb, bs, hp, dp_ = kp.shape
        if (Lw, H, D) != (Lp, hp, dp_) or R != B * (nd + 1):
            raise ValueError(f"window {tuple(wk.shape)} does not match pool {tuple(kp.shape)} "
                             f"and {B} sequences of {nd + 1} rows")
        bt, cx = i32(block_tables), i32(ctx_lens)
        a.win_k, a.win_v = wk.data_ptr(), wv.data_ptr()
        a.win_stride_layer, a.win_stride_row, a.win_stride_head = wk.stride(0), wk.stride(1), wk.stride(2)
        a.key_pool, a.value_pool = kp.data_ptr(), vp.data_ptr()
        a.pool_stride_layer, a.pool_stride_block = kp.stride(0), kp.stride(1)
        a.pool_stride_slot, a.pool_stride_head = kp.stride(2), kp.stride(3)
        a.num_layers, a.num_blocks, a.block_size = Lp, nb, bs
        a.block_tables, a.table_stride = bt.data_ptr(), bt.stride(0)
        a.ctx_lens = cx.data_ptr()
        a.num_kv_heads, a.head_dim, a.elem_bytes = H, D, wk.element_size()
    a.err_flag = K.err_word(dev).data_ptr()
    rc = L.lib().mf_accept_commit(ctypes.byref(a), K._stream_ptr(dev))
    L.check(rc, "mf_accept_commit")
    K.launch_counter["accept_commit"] = K.launch_counter.get("accept_commit", 0) + 1
    K._after("accept_commit", dev)
    return num_accepted, next_token
