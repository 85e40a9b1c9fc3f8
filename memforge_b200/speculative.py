"""
Speculative verify and commit on the paged pool.

MemForge's batched engine verifies K drafts plus one bonus token per sequence
in one target pass and then writes only the confirmed prefix into the pool
(``scatter_accepted_kv``, ``memforge_ml/runtime/batched_speculative.py:780-811``):
rejected slots keep their old contents.  Here the verify kernel reads the K+1
new K/V from a side buffer (the window) instead of the pool, so nothing is
written before acceptance, and ``commit_accepted`` then scatters exactly the
confirmed rows with one reshape_and_cache launch.  The pool afterwards is
byte-identical to the reference's.
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
