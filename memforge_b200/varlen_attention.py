"""
Varlen paged attention, B200 edition of ``memforge_ml/kernels/varlen_attention.py``.

``paged_attention_varlen`` and ``paged_attention_varlen_materialised`` keep the
reference's signatures, validation and result; both run one sm_100a paged
attention launch (decode rows, speculative windows and prefill chunks alike).

Per call, nothing is synchronised and nothing is pinned:

* the plan (segments, row order) depends only on ``seq_ids``, ``positions`` and
  the tables' lengths; it is memoised, and its int32 metadata is uploaded once
  per distinct pass, so the layers of one forward pass after the first reuse it;
* device block tables are assembled on the device (one concatenation and one
  gather per call), so their contents are never read by the host and the call
  can be captured in a CUDA graph after one warm-up call with the same
  arguments (the graph then re-reads the tables on every replay).
"""

from __future__ import annotations

import math
import threading
from collections import OrderedDict
from typing import Optional, Sequence

import numpy as np
import torch

from . import _kernels as K
from .varlen_plan import VarlenPlan, group_by_sequence, plan_varlen  # noqa: F401

MASK_FILL = float("-inf")

_MEMO_ENTRIES = 16
_memo: "OrderedDict[tuple, tuple]" = OrderedDict()
_memo_lock = threading.Lock()


def _on_device(tables, device) -> bool:
    return len(tables) > 0 and all(isinstance(t, torch.Tensor) and t.device == device
                                   for t in tables)


def _plan(total, block_tables, seq_ids, positions, block_size, num_heads, num_kv_heads, device):
    """(plan, device cu, device kv, device row_map or None, device table index or None)."""
    sizes = tuple(int(t.numel()) if hasattr(t, "numel") else int(np.asarray(t).size)
                  for t in block_tables)
    on_dev = _on_device(block_tables, device)
    key = (tuple(seq_ids), tuple(positions), sizes, block_size, num_heads, num_kv_heads,
           str(device), on_dev)
    with _memo_lock:
        hit = _memo.get(key)
        if hit is not None:
            _memo.move_to_end(key)
            return hit
    plan = plan_varlen(total, block_tables, seq_ids, positions, block_size, num_heads,
                       num_kv_heads)
    if torch.cuda.is_current_stream_capturing():
        raise RuntimeError("paged_attention_varlen: make one call with these arguments before "
                           "capturing a CUDA graph (the plan is uploaded on first use)")
    parts = [plan.cu_seqlens, plan.kv_lens]
    if plan.row_map is not None:
        parts.append(plan.row_map)
    host = np.concatenate([p.astype(np.int32) for p in parts])
    dev = torch.from_numpy(host).to(device)
    at, views = 0, []
    for p in parts:
        views.append(dev[at:at + p.size])
        at += p.size
    index = None
    if on_dev:
        index = torch.from_numpy(plan.table_index(sizes)).to(device)
    entry = (plan, views[0], views[1], views[2] if len(views) > 2 else None, index)
    with _memo_lock:
        _memo[key] = entry
        while len(_memo) > _MEMO_ENTRIES:
            _memo.popitem(last=False)
    return entry


def _tables(plan: VarlenPlan, block_tables, index, device) -> torch.Tensor:
    """int32 [segments, width] block ids on the device."""
    if index is not None:
        parts = [t.reshape(-1) for t in block_tables]
        parts.append(torch.zeros(1, dtype=parts[0].dtype, device=device))
        return torch.cat(parts)[index].to(torch.int32)
    return torch.from_numpy(plan.host_tables(block_tables)).to(device)


def _run(query, key_layer, value_layer, block_tables, seq_ids, positions, scale, block_size):
    K.require_cuda("paged_attention_varlen", query, key_layer, value_layer)
    if query.shape[0] != 1:
        raise ValueError(f"expected a packed batch of 1, got {tuple(query.shape)}")
    plan, cu, kv, row_map, index = _plan(query.shape[2], block_tables, seq_ids, positions,
                                         block_size, query.shape[1], key_layer.shape[2],
                                         query.device)
    if key_layer.shape[1] != block_size:
        raise ValueError(f"pool block size {key_layer.shape[1]} does not match {block_size}")
    head_dim = query.shape[3]
    scale = scale if scale is not None else 1.0 / math.sqrt(head_dim)
    tables = _tables(plan, block_tables, index, query.device)
    out = torch.empty_like(query, memory_format=torch.contiguous_format)
    if plan.uniform_q:
        K.paged_attention(query[0].transpose(0, 1), out[0].transpose(0, 1), key_layer,
                          value_layer, tables, kv, q_per_seq=plan.uniform_q, scale=scale,
                          causal=True)
    else:
        K.paged_attention(query[0].transpose(0, 1), out[0].transpose(0, 1), key_layer,
                          value_layer, tables, kv, cu_seqlens_q=cu, max_q_len=plan.max_q_len,
                          scale=scale, causal=True, row_map=row_map)
    return out


def paged_attention_varlen(query: torch.Tensor, key_pool: torch.Tensor, value_pool: torch.Tensor,
                           layer_idx: int, block_tables: Sequence[torch.Tensor],
                           seq_ids: Sequence[int], positions: Sequence[int], block_size: int,
                           scale: Optional[float] = None) -> torch.Tensor:
    """
    Attention for a packed run of query tokens from several sequences
    (``varlen_attention.py:78-235``): row r attends to keys ``0..positions[r]``
    of ``block_tables[seq_ids[r]]``.  ``query`` is ``(1, H, T, D)``; the result
    has the same shape and dtype.
    """
    return _run(query, key_pool[layer_idx], value_pool[layer_idx], block_tables, seq_ids,
                positions, scale, block_size)


def paged_attention_varlen_materialised(query: torch.Tensor, pool, layer_idx: int,
                                        block_tables: Sequence[torch.Tensor],
                                        seq_ids: Sequence[int], positions: Sequence[int],
                                        scale: Optional[float] = None) -> torch.Tensor:
    """
    Same function as ``paged_attention_varlen`` (``varlen_attention.py:291-395``).
    On B200 nothing is materialised: both names run the same kernel.
    """
    return _run(query, pool.key_pool[layer_idx], pool.value_pool[layer_idx], block_tables,
                seq_ids, positions, scale, pool.block_size)
