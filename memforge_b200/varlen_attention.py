"""
Varlen paged attention, B200 edition of ``memforge_ml/kernels/varlen_attention.py``.

``paged_attention_varlen`` and ``paged_attention_varlen_materialised`` keep the
reference's signatures, validation and result; both run one sm_100a paged
attention launch (decode rows, speculative windows and prefill chunks alike).
``reference_varlen_attention`` is kept as the reference's plain-softmax
definition for callers that want an independent check.
"""

from __future__ import annotations

import math
from typing import Optional, Sequence

import torch

from . import _kernels as K
from .varlen_plan import VarlenPlan, group_by_sequence, plan_varlen  # noqa: F401

MASK_FILL = float("-inf")


def upload_plan(plan: VarlenPlan, device: torch.device):
    """One host->device copy of every int32 array the kernel reads."""
    buf, offs = plan.packed()
    host = torch.from_numpy(buf)
    if device.type == "cuda":
        host = host.pin_memory()
    dev = host.to(device, non_blocking=True)

    def view(name):
        o, n = offs[name]
        return dev[o:o + n]

    tables = view("tables").view(plan.tables.shape)
    row_map = view("row_map") if "row_map" in offs else None
    return tables, view("cu"), view("kv"), row_map


def _run(query, key_layer, value_layer, plan: VarlenPlan, scale, block_size):
    K.require_cuda("paged_attention_varlen", query, key_layer, value_layer)
    if key_layer.shape[1] != block_size:
        raise ValueError(f"pool block size {key_layer.shape[1]} does not match {block_size}")
    head_dim = query.shape[3]
    scale = scale if scale is not None else 1.0 / math.sqrt(head_dim)
    if query.stride(-1) != 1:
        query = query.contiguous()
    tables, cu, kv, row_map = upload_plan(plan, query.device)
    out = torch.empty_like(query)
    K.paged_attention(query[0].permute(1, 0, 2), out[0].permute(1, 0, 2), key_layer, value_layer,
                      tables, kv, cu_seqlens_q=cu, max_q_len=plan.max_q_len, scale=scale,
                      causal=True, row_map=row_map)
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
    if query.shape[0] != 1:
        raise ValueError(f"expected a packed batch of 1, got {tuple(query.shape)}")
    plan = plan_varlen(query.shape[2], block_tables, seq_ids, positions, block_size,
                       query.shape[1], key_pool.shape[3])
    return _run(query, key_pool[layer_idx], value_pool[layer_idx], plan, scale, block_size)


def paged_attention_varlen_materialised(query: torch.Tensor, pool, layer_idx: int,
                                        block_tables: Sequence[torch.Tensor],
                                        seq_ids: Sequence[int], positions: Sequence[int],
                                        scale: Optional[float] = None) -> torch.Tensor:
    """
    Same function as ``paged_attention_varlen`` (``varlen_attention.py:291-395``).
    On B200 nothing is materialised: both names run the same kernel.
    """
    if query.shape[0] != 1:
        raise ValueError(f"expected a packed batch of 1, got {tuple(query.shape)}")
    plan = plan_varlen(query.shape[2], block_tables, seq_ids, positions, pool.block_size,
                       query.shape[1], pool.key_pool.shape[3])
    return _run(query, pool.key_pool[layer_idx], pool.value_pool[layer_idx], plan, scale,
                pool.block_size)


def reference_varlen_attention(query, key_pool, value_pool, layer_idx, block_tables, seq_ids,
                               positions, block_size, scale=None):
    """
    The reference's plain definition (``varlen_attention.py:238-288``): each
    row's visible context gathered token by token, one softmax.  Slow; for checks.
    """
    num_heads, head_dim = query.shape[1], query.shape[3]
    group = num_heads // key_pool.shape[3]
    scale = scale if scale is not None else 1.0 / math.sqrt(head_dim)
    out = torch.zeros((num_heads, query.shape[2], head_dim), dtype=torch.float32,
                      device=query.device)
    for row in range(query.shape[2]):
        table = block_tables[seq_ids[row]]
        visible = positions[row] + 1
        pos = torch.arange(visible, device=key_pool.device)
        phys = torch.as_tensor(table, device=key_pool.device).long()[pos // block_size]
        keys = key_pool[layer_idx, phys, pos % block_size].float()
        values = value_pool[layer_idx, phys, pos % block_size].float()
        if group > 1:
            keys = keys.repeat_interleave(group, dim=1)
            values = values.repeat_interleave(group, dim=1)
        q = query[0, :, row, :].float()
        w = torch.softmax(torch.einsum("hd,thd->ht", q, keys) * scale, dim=-1)
        out[:, row, :] = torch.einsum("ht,thd->hd", w, values)
    return out.unsqueeze(0).to(query.dtype)
