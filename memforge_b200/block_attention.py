"""
Single-query paged decode, B200 edition of ``memforge_ml/kernels/block_attention.py``.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from . import _kernels as K


def paged_attention_blockwise(query: torch.Tensor, key_pool: torch.Tensor,
                              value_pool: torch.Tensor, layer_idx: int,
                              block_table: torch.Tensor, context_length: int, block_size: int,
                              scale: Optional[float] = None) -> torch.Tensor:
    """
    One decode step for one sequence read straight from the pool
    (``block_attention.py:51-145``): ``query (1, H, 1, D)`` against the first
    ``context_length`` tokens of ``block_table``; GQA when H exceeds the pool's
    kv heads.  Returns ``(1, H, 1, D)`` in the query dtype.
    """
    if query.shape[0] != 1 or query.shape[2] != 1:
        raise ValueError(
            f"expected a single query position (1, H, 1, D), got {tuple(query.shape)}")
    if context_length <= 0:
        raise ValueError(f"context_length must be positive, got {context_length}")
    num_heads, head_dim = query.shape[1], query.shape[3]
    num_kv_heads = key_pool.shape[3]
    if num_heads % num_kv_heads != 0:
        raise ValueError(
            f"{num_heads} query heads is not a multiple of {num_kv_heads} kv heads")
    num_logical = (context_length + block_size - 1) // block_size
    if num_logical > block_table.numel():
        raise IndexError(
            f"context of {context_length} tokens needs {num_logical} blocks, "
            f"block table has {block_table.numel()}")
    K.require_cuda("paged_attention_blockwise", query, key_pool, value_pool)
    scale = scale if scale is not None else 1.0 / math.sqrt(head_dim)
    dev = query.device
    table = block_table.to(device=dev, dtype=torch.int32).reshape(1, -1)
    kv = torch.tensor([context_length], dtype=torch.int32).to(dev, non_blocking=True)
    q = query if query.stride(-1) == 1 else query.contiguous()
    out = torch.empty_like(q)
    K.paged_attention(q[0].permute(1, 0, 2), out[0].permute(1, 0, 2), key_pool[layer_idx],
                      value_pool[layer_idx], table, kv, q_per_seq=1, scale=scale, causal=True)
    return out
