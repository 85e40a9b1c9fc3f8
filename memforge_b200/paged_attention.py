"""
Standalone PagedAttention operator, B200 edition of
``memforge_ml/models/paged_attention.py``.

``PagedKVCache`` keeps the operator's own cache layout
``(num_blocks, num_heads, block_size, head_dim)`` (``paged_attention.py:34-43``);
writes go through the sm_100a scatter kernel (heads-major addressing) and
``PagedAttention.forward`` through the paged attention kernel with every query
row seeing all ``context_len`` keys, as the reference computes it (no causal
mask, ``paged_attention.py:108-141``).  Unlike the reference, query heads may be
a multiple of the cache's heads (grouped-query attention).
"""

from __future__ import annotations

import math
from typing import List, Optional, Tuple

import torch
import torch.nn as nn

from . import _kernels as K


class PagedKVCache:
    """Physical K/V blocks of shape (num_heads, block_size, head_dim) each."""

    def __init__(self, num_blocks: int, block_size: int, num_heads: int, head_dim: int,
                 dtype: torch.dtype = torch.float32, device: str = "cuda"):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = device
        shape = (num_blocks, num_heads, block_size, head_dim)
        self.key_cache = torch.zeros(shape, dtype=dtype, device=device)
        self.value_cache = torch.zeros(shape, dtype=dtype, device=device)

    def _slots(self, block_table: List[int], start: int, n: int) -> torch.Tensor:
        slots = []
        for i in range(n):
            pos = start + i
            logical = pos // self.block_size
            if logical >= len(block_table):
                raise IndexError(
                    f"Logical block {logical} exceeds allocated block table length "
                    f"{len(block_table)}")
            slots.append(int(block_table[logical]) * self.block_size + pos % self.block_size)
        return torch.tensor(slots, dtype=torch.int32)

    def write_kv(self, key_states: torch.Tensor, value_states: torch.Tensor,
                 block_table: List[int], start_pos: int) -> None:
        """Scatter ``(1, H, S, D)`` states at positions ``start_pos..`` (``paged_attention.py:45-67``)."""
        n = key_states.shape[2]
        slots = self._slots(block_table, start_pos, n).to(self.key_cache.device, non_blocking=True)
        k = key_states[0].permute(1, 0, 2).to(self.dtype)
        v = value_states[0].permute(1, 0, 2).to(self.dtype)
        K.reshape_and_cache(k, v, self.key_cache, self.value_cache, slots, heads_major=True)

    def read_kv(self, block_table: List[int], total_len: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Materialise ``(H, total_len, D)`` K/V (``paged_attention.py:69-97``)."""
        nblk = (total_len + self.block_size - 1) // self.block_size
        ks, vs = [], []
        for logical in range(nblk):
            phys = block_table[logical]
            n = min(self.block_size, total_len - logical * self.block_size)
            ks.append(self.key_cache[phys, :, :n, :])
            vs.append(self.value_cache[phys, :, :n, :])
        return torch.cat(ks, dim=1), torch.cat(vs, dim=1)


class PagedAttention(nn.Module):
    """softmax(Q K^T * scale) V against a PagedKVCache (``paged_attention.py:100-141``)."""

    def __init__(self, scale: Optional[float] = None):
        super().__init__()
        self.scale = scale

    def forward(self, query: torch.Tensor, paged_kv: PagedKVCache, block_table: List[int],
                context_len: int) -> torch.Tensor:
        """``query (1, H, q_len, D)`` -> ``(1, q_len, H*D)``."""
        _, num_heads, q_len, head_dim = query.shape
        scale = self.scale or (1.0 / math.sqrt(head_dim))
        if num_heads % paged_kv.num_heads:
            raise ValueError(
                f"{num_heads} query heads is not a multiple of {paged_kv.num_heads} cache heads")
        nblk = (context_len + paged_kv.block_size - 1) // paged_kv.block_size
        if nblk > len(block_table):
            raise IndexError(
                f"context of {context_len} tokens needs {nblk} blocks, block table has "
                f"{len(block_table)}")
        dev = query.device
        K.require_cuda("PagedAttention", query, paged_kv.key_cache)
        meta = torch.tensor([context_len] + [int(b) for b in block_table[:max(nblk, 1)]],
                            dtype=torch.int32).to(dev, non_blocking=True)
        q = query.to(paged_kv.dtype)
        if q.stride(-1) != 1:
            q = q.contiguous()
        out = torch.empty((1, q_len, num_heads, head_dim), device=dev, dtype=q.dtype)
        K.paged_attention(q[0].permute(1, 0, 2), out[0], paged_kv.key_cache, paged_kv.value_cache,
                          meta[1:].view(1, -1), meta[:1], q_per_seq=q_len, scale=scale,
                          causal=False, heads_major=True)
        return out.view(1, q_len, num_heads * head_dim).to(query.dtype)
