"""
Paged KV pool, B200 edition of ``memforge_ml/runtime/kv_pool.py``.

Same layout and API: ``key_pool``/``value_pool`` are
``(num_layers, num_blocks, block_size, num_kv_heads, head_dim)`` tensors
(``kv_pool.py:66-68``), so the kernels read and write MemForge's own pool in
place.  Writes go through the sm_100a scatter kernel.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Tuple

import torch

from . import paged_gather


@dataclass(frozen=True)
class ModelKVSpec:
    """Per-token KV geometry (``kv_pool.py:27-55``)."""

    num_layers: int
    num_kv_heads: int
    head_dim: int
    dtype: torch.dtype
    device: str

    @classmethod
    def from_config(cls, config, dtype: torch.dtype, device: str) -> "ModelKVSpec":
        head_dim = getattr(config, "head_dim", None) or (
            config.hidden_size // config.num_attention_heads)
        num_kv_heads = getattr(config, "num_key_value_heads", None) or config.num_attention_heads
        return cls(num_layers=config.num_hidden_layers, num_kv_heads=num_kv_heads,
                   head_dim=head_dim, dtype=dtype, device=device)

    @property
    def bytes_per_token(self) -> int:
        elem = torch.empty(0, dtype=self.dtype).element_size()
        return 2 * self.num_layers * self.num_kv_heads * self.head_dim * elem


class PagedKVPool:
    """Fixed-size physical block pool backing the paged KV cache."""

    def __init__(self, spec: ModelKVSpec, num_blocks: int, block_size: int = 16):
        self.spec = spec
        self.num_blocks = num_blocks
        self.block_size = block_size
        shape = (spec.num_layers, num_blocks, block_size, spec.num_kv_heads, spec.head_dim)
        self.key_pool = torch.zeros(shape, dtype=spec.dtype, device=spec.device)
        self.value_pool = torch.zeros(shape, dtype=spec.dtype, device=spec.device)

    @property
    def bytes_per_block(self) -> int:
        return self.spec.bytes_per_token * self.block_size

    @property
    def total_bytes(self) -> int:
        return self.bytes_per_block * self.num_blocks

    @property
    def capacity_tokens(self) -> int:
        return self.num_blocks * self.block_size

    @staticmethod
    def blocks_for_budget(spec: ModelKVSpec, block_size: int, budget_mb: float) -> int:
        per_block = spec.bytes_per_token * block_size
        return max(1, int((budget_mb * 1024 * 1024) // per_block))

    def slot_indices(self, block_table: torch.Tensor, start: int,
                     end: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Logical ``[start, end)`` -> (physical block, slot) (``kv_pool.py:92-110``)."""
        positions = torch.arange(start, end, device=block_table.device)
        logical = torch.div(positions, self.block_size, rounding_mode="floor")
        slots = positions % self.block_size
        if logical.numel() and int(logical.max()) >= block_table.numel():
            raise IndexError(
                f"logical block {int(logical.max())} is outside a block table of "
                f"{block_table.numel()} entries (token range {start}:{end})")
        return block_table[logical], slots

    @staticmethod
    def block_table_tensor(block_table: List[int], device: str) -> torch.Tensor:
        return torch.tensor(block_table, dtype=torch.long, device=device)

    def flat_indices(self, block_table: torch.Tensor, start: int, end: int) -> torch.Tensor:
        physical, slots = self.slot_indices(block_table, start, end)
        return paged_gather.flat_slot_index(physical, slots, self.block_size)

    def write(self, layer_idx: int, physical: torch.Tensor, slots: torch.Tensor,
              keys: torch.Tensor, values: torch.Tensor) -> None:
        """Scatter ``(1, H, T, D)`` K/V at (physical, slot) (``kv_pool.py:134-149``)."""
        flat = paged_gather.flat_slot_index(physical, slots, self.block_size)
        paged_gather.scatter_kv(self.key_pool, self.value_pool, layer_idx, flat, keys, values,
                                self.block_size)

    def gather(self, layer_idx: int, physical: torch.Tensor,
               slots: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Contiguous ``(1, H, T, D)`` K/V at (physical, slot) (``kv_pool.py:151-170``)."""
        flat = paged_gather.flat_slot_index(physical, slots, self.block_size)
        return self.gather_flat(layer_idx, flat)

    def gather_flat(self, layer_idx: int, flat_index: torch.Tensor):
        """``kv_pool.py:172-179``: one gather kernel for K and V."""
        return paged_gather.gather_kv(self.key_pool, self.value_pool, layer_idx, flat_index,
                                      self.block_size)

    def write_flat(self, layer_idx: int, flat_index: torch.Tensor, keys: torch.Tensor,
                   values: torch.Tensor) -> None:
        """``kv_pool.py:181-192``: one scatter kernel for K and V."""
        paged_gather.scatter_kv(self.key_pool, self.value_pool, layer_idx, flat_index, keys,
                                values, self.block_size)

    def zero_(self) -> None:
        self.key_pool.zero_()
        self.value_pool.zero_()

    def describe(self) -> dict:
        return {
            "num_blocks": self.num_blocks, "block_size": self.block_size,
            "capacity_tokens": self.capacity_tokens,
            "bytes_per_token": self.spec.bytes_per_token, "bytes_per_block": self.bytes_per_block,
            "total_mb": round(self.total_bytes / (1024 * 1024), 2),
            "num_layers": self.spec.num_layers, "num_kv_heads": self.spec.num_kv_heads,
            "head_dim": self.spec.head_dim, "dtype": str(self.spec.dtype),
            "device": self.spec.device,
        }
