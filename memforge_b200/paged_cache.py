"""
``PagedCache``: a ``transformers.Cache`` whose storage is the paged KV pool,
served by the sm_100a kernels.  B200 edition of
``memforge_ml/runtime/paged_cache.py``.

Every attention layer of an unmodified Hugging Face model writes its new keys
and values into 16-token physical blocks through the sequence's block table
(one ``mf_reshape_and_cache`` launch per layer).  What ``update`` hands back to
the model depends on how attention runs:

* with the ``memforge_paged`` attention function and ``paged_attention_context``
  bound (``lazy_read=True``), the attention kernel reads the context straight
  from the pool pages, for a decode token and for a prompt or chunk alike, so
  ``update`` returns only the new rows: nothing is materialised;
* otherwise (any other attention function) ``update`` returns the whole context
  gathered from the pool into contiguous ``(1, H, T, D)`` tensors by the gather
  kernel (``mf_gather_kv``), as the reference's non-lazy mode does.

``rollback(n)`` only moves the write cursor; ``seed_position`` declares a cached
prefix (after a prefix-cache hit).  The contiguous decode mirror of the
reference (``view_capacity``, ``decode_view_cache.py``) is not part of this
build: it is an alternative to paging, and passing it raises.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import torch
from transformers.cache_utils import Cache, CacheLayerMixin

from .kv_pool import PagedKVPool


class PagedCacheLayer(CacheLayerMixin):
    """One attention layer's cursor into the shared paged pool."""

    is_sliding = False
    is_compileable = False
    supports_early_init = False

    def __init__(self, owner: "PagedCache", layer_idx: int):
        super().__init__()
        self.owner = owner
        self.layer_idx = layer_idx
        self.position = 0
        self.is_initialized = True

    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor,
                            *args, **kwargs) -> None:
        self.is_initialized = True   # the pool exists before the first token

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args,
               **kwargs) -> Tuple[torch.Tensor, torch.Tensor]:
        if key_states.shape[0] != 1:
            raise ValueError(
                f"PagedCache is a single-sequence cache; got batch size {key_states.shape[0]}. "
                "Batched decoding goes through ContinuousBatchingEngine instead.")
        start = self.position
        end = start + key_states.shape[-2]
        owner = self.owner
        owner.pool.write_flat(self.layer_idx, owner.flat_indices(start, end), key_states,
                              value_states)
        self.position = end
        if owner.lazy_read and owner.reads_from_pool(end - start):
            return key_states, value_states
        return owner.pool.gather_flat(self.layer_idx, owner.flat_indices(0, end))

    def get_mask_sizes(self, query_length: int, *args, **kwargs) -> Tuple[int, int]:
        return self.position + query_length, 0

    def get_seq_length(self) -> int:
        return self.position

    def get_max_length(self) -> int:
        return self.owner.pool.capacity_tokens

    def get_max_cache_shape(self) -> int:
        return self.owner.pool.capacity_tokens

    def reset(self) -> None:
        self.position = 0

    def crop(self, tokens_to_remove: int) -> None:
        self.position = max(0, self.position - abs(tokens_to_remove))


class PagedCache(Cache):
    """
    Single-sequence KV cache whose storage is a ``PagedKVPool``.

    The engine calls ``set_block_table`` when the allocator grows the
    sequence's table and ``begin_step`` before each forward pass; the index
    translation of a step is computed once and shared by all layers.
    """

    def __init__(self, pool: PagedKVPool, block_table: List[int],
                 device: Optional[str] = None, view_capacity: Optional[int] = None,
                 lazy_read: bool = False):
        if lazy_read and view_capacity:
            raise ValueError(
                "lazy_read and view_capacity are mutually exclusive: the mirror "
                "materialises the context, lazy mode avoids materialising it")
        if view_capacity:
            raise NotImplementedError(
                "the contiguous decode mirror (view_capacity) is not part of the sm_100a build; "
                "use lazy_read=True with the memforge_paged attention function")
        self.pool = pool
        self.device_str = device or pool.spec.device
        self._block_table = PagedKVPool.block_table_tensor(block_table, self.device_str)
        self._flat_memo: Dict[Tuple[int, int], torch.Tensor] = {}
        self._index_memo: Dict[Tuple[int, int], Tuple[torch.Tensor, torch.Tensor]] = {}
        self.lazy_read = bool(lazy_read)
        self.view_cache = None
        super().__init__(layers=[PagedCacheLayer(self, i) for i in range(pool.spec.num_layers)])

    # -------------------------------------------------------------- reading

    @staticmethod
    def reads_from_pool(num_new: int) -> bool:
        """Whether attention reads this step's context from the pool itself."""
        from . import attention_backend
        return num_new == 1 or attention_backend.any_binding_active()

    # ------------------------------------------------------ engine interface

    def set_block_table(self, block_table: List[int]) -> None:
        new = PagedKVPool.block_table_tensor(block_table, self.device_str)
        if self._block_table.numel() != new.numel() or not torch.equal(self._block_table, new):
            self._block_table = new
            self._flat_memo.clear()
            self._index_memo.clear()

    def begin_step(self, block_table: Optional[List[int]] = None) -> None:
        if block_table is not None:
            self.set_block_table(block_table)
        self._flat_memo.clear()
        self._index_memo.clear()

    def seed_position(self, num_cached_tokens: int) -> None:
        """Positions ``0 .. num_cached_tokens-1`` are already in the pool (a shared prefix)."""
        if num_cached_tokens < 0:
            raise ValueError(f"num_cached_tokens must be non-negative, got {num_cached_tokens}")
        for layer in self.layers:
            layer.position = num_cached_tokens
        self._flat_memo.clear()
        self._index_memo.clear()

    def indices(self, start: int, end: int) -> Tuple[torch.Tensor, torch.Tensor]:
        key = (start, end)
        if key not in self._index_memo:
            self._index_memo[key] = self.pool.slot_indices(self._block_table, start, end)
        return self._index_memo[key]

    def flat_indices(self, start: int, end: int) -> torch.Tensor:
        key = (start, end)
        if key not in self._flat_memo:
            self._flat_memo[key] = self.pool.flat_indices(self._block_table, start, end)
        return self._flat_memo[key]

    @property
    def block_table(self) -> List[int]:
        return self._block_table.tolist()

    def block_table_tensor_cached(self) -> torch.Tensor:
        """The block table as the device tensor it is stored as (read-only)."""
        return self._block_table

    @property
    def position(self) -> int:
        return self.layers[0].position

    def rollback(self, num_tokens: int) -> None:
        """Drop the last ``num_tokens`` positions: only the cursor moves."""
        if num_tokens <= 0:
            return
        for layer in self.layers:
            layer.crop(num_tokens)
        self._flat_memo.clear()
        self._index_memo.clear()

    def reset(self) -> None:
        for layer in self.layers:
            layer.reset()
        self._flat_memo.clear()
        self._index_memo.clear()

    def num_blocks_needed(self, total_tokens: int) -> int:
        bs = self.pool.block_size
        return (total_tokens + bs - 1) // bs

    def get_max_cache_shape(self, layer_idx: int = 0) -> int:
        return self.pool.capacity_tokens


class VarlenPackedCacheLayer(CacheLayerMixin):
    """One layer's write of a packed multi-sequence pass (``varlen_cache.py``)."""

    is_sliding = False
    is_compileable = False
    supports_early_init = False

    def __init__(self, owner: "VarlenPackedCache", layer_idx: int):
        super().__init__()
        self.owner = owner
        self.layer_idx = layer_idx
        self.is_initialized = True

    def lazy_initialization(self, *args, **kwargs) -> None:
        self.is_initialized = True

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args,
               **kwargs) -> Tuple[torch.Tensor, torch.Tensor]:
        if key_states.shape[0] != 1:
            raise ValueError(f"VarlenPackedCache takes one packed row, got batch "
                             f"{key_states.shape[0]}")
        if key_states.shape[-2] != self.owner.num_tokens:
            raise ValueError(f"{key_states.shape[-2]} key states for {self.owner.num_tokens} "
                             f"packed tokens")
        self.owner.pool.write_flat(self.layer_idx, self.owner.write_index, key_states,
                                   value_states)
        return key_states, value_states

    def get_mask_sizes(self, query_length: int, *args, **kwargs) -> Tuple[int, int]:
        return query_length, 0

    def get_seq_length(self) -> int:
        return 0

    def get_max_length(self) -> int:
        return self.owner.pool.capacity_tokens

    def get_max_cache_shape(self) -> int:
        return self.owner.pool.capacity_tokens

    def reset(self) -> None:
        pass

    def crop(self, tokens_to_remove: int) -> None:
        raise NotImplementedError(
            "VarlenPackedCache holds no per-sequence cursor to crop; roll back the owning "
            "sequences' PagedCache positions instead")


class VarlenPackedCache(Cache):
    """
    Cache of one packed forward pass over rows of several sequences
    (``memforge_ml/runtime/varlen_cache.py``): each row's K/V goes to its own
    sequence's slot; attention runs under ``varlen_attention_context``.
    """

    def __init__(self, pool, num_layers: int, block_tables, seq_ids, positions):
        if len(seq_ids) != len(positions):
            raise ValueError(f"{len(seq_ids)} seq_ids but {len(positions)} positions")
        if not seq_ids:
            raise ValueError("a packed pass needs at least one token")
        self.pool = pool
        self.block_tables = list(block_tables)
        self.seq_ids = list(seq_ids)
        self.positions = list(positions)
        self.num_tokens = len(seq_ids)
        self.write_index = self._write_index()
        super().__init__(layers=[VarlenPackedCacheLayer(self, i) for i in range(num_layers)])

    def _write_index(self) -> torch.Tensor:
        """
        One flat pool slot per packed token, computed once for every layer.
        Validation reads only the tables' lengths; with device tables the slots
        are computed on the device (one gather), so nothing synchronises.  Two
        tokens of one sequence at one position are rejected here; with host
        tables a slot named by two sequences is rejected too.
        """
        bs = self.pool.block_size
        device = self.pool.key_pool.device
        sizes = [int(t.numel()) if hasattr(t, "numel") else len(t) for t in self.block_tables]
        offs = [0]
        for n in sizes:
            offs.append(offs[-1] + n)
        index, within, seen = [], [], set()
        for seq_id, position in zip(self.seq_ids, self.positions):
            if seq_id < 0 or seq_id >= len(self.block_tables):
                raise IndexError(f"seq_id {seq_id} has no block table "
                                 f"(got {len(self.block_tables)})")
            if position < 0:
                raise ValueError(f"negative position {position}")
            logical = position // bs
            if logical >= sizes[seq_id]:
                raise IndexError(f"position {position} needs logical block {logical} but "
                                 f"sequence {seq_id} has a block table of {sizes[seq_id]}")
            if (seq_id, position) in seen:
                raise ValueError("two packed tokens map to the same pool slot; the step's "
                                 "sequence ids and positions overlap")
            seen.add((seq_id, position))
            index.append(offs[seq_id] + logical)
            within.append(position % bs)
        on_device = device.type == "cuda" and all(
            isinstance(t, torch.Tensor) and t.device == device for t in self.block_tables)
        if on_device:
            cat = torch.cat([t.reshape(-1) for t in self.block_tables]).long()
            meta = torch.tensor([index, within], dtype=torch.long).to(device)
            return cat[meta[0]] * bs + meta[1]
        flat_tables = [int(b) for t in self.block_tables
                       for b in (t.tolist() if hasattr(t, "tolist") else t)]
        flat = [flat_tables[i] * bs + w for i, w in zip(index, within)]
        if len(set(flat)) != len(flat):
            raise ValueError("two packed tokens map to the same pool slot; the step's "
                             "sequence ids and positions overlap")
        return torch.tensor(flat, dtype=torch.long, device=device)

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return 0

    def get_max_cache_shape(self, layer_idx: int = 0) -> int:
        return self.pool.capacity_tokens

    def reset(self) -> None:
        pass

    def __len__(self) -> int:
        return len(self.layers)
