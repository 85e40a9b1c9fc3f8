"""
Paged KV gather and scatter, B200 edition of ``memforge_ml/kernels/paged_gather.py``.

``scatter_kv`` (the reshape_and_cache hot op) runs the sm_100a slot-mapping
scatter kernel; ``gather_kv`` the gather kernel (``mf_gather_kv``), the
materialising read for callers that still want a contiguous context (the
attention kernels never need it); ``flat_slot_index`` is the same integer
arithmetic as the reference.
"""

from __future__ import annotations

from typing import Tuple

import torch

from . import _kernels as K


def flat_slot_index(physical: torch.Tensor, slots: torch.Tensor,
                    block_size: int) -> torch.Tensor:
    """``physical * block_size + slot``, contiguous (``paged_gather.py:42-55``)."""
    return (physical * block_size + slots).contiguous()


def gather_kv(key_pool: torch.Tensor, value_pool: torch.Tensor, layer_idx: int,
              flat_index: torch.Tensor, block_size: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """
    Materialise ``(1, heads, tokens, head_dim)`` K/V of one layer
    (``paged_gather.py:58-89``) with one gather launch for K and V.
    """
    slots_per_block = key_pool.shape[2]
    assert slots_per_block == block_size, (
        f"pool block size {slots_per_block} does not match {block_size}"
    )
    return K.gather_kv(key_pool[layer_idx], value_pool[layer_idx], flat_index)


_NARROWING = {(torch.float32, torch.bfloat16), (torch.float32, torch.float16)}


def scatter_kv(key_pool: torch.Tensor, value_pool: torch.Tensor, layer_idx: int,
               flat_index: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
               block_size: int) -> None:
    """
    Write ``(1, heads, tokens, head_dim)`` K/V into the pool at ``flat_index``
    (``paged_gather.py:92-117``), in place, with the reference's cast to the
    pool dtype.  One kernel launch for K and V together; the (1,H,T,D) ->
    (T,H,D) permute is a stride change, not a copy.
    """
    pool_dt = key_pool.dtype
    k = keys[0].permute(1, 0, 2)
    v = values[0].permute(1, 0, 2)
    if k.dtype != pool_dt and (k.dtype, pool_dt) not in _NARROWING:
        k, v = k.to(pool_dt), v.to(pool_dt)   # exact widening / other casts
    kp, vp = key_pool[layer_idx], value_pool[layer_idx]
    if kp.shape[1] != block_size:
        raise ValueError(f"pool block size {kp.shape[1]} does not match {block_size}")
    K.reshape_and_cache(k, v, kp, vp, flat_index)
