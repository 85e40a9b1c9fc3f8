"""
CUDA-graph-safe batched decode with the signature of MemForge's Triton kernel
(``memforge_ml/kernels/triton_paged_decode.py:129-176``), served by the sm_100a
stream-K decode kernel.

``num_splits``/``tile``/``max_ctx`` are accepted for drop-in compatibility and
ignored: the kernel splits every sequence's pages across all SMs itself and
reads the context lengths from the device, so one captured graph serves any
lengths (make one call before capture so the workspace exists).
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _kernels as K
from . import _lib as L


def available() -> bool:
    """True when the library loads and device 0 is an sm_100 GPU."""
    if not torch.cuda.is_available():
        return False
    try:
        import ctypes
        n, ok = ctypes.c_int(0), ctypes.c_int(0)
        L.lib().mf_device_info(torch.cuda.current_device(), ctypes.byref(n), ctypes.byref(ok))
        return bool(ok.value)
    except Exception:
        return False


def paged_decode_attention(q: torch.Tensor, key_flat: torch.Tensor, value_flat: torch.Tensor,
                           block_tables: torch.Tensor, ctx_lens: torch.Tensor, block_size: int,
                           max_ctx: int, scale: float, num_splits: int = 8, tile: int = 64,
                           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """
    Single-token attention for each of B sequences over a paged cache.

    q ``[B, Hq, D]``; key_flat/value_flat one layer viewed ``[slots, Hkv, D]``;
    block_tables ``[B, max_blocks]`` int; ctx_lens ``[B]`` int counting the new
    token.  Returns ``[B, Hq, D]`` in q's dtype.
    """
    B, Hq, D = q.shape
    Hkv = key_flat.shape[1]
    if Hq % Hkv:
        raise ValueError("query heads must be a multiple of kv heads")
    K.require_cuda("paged_decode_attention", q, key_flat, value_flat, block_tables, ctx_lens)
    if key_flat.shape[0] % block_size:
        raise ValueError("pool slots are not a whole number of blocks")
    if block_tables.dtype != torch.int32:
        block_tables = block_tables.to(torch.int32)
    if ctx_lens.dtype != torch.int32:
        ctx_lens = ctx_lens.to(torch.int32)
    kp = key_flat.view(-1, block_size, Hkv, D)
    vp = value_flat.view(-1, block_size, Hkv, D)
    if out is None:
        out = torch.empty((B, Hq, D), device=q.device, dtype=q.dtype)
    K.paged_attention(q, out, kp, vp, block_tables, ctx_lens, q_per_seq=1, scale=scale,
                      causal=True)
    return out
