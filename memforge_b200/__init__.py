"""
memforge_b200 — MemForge's paged-attention hot path on NVIDIA B200 (sm_100a).

The kernels live in ``libmemforge_sm100.so`` (C ABI: include/memforge_sm100.h);
these modules keep MemForge's operator API so they drop in for it:

* ``paged_gather`` / ``kv_pool``       — slot math, ``scatter_kv`` / ``write_flat``
* ``block_attention``                  — ``paged_attention_blockwise``
* ``varlen_attention``                 — ``paged_attention_varlen[_materialised]``
* ``paged_decode``                     — ``paged_decode_attention`` (Triton signature)
* ``paged_attention``                  — standalone ``PagedKVCache`` / ``PagedAttention``
* ``attention_backend``                — the transformers registry function
* ``speculative``                      — verify over a side window + confirmed-prefix commit
* ``kv_shard``                         — KV-head sharding across GPUs with an NCCL all-gather
"""

from . import _lib  # noqa: F401

__all__ = ["build_library"]


def build_library(force: bool = False) -> str:
    from .build import build
    return build(force=force)
