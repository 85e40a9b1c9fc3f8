"""
The ``memforge_paged`` attention function for transformers, served by the
sm_100a paged-attention kernel.

Interface kept from ``memforge_ml/kernels/attention_backend.py``: the registry
name, ``paged_attention_forward(module, query, key, value, attention_mask,
scaling, dropout, **kw) -> ((B, q_len, H, D), None)`` (``:195-292``), the two
binding context managers ``paged_attention_context(pool, cache)`` and
``varlen_attention_context(pool, block_tables, seq_ids, positions,
block_wise=False)`` with their ``used`` / ``fallbacks`` counters, and
``register`` / ``enable_on`` / ``is_enabled_on`` / ``backend_enabled_on``
(``:360-465``).

How this one works:

* A binding says where a layer's keys live: a pool and block tables.  While one
  is active, every layer reads its K/V from the pool pages (the cache's
  ``update`` wrote this step's rows just before), for any query length:
  decode, a whole prompt, a chunk over a cached prefix.  The ``key``/``value``
  the model hands over are not read.
* A binding's kernel metadata (int32 tables, row offsets, key counts, row order)
  is built on its first use and uploaded once; every later layer of the same
  forward pass reuses the device copy.
* ``graph_attention_context`` binds a batched decode step whose tables and
  lengths are device tensors (the graphed decoder captures it in a CUDA graph).
* Outside any binding, the handed ``key``/``value`` are first written into a
  transient paged pool by the KV-write kernel (slot = position), then attended
  by the same kernel.  A padding mask or a non-causal mask function cannot be
  expressed that way and raises: there is no second attention implementation to
  fall back to.
* ``fallbacks`` exists for interface compatibility and stays 0.
"""

from __future__ import annotations

import math
import threading
from contextlib import contextmanager
from typing import Any, List, Optional, Sequence, Tuple

import torch

from . import _kernels as K
from .varlen_attention import _plan as _varlen_plan
from .varlen_attention import _tables as _varlen_tables

BACKEND_NAME = "memforge_paged"

_local = threading.local()


# ------------------------------------------------------------------ bindings

class _DeviceRows:
    """Kernel metadata of one set of query rows, resident on the device."""

    __slots__ = ("tables", "cu", "kv", "row_map", "max_q", "rows", "q_per_seq")

    def __init__(self, tables, cu, kv, row_map, max_q, rows, q_per_seq=0):
        self.tables, self.cu, self.kv, self.row_map = tables, cu, kv, row_map
        self.max_q, self.rows = max_q, rows
        self.q_per_seq = q_per_seq  # > 0: every sequence has this many rows, in order


def _upload(arrays: List, device) -> List[torch.Tensor]:
    """int32 host arrays -> device tensors with one host-to-device copy."""
    import numpy as np
    flat = np.concatenate([np.asarray(a, np.int32).reshape(-1) for a in arrays])
    dev = torch.from_numpy(flat).to(device, non_blocking=False)
    out, at = [], 0
    for a in arrays:
        n = int(np.asarray(a).size)
        out.append(dev[at:at + n].view(np.asarray(a).shape))
        at += n
    return out


class _Binding:
    """One sequence's ``PagedCache`` over a pool; the context length is read per call."""

    __slots__ = ("pool", "cache", "used", "fallbacks", "_meta")

    def __init__(self, pool, cache):
        self.pool = pool
        self.cache = cache
        self.used = 0
        self.fallbacks = 0
        self._meta = {}

    @property
    def block_table(self) -> torch.Tensor:
        return self.cache.block_table_tensor_cached()

    @property
    def context_length(self) -> int:
        return self.cache.position

    def rows(self, q_len: int, device) -> _DeviceRows:
        ctx = self.context_length
        key = (ctx, q_len)
        meta = self._meta.get(key)
        if meta is None:
            if ctx < q_len:
                raise ValueError(f"{q_len} query rows but only {ctx} cached positions: the "
                                 f"cache must write this step's keys before attention runs")
            need = (ctx + self.pool.block_size - 1) // self.pool.block_size
            table = self.block_table
            if need > table.numel():
                raise IndexError(f"context of {ctx} tokens needs {need} blocks, but the block "
                                 f"table has {table.numel()} entries")
            tables = table.reshape(1, -1).to(device=device, dtype=torch.int32)
            cu, kv = _upload([[0, q_len], [ctx]], device)
            meta = _DeviceRows(tables, cu, kv, None, q_len, q_len, q_per_seq=q_len)
            self._meta[key] = meta
        return meta


class _VarlenBinding:
    """A packed multi-sequence pass: per-row sequence ids and absolute positions."""

    __slots__ = ("pool", "block_tables", "seq_ids", "positions", "used", "fallbacks",
                 "block_wise", "_meta")

    def __init__(self, pool, block_tables, seq_ids, positions, block_wise=False):
        self.pool = pool
        self.block_tables = list(block_tables)
        self.seq_ids = list(seq_ids)
        self.positions = list(positions)
        self.block_wise = bool(block_wise)   # accepted; both forms run the same kernel
        self.used = 0
        self.fallbacks = 0
        self._meta = None

    def rows(self, num_heads: int, device) -> _DeviceRows:
        if self._meta is None:
            plan, cu, kv, row_map, index = _varlen_plan(
                len(self.seq_ids), self.block_tables, self.seq_ids, self.positions,
                self.pool.block_size, num_heads, self.pool.key_pool.shape[3], device)
            tables = _varlen_tables(plan, self.block_tables, index, device)
            self._meta = _DeviceRows(tables, cu, kv, row_map, plan.max_q_len, plan.total,
                                     q_per_seq=plan.uniform_q)
        return self._meta


class _GraphBinding:
    """A graphed decode step: one new token per row, device tables and lengths."""

    __slots__ = ("pool", "tables", "ctx", "used", "fallbacks")

    def __init__(self, pool, tables: torch.Tensor, ctx: torch.Tensor):
        self.pool, self.tables, self.ctx = pool, tables, ctx
        self.used = 0
        self.fallbacks = 0


def _current() -> Optional[_Binding]:
    return getattr(_local, "binding", None)


def _current_graph() -> Optional[_GraphBinding]:
    return getattr(_local, "graph", None)


def _current_varlen() -> Optional[_VarlenBinding]:
    return getattr(_local, "varlen", None)


@contextmanager
def paged_attention_context(pool, cache):
    """Bind one sequence's paged cache for the attention calls of a forward pass."""
    saved = _current()
    _local.binding = _Binding(pool, cache)
    try:
        yield _local.binding
    finally:
        _local.binding = saved


@contextmanager
def varlen_attention_context(pool, block_tables: Sequence[torch.Tensor], seq_ids: Sequence[int],
                             positions: Sequence[int], block_wise: bool = False):
    """Bind a packed pass (rows of several sequences at absolute positions)."""
    saved = _current_varlen()
    _local.varlen = _VarlenBinding(pool, block_tables, seq_ids, positions, block_wise)
    try:
        yield _local.varlen
    finally:
        _local.varlen = saved


@contextmanager
def graph_attention_context(pool, block_tables: torch.Tensor, ctx_lens: torch.Tensor):
    """
    Bind a batched decode step whose int32 block tables ``[B, width]`` and
    context lengths ``[B]`` (counting the new token) live on the device, so the
    step can be captured in a CUDA graph and replayed with new values.
    """
    saved = _current_graph()
    _local.graph = _GraphBinding(pool, block_tables, ctx_lens)
    try:
        yield _local.graph
    finally:
        _local.graph = saved


def any_binding_active() -> bool:
    return (_current() is not None or _current_varlen() is not None
            or _current_graph() is not None)


# ------------------------------------------------------------ the function

def _run(query_rows, out_rows, pool, layer_idx, meta: _DeviceRows, scale, causal=True):
    if meta.q_per_seq:
        K.paged_attention(query_rows, out_rows, pool.key_pool[layer_idx],
                          pool.value_pool[layer_idx], meta.tables, meta.kv,
                          q_per_seq=meta.q_per_seq, scale=scale, causal=causal)
    else:
        K.paged_attention(query_rows, out_rows, pool.key_pool[layer_idx],
                          pool.value_pool[layer_idx], meta.tables, meta.kv, cu_seqlens_q=meta.cu,
                          max_q_len=meta.max_q, scale=scale, causal=causal, row_map=meta.row_map)


def paged_attention_forward(module: Any, query: torch.Tensor, key: torch.Tensor,
                            value: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                            scaling: Optional[float] = None, dropout: float = 0.0,
                            **kwargs: Any) -> Tuple[torch.Tensor, None]:
    """
    ``query`` ``(B, Hq, q_len, D)``; returns ``((B, q_len, Hq, D), None)``.
    Bound calls read K/V from the pool; unbound calls attend to ``key``/``value``.
    """
    if dropout and getattr(module, "training", False):
        raise NotImplementedError("memforge_paged serves inference only (dropout > 0)")
    head_dim = query.shape[-1]
    scale = scaling if scaling is not None else 1.0 / math.sqrt(head_dim)
    B, Hq, q_len, _ = query.shape
    # Output allocated in the returned layout; the kernel writes it through a
    # (rows, heads, D) view, so no transpose copy follows.
    out = torch.empty((B, q_len, Hq, head_dim), dtype=query.dtype, device=query.device)

    graph = _current_graph()
    if graph is not None:
        if q_len != 1:
            raise ValueError(f"a graphed decode step has one query row per sequence, got "
                             f"{q_len}")
        pool = graph.pool
        K.paged_attention(query[:, :, 0], out[:, 0], pool.key_pool[module.layer_idx],
                          pool.value_pool[module.layer_idx], graph.tables, graph.ctx,
                          q_per_seq=1, scale=scale, causal=True)
        graph.used += 1
        return out, None

    varlen = _current_varlen()
    if varlen is not None:
        if B != 1 or q_len != len(varlen.seq_ids):
            raise ValueError(f"varlen pass expected one packed row of {len(varlen.seq_ids)} "
                             f"tokens, got {tuple(query.shape)}")
        meta = varlen.rows(Hq, query.device)
        _run(query[0].transpose(0, 1), out[0], varlen.pool, module.layer_idx, meta, scale)
        varlen.used += 1
        return out, None

    binding = _current()
    if binding is not None:
        if B != 1:
            raise ValueError(f"a paged cache binding is one sequence; got batch {B}")
        meta = binding.rows(q_len, query.device)
        _run(query[0].transpose(0, 1), out[0], binding.pool, module.layer_idx, meta, scale)
        binding.used += 1
        return out, None

    return _unbound(module, query, key, value, attention_mask, scale, out), None


def _unbound(module, query, key, value, attention_mask, scale, out):
    """Stage the handed K/V into a transient paged pool, then run the same kernel."""
    B, Hq, q_len, D = query.shape
    Hkv, kv_len = key.shape[1], key.shape[2]
    causal = bool(getattr(module, "is_causal", True))
    if attention_mask is not None:
        _require_plain(attention_mask, q_len, kv_len, causal)
    bs = 16
    nblk = (kv_len + bs - 1) // bs
    pool_k = torch.zeros((B * nblk, bs, Hkv, D), dtype=query.dtype, device=query.device)
    pool_v = torch.zeros_like(pool_k)
    tok = torch.arange(kv_len, device=query.device, dtype=torch.int32)
    for b in range(B):
        K.reshape_and_cache(key[b].transpose(0, 1), value[b].transpose(0, 1), pool_k, pool_v,
                            tok + b * nblk * bs)
    tables = torch.arange(B * nblk, device=query.device, dtype=torch.int32).view(B, nblk)
    kv = torch.full((B,), kv_len, device=query.device, dtype=torch.int32)
    rows = query.transpose(1, 2).reshape(B * q_len, Hq, D)
    K.paged_attention(rows, out.view(B * q_len, Hq, D), pool_k, pool_v, tables, kv,
                      q_per_seq=q_len, scale=scale, causal=causal)
    return out


def _require_plain(mask: torch.Tensor, q_len: int, kv_len: int, causal: bool) -> None:
    """Accept only the mask the kernel computes itself (bottom-right causal, or none)."""
    allowed = mask if mask.dtype == torch.bool else (mask == 0)
    allowed = allowed[..., :kv_len]
    if causal:
        rows = torch.arange(q_len, device=mask.device)[:, None] + (kv_len - q_len)
        want = torch.arange(kv_len, device=mask.device)[None, :] <= rows
    else:
        want = torch.ones((q_len, kv_len), dtype=torch.bool, device=mask.device)
    if not bool((allowed == want).all()):
        raise NotImplementedError(
            "memforge_paged: this attention mask (padding or a custom pattern) is not "
            "expressible by the paged kernel; bind a paged cache or pack the batch "
            "(varlen_attention_context) instead")


def paged_mask(batch_size: int, q_length: int, kv_length: int, q_offset: int = 0,
               kv_offset: int = 0, mask_function=None, attention_mask=None, **kwargs):
    """
    The mask hook for ``memforge_paged``: the kernel derives visibility from
    positions, so no mask tensor is ever built.  Unbound calls with padding or a
    non-causal mask function are rejected here, before the layers run.
    """
    if any_binding_active():
        return None
    from transformers.masking_utils import bidirectional_mask_function, causal_mask_function
    if mask_function not in (None, causal_mask_function, bidirectional_mask_function):
        raise NotImplementedError("memforge_paged: custom mask functions are not supported")
    if attention_mask is not None and not bool(attention_mask.all()):
        raise NotImplementedError("memforge_paged: padded batches are not supported unbound; "
                                  "pack them (varlen_attention_context)")
    return None


# ---------------------------------------------------------- registration

def register() -> bool:
    """
    Add the function and its mask hook to the transformers registries
    (idempotent).  Both go into the library-wide mappings (``register``), which
    is where mask creation looks an implementation up.
    """
    try:
        from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS
        from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    except ImportError:
        return False
    if ALL_ATTENTION_FUNCTIONS._global_mapping.get(BACKEND_NAME) is not paged_attention_forward:
        ALL_ATTENTION_FUNCTIONS.register(BACKEND_NAME, paged_attention_forward)
    if ALL_MASK_ATTENTION_FUNCTIONS._global_mapping.get(BACKEND_NAME) is not paged_mask:
        ALL_MASK_ATTENTION_FUNCTIONS.register(BACKEND_NAME, paged_mask)
    return True


def _configs(model):
    """The model config and any sub-config that carries its own attention choice."""
    found = [model.config]
    for name in ("text_config", "decoder"):
        sub = getattr(model.config, name, None)
        if sub is not None and hasattr(sub, "_attn_implementation"):
            found.append(sub)
    return found


def enable_on(model) -> bool:
    if not register():
        return False
    for cfg in _configs(model):
        cfg._attn_implementation = BACKEND_NAME
    return True


def is_enabled_on(model) -> bool:
    return getattr(model.config, "_attn_implementation", None) == BACKEND_NAME


@contextmanager
def backend_enabled_on(model):
    """Route ``model`` through ``memforge_paged`` for the duration of the block."""
    if not register():
        yield False
        return
    cfgs = _configs(model)
    saved = [getattr(c, "_attn_implementation", None) for c in cfgs]
    for c in cfgs:
        c._attn_implementation = BACKEND_NAME
    try:
        yield True
    finally:
        for c, s in zip(cfgs, saved):
            c._attn_implementation = s
