"""
transformers attention-registry backend, B200 edition of
``memforge_ml/kernels/attention_backend.py``.

Registers ``memforge_paged`` in ``ALL_ATTENTION_FUNCTIONS`` (and aliases eager's
mask builder, ``attention_backend.py:360-401``).  The registered function has the
reference's contract (``attention_backend.py:195-272``):

* inside ``varlen_attention_context`` (a packed prefill+decode pass) every layer
  runs the varlen kernel over the bound pool, tables, seq_ids and positions;
* inside ``paged_attention_context`` a single-query, unmasked decode reads the
  bound sequence's pool pages directly;
* otherwise it computes plain attention over the ``key``/``value`` it was
  handed (prefill, padded batches) and counts a fallback.

Returns ``(B, q_len, H, D)`` (``attention_backend.py:275-292``).
"""

from __future__ import annotations

import math
import threading
from contextlib import contextmanager
from typing import Any, Optional, Tuple

import torch

from .block_attention import paged_attention_blockwise
from .varlen_attention import paged_attention_varlen, paged_attention_varlen_materialised

BACKEND_NAME = "memforge_paged"

_state = threading.local()


class _Binding:
    """Pool + one sequence's cache; ``context_length`` is read at attention time."""

    __slots__ = ("pool", "cache", "used", "fallbacks")

    def __init__(self, pool, cache):
        self.pool = pool
        self.cache = cache
        self.used = 0
        self.fallbacks = 0

    @property
    def block_table(self) -> torch.Tensor:
        return self.cache.block_table_tensor_cached()

    @property
    def context_length(self) -> int:
        return self.cache.position


class _VarlenBinding:
    """A packed multi-sequence pass: per-row sequence ids and positions."""

    __slots__ = ("pool", "block_tables", "seq_ids", "positions", "used", "block_wise")

    def __init__(self, pool, block_tables, seq_ids, positions, block_wise=False):
        self.pool = pool
        self.block_tables = list(block_tables)
        self.seq_ids = list(seq_ids)
        self.positions = list(positions)
        self.block_wise = bool(block_wise)
        self.used = 0


def _current() -> Optional[_Binding]:
    return getattr(_state, "binding", None)


def _current_varlen() -> Optional[_VarlenBinding]:
    return getattr(_state, "varlen", None)


@contextmanager
def paged_attention_context(pool, cache):
    previous = _current()
    binding = _Binding(pool, cache)
    _state.binding = binding
    try:
        yield binding
    finally:
        _state.binding = previous


@contextmanager
def varlen_attention_context(pool, block_tables, seq_ids, positions, block_wise=False):
    previous = _current_varlen()
    binding = _VarlenBinding(pool, block_tables, seq_ids, positions, block_wise=block_wise)
    _state.varlen = binding
    try:
        yield binding
    finally:
        _state.varlen = previous


def _mask_is_permissive(attention_mask: Optional[torch.Tensor]) -> bool:
    if attention_mask is None:
        return True
    if attention_mask.dtype == torch.bool:
        return bool(attention_mask.all())
    return bool(torch.all(attention_mask == 0))


def paged_attention_forward(module: Any, query: torch.Tensor, key: torch.Tensor,
                            value: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                            scaling: Optional[float] = None, dropout: float = 0.0,
                            **kwargs: Any) -> Tuple[torch.Tensor, None]:
    varlen = _current_varlen()
    if varlen is not None:
        if query.shape[0] != 1 or query.shape[2] != len(varlen.seq_ids):
            raise ValueError(
                f"varlen pass expected one packed row of {len(varlen.seq_ids)} tokens, got "
                f"{tuple(query.shape)}")
        varlen.used += 1
        if varlen.block_wise:
            out = paged_attention_varlen(query, varlen.pool.key_pool, varlen.pool.value_pool,
                                         module.layer_idx, varlen.block_tables, varlen.seq_ids,
                                         varlen.positions, varlen.pool.block_size, scale=scaling)
        else:
            out = paged_attention_varlen_materialised(query, varlen.pool, module.layer_idx,
                                                      varlen.block_tables, varlen.seq_ids,
                                                      varlen.positions, scale=scaling)
        return _to_attention_output_layout(out), None

    binding = _current()
    single_query = query.shape[0] == 1 and query.shape[2] == 1
    if (binding is not None and single_query and _mask_is_permissive(attention_mask)
            and binding.context_length > 0):
        binding.used += 1
        out = paged_attention_blockwise(query, binding.pool.key_pool, binding.pool.value_pool,
                                        module.layer_idx, binding.block_table,
                                        binding.context_length, binding.pool.block_size,
                                        scale=scaling)
        return _to_attention_output_layout(out), None

    if binding is not None:
        binding.fallbacks += 1
    return _eager_attention(query, key, value, attention_mask, scaling), None


def _to_attention_output_layout(attn_output: torch.Tensor) -> torch.Tensor:
    """(batch, heads, q_len, D) -> (batch, q_len, heads, D)."""
    return attn_output.transpose(1, 2).contiguous()


def _eager_attention(query, key, value, attention_mask, scaling):
    """Plain scaled dot-product attention with GQA expansion (``attention_backend.py:295-326``)."""
    num_heads, head_dim = query.shape[1], query.shape[3]
    scaling = scaling if scaling is not None else 1.0 / math.sqrt(head_dim)
    group = num_heads // key.shape[1]
    k, v = key, value
    if group > 1:
        k = k.repeat_interleave(group, dim=1)
        v = v.repeat_interleave(group, dim=1)
    scores = torch.matmul(query, k.transpose(2, 3)) * scaling
    if attention_mask is not None:
        scores = scores + attention_mask[:, :, :, : k.shape[-2]]
    else:
        q_len, kv_len = scores.shape[-2], scores.shape[-1]
        if q_len > 1:
            causal = torch.ones(q_len, kv_len, dtype=torch.bool, device=scores.device).tril(
                diagonal=kv_len - q_len)
            scores = scores.masked_fill(~causal, torch.finfo(scores.dtype).min)
    weights = torch.softmax(scores, dim=-1, dtype=torch.float32).to(query.dtype)
    return _to_attention_output_layout(torch.matmul(weights, v))


def register() -> bool:
    """Add the backend and its mask alias to the transformers registries (idempotent)."""
    try:
        from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    except ImportError:
        return False
    try:
        if BACKEND_NAME not in ALL_ATTENTION_FUNCTIONS:
            ALL_ATTENTION_FUNCTIONS[BACKEND_NAME] = paged_attention_forward
    except Exception:
        return False
    try:
        from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS
        if BACKEND_NAME not in ALL_MASK_ATTENTION_FUNCTIONS:
            ALL_MASK_ATTENTION_FUNCTIONS[BACKEND_NAME] = ALL_MASK_ATTENTION_FUNCTIONS["eager"]
    except Exception:
        return False
    return True


def _attn_config_holders(model):
    holders = [model.config]
    for attr in ("text_config", "decoder"):
        sub = getattr(model.config, attr, None)
        if sub is not None and hasattr(sub, "_attn_implementation"):
            holders.append(sub)
    return holders


def enable_on(model) -> bool:
    if not register():
        return False
    for holder in _attn_config_holders(model):
        holder._attn_implementation = BACKEND_NAME
    return True


def is_enabled_on(model) -> bool:
    return getattr(model.config, "_attn_implementation", None) == BACKEND_NAME


@contextmanager
def backend_enabled_on(model):
    if not register():
        yield False
        return
    holders = _attn_config_holders(model)
    previous = [getattr(h, "_attn_implementation", None) for h in holders]
    for holder in holders:
        holder._attn_implementation = BACKEND_NAME
    try:
        yield True
    finally:
        for holder, original in zip(holders, previous):
            holder._attn_implementation = original
