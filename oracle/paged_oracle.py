"""
CPU oracle for MemForge's paged-attention hot path.  TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, what the reference computes on the path this
project accelerates.  Only the test suite, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it, and
only as the checker or as the timed CPU baseline.  The product path
(``memforge_b200``) never calls it: a missing CUDA extension is an error there,
not a reason to come here.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference's own
functions on seeded inputs and stores their outputs under ``tests/golden``;
``tests/test_oracle.py`` checks every function below against those fixtures and
against the known-answer vectors written in the reference's test files.

Conventions
-----------
* bf16 / fp16 tensors are carried as numpy ``uint16`` bit patterns (bf16) or
  ``float16`` (fp16); attention arithmetic is always fp32, as the reference does
  (``block_attention.py:96``, ``varlen_attention.py:133``).
* The KV pool per layer is ``(num_blocks, block_size, num_kv_heads, head_dim)``
  (``memforge_ml/runtime/kv_pool.py:66``).  Viewed flat it is
  ``(num_blocks * block_size, num_kv_heads, head_dim)``
  (``memforge_ml/kernels/paged_gather.py:81-82``).
"""

from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple

import numpy as np

# --------------------------------------------------------------------------
# bf16 bit-pattern helpers (byte work; exact)
# --------------------------------------------------------------------------


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """Widen bf16 bit patterns (uint16) to float32 exactly."""
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """
    Round float32 to bf16 (round-to-nearest-even), returned as uint16 bits.

    This is the IEEE rounding torch applies in ``tensor.to(torch.bfloat16)``,
    which the reference's ``scatter_kv`` uses to cast into the pool dtype
    (``paged_gather.py:113-114``).  Every NaN becomes torch's canonical 0x7FC0.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    rounded = ((u + 0x7FFF + lsb) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        rounded = np.where(nan, np.uint16(0x7FC0), rounded)
    return rounded.astype(np.uint16)


def to_f32(arr: np.ndarray, dtype: str) -> np.ndarray:
    """Decode a stored tensor ('f32' | 'f16' | 'bf16') to float32."""
    if dtype == "bf16":
        return bf16_to_f32(arr)
    return np.asarray(arr).astype(np.float32)


def from_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    """Encode float32 into the stored representation of ``dtype``."""
    if dtype == "bf16":
        return f32_to_bf16(x)
    if dtype == "f16":
        return np.asarray(x, dtype=np.float32).astype(np.float16)
    return np.asarray(x, dtype=np.float32).copy()


# --------------------------------------------------------------------------
# (a1) slot arithmetic — integer, exact
# --------------------------------------------------------------------------


def slot_indices(block_table: np.ndarray, start: int, end: int,
                 block_size: int) -> Tuple[np.ndarray, np.ndarray]:
    """
    Logical token range ``[start, end)`` -> (physical block, slot) arrays.

    Follows ``PagedKVPool.slot_indices`` (``kv_pool.py:92-110``): logical block
    ``pos // block_size``, slot ``pos % block_size``, and an IndexError when a
    position falls past the block table.
    """
    table = np.asarray(block_table, dtype=np.int64)
    positions = np.arange(start, end, dtype=np.int64)
    logical = positions // block_size
    slots = positions % block_size
    if logical.size and int(logical.max()) >= table.size:
        raise IndexError(
            f"logical block {int(logical.max())} is outside a block table of "
            f"{table.size} entries (token range {start}:{end})"
        )
    return table[logical], slots


def flat_slot_index(physical: np.ndarray, slots: np.ndarray,
                    block_size: int) -> np.ndarray:
    """``physical * block_size + slot`` (``paged_gather.py:42-55``)."""
    return (np.asarray(physical, dtype=np.int64) * block_size
            + np.asarray(slots, dtype=np.int64))


def flat_indices(block_table: np.ndarray, start: int, end: int,
                 block_size: int) -> np.ndarray:
    """``PagedKVPool.flat_indices`` (``kv_pool.py:116-130``)."""
    physical, slots = slot_indices(block_table, start, end, block_size)
    return flat_slot_index(physical, slots, block_size)


# --------------------------------------------------------------------------
# (a2) reshape_and_cache — byte copy, exact
# --------------------------------------------------------------------------


def scatter_kv(key_pool: np.ndarray, value_pool: np.ndarray, layer_idx: int,
               flat_index: np.ndarray, keys: np.ndarray, values: np.ndarray,
               pool_dtype: str, src_dtype: str) -> None:
    """
    In-place scatter of ``(1, H, T, D)`` keys/values into the flat pool.

    Follows ``paged_gather.scatter_kv`` (``paged_gather.py:92-117``): permute
    to ``(T, H, D)``, cast to the pool dtype, ``index_copy_`` at ``flat_index``
    on the layer's ``(num_blocks*block_size, H, D)`` view.  Arrays carry the
    storage representation of their dtype (see module docstring).  Slots equal
    to -1 are skipped, which is the C ABI's convention for padding rows (the
    reference has no padding rows, so it never produces -1).
    """
    nb, bs = key_pool.shape[1], key_pool.shape[2]
    flat_k = key_pool[layer_idx].reshape(nb * bs, *key_pool.shape[3:])
    flat_v = value_pool[layer_idx].reshape(nb * bs, *value_pool.shape[3:])
    k = np.transpose(keys[0], (1, 0, 2))
    v = np.transpose(values[0], (1, 0, 2))
    if src_dtype != pool_dtype:
        k = from_f32(to_f32(k, src_dtype), pool_dtype)
        v = from_f32(to_f32(v, src_dtype), pool_dtype)
    idx = np.asarray(flat_index, dtype=np.int64)
    keep = idx >= 0
    flat_k[idx[keep]] = k[keep]
    flat_v[idx[keep]] = v[keep]


def commit_accepted(key_pool: np.ndarray, value_pool: np.ndarray,
                    layer_idx: int, block_table: np.ndarray,
                    context_length: int, keys: np.ndarray, values: np.ndarray,
                    num_confirmed: int, block_size: int, dtype: str) -> None:
    """
    Write only the confirmed prefix of a speculative window into the pool.

    Follows ``scatter_accepted_kv`` (``batched_speculative.py:780-811``):
    positions ``context_length .. context_length+num_confirmed-1`` receive the
    first ``num_confirmed`` window tokens; rejected slots are left untouched.
    ``keys``/``values`` are ``(1, H, K+1, D)``.
    """
    if num_confirmed <= 0:
        return
    flat = flat_indices(block_table, context_length,
                        context_length + num_confirmed, block_size)
    scatter_kv(key_pool, value_pool, layer_idx, flat,
               keys[:, :, :num_confirmed], values[:, :, :num_confirmed],
               dtype, dtype)


def copy_block(key_pool: np.ndarray, value_pool: np.ndarray, src: int,
               dst: int) -> None:
    """All-layer block copy for copy-on-write (``prefix_sharing.py:28-42``)."""
    if src == dst:
        return
    key_pool[:, dst] = key_pool[:, src]
    value_pool[:, dst] = value_pool[:, src]


# --------------------------------------------------------------------------
# (a4, a5) attention — fp32
# --------------------------------------------------------------------------


def group_by_sequence(seq_ids: Sequence[int]) -> List[Tuple[int, List[int]]]:
    """Rows per sequence in first-seen order (``varlen_attention.py:60-75``)."""
    order: List[int] = []
    rows: dict = {}
    for row, seq_id in enumerate(seq_ids):
        if seq_id not in rows:
            rows[seq_id] = []
            order.append(seq_id)
        rows[seq_id].append(row)
    return [(s, rows[s]) for s in order]


def varlen_attention(query: np.ndarray, key_pool: np.ndarray,
                     value_pool: np.ndarray, layer_idx: int,
                     block_tables: Sequence[np.ndarray],
                     seq_ids: Sequence[int], positions: Sequence[int],
                     block_size: int, scale: Optional[float] = None,
                     window: Optional[dict] = None) -> np.ndarray:
    """
    Packed multi-sequence paged attention, fp32.  Returns ``(H, T, D)`` fp32.

    Follows ``paged_attention_varlen_materialised`` (``varlen_attention.py:
    291-395``): validation (``:325-344``), per-sequence gather of positions
    ``0..max(p)`` through the block table (``:351-377``), GQA by repeating each
    KV head ``group`` times (``:378-380``), scores ``q.k * scale`` (``:382-383``),
    the mask ``key_pos <= query_pos`` (``:388-390``), softmax and the weighted
    sum (``:392-393``).

    ``query`` is fp32 ``(H, T, D)``; pools are fp32
    ``(layers, blocks, slots, Hkv, D)``.

    ``window`` (optional) models the speculative-verify side buffer: a dict of
    ``{seq_id: (start, k_win (Hkv, W, D), v_win (Hkv, W, D))}`` whose keys at
    positions ``start .. start+W-1`` come from the window instead of the pool,
    as if they had been written there first (the reference's single-sequence
    verify writes them, ``speculative_runtime.py:250-265``).
    """
    num_heads, total, head_dim = query.shape
    if len(seq_ids) != total or len(positions) != total:
        raise ValueError(
            f"{total} query tokens but {len(seq_ids)} seq_ids and "
            f"{len(positions)} positions"
        )
    if total == 0:
        raise ValueError("paged_attention_varlen requires at least one query token")
    if any(p < 0 for p in positions):
        raise ValueError(f"negative query position in {list(positions)}")
    num_kv_heads = key_pool.shape[3]
    if num_heads % num_kv_heads != 0:
        raise ValueError(
            f"{num_heads} query heads is not a multiple of {num_kv_heads} kv heads"
        )
    group = num_heads // num_kv_heads
    scale = scale if scale is not None else 1.0 / math.sqrt(head_dim)

    out = np.zeros((num_heads, total, head_dim), dtype=np.float32)
    nb, bs = key_pool.shape[1], key_pool.shape[2]
    flat_k = key_pool[layer_idx].reshape(nb * bs, num_kv_heads, head_dim)
    flat_v = value_pool[layer_idx].reshape(nb * bs, num_kv_heads, head_dim)
    for seq_id, rows in group_by_sequence(seq_ids):
        if seq_id < 0 or seq_id >= len(block_tables):
            raise IndexError(
                f"seq_id {seq_id} has no block table (got {len(block_tables)})"
            )
        table = np.asarray(block_tables[seq_id], dtype=np.int64)
        row_pos = np.asarray([positions[r] for r in rows], dtype=np.int64)
        ctx = int(row_pos.max()) + 1
        needed = (ctx + block_size - 1) // block_size
        if needed > table.size:
            raise IndexError(
                f"sequence {seq_id} reads up to position {ctx - 1}, "
                f"needing {needed} blocks, but its block table has "
                f"{table.size} entries"
            )
        flat = flat_indices(table, 0, ctx, block_size)
        keys = flat_k[flat].astype(np.float32)       # (ctx, Hkv, D)
        values = flat_v[flat].astype(np.float32)
        if window is not None and seq_id in window:
            start, kw, vw = window[seq_id]
            width = kw.shape[1]
            hi = min(ctx, start + width)
            if hi > start:
                keys[start:hi] = np.transpose(kw, (1, 0, 2))[: hi - start]
                values[start:hi] = np.transpose(vw, (1, 0, 2))[: hi - start]
        keys = np.repeat(np.transpose(keys, (1, 0, 2)), group, axis=0)   # (H, ctx, D)
        values = np.repeat(np.transpose(values, (1, 0, 2)), group, axis=0)
        q = query[:, rows, :].astype(np.float32)                          # (H, R, D)
        scores = np.matmul(q, np.transpose(keys, (0, 2, 1))) * np.float32(scale)
        visible = np.arange(ctx)[None, :] <= row_pos[:, None]             # (R, ctx)
        scores = np.where(visible[None], scores, -np.inf).astype(np.float32)
        mx = scores.max(axis=-1, keepdims=True)
        e = np.exp(scores - mx)
        w = e / e.sum(axis=-1, keepdims=True)
        out[:, rows, :] = np.matmul(w.astype(np.float32), values)
    return out


def decode_attention(q: np.ndarray, key_flat: np.ndarray, value_flat: np.ndarray,
                     block_tables: np.ndarray, ctx_lens: Sequence[int],
                     block_size: int, scale: float) -> np.ndarray:
    """
    Single-token paged decode, ``[B, Hq, D]`` fp32 out.

    The contract of ``paged_decode_attention`` (``triton_paged_decode.py:
    129-176``): ``ctx_lens`` counts the new token, ``key_flat`` is one layer's
    pool viewed ``(slots, Hkv, D)``.  Computed as the materialised softmax the
    reference's own test compares the Triton kernel to
    (``tests/python/test_triton_paged_decode.py:10-25``).
    """
    B, Hq, D = q.shape
    Hkv = key_flat.shape[1]
    G = Hq // Hkv
    out = np.zeros((B, Hq, D), dtype=np.float32)
    for b in range(B):
        n = int(ctx_lens[b])
        pos = np.arange(n)
        slots = np.asarray(block_tables[b], dtype=np.int64)[pos // block_size] * block_size + pos % block_size
        k = key_flat[slots].astype(np.float32)          # (n, Hkv, D)
        v = value_flat[slots].astype(np.float32)
        qb = q[b].astype(np.float32).reshape(Hkv, G, D)
        s = np.einsum("hgd,nhd->hgn", qb, k) * np.float32(scale)
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=-1, keepdims=True)
        out[b] = np.einsum("hgn,nhd->hgd", p, v).reshape(Hq, D)
    return out


def standalone_paged_attention(query: np.ndarray, key_cache: np.ndarray,
                               value_cache: np.ndarray, block_table: Sequence[int],
                               context_len: int, scale: Optional[float] = None,
                               probs_dtype: str = "f32") -> np.ndarray:
    """
    ``PagedAttention.forward`` (``memforge_ml/models/paged_attention.py:108-141``).

    The standalone operator's cache layout is ``(num_blocks, H, block_size, D)``
    (``:34-43``).  Every query row sees all ``context_len`` keys (no causal
    mask), probabilities are cast to the query dtype before the value product
    (``:133``), and the result is ``(1, q_len, H*D)``.  ``query`` is fp32
    ``(1, H, q_len, D)``; a ``scale`` of 0/None means ``1/sqrt(D)`` (``:119``).
    Grouped-query attention is applied when H is a multiple of the cache's
    head count (the reference itself supports only H equal to it).
    """
    head_dim = query.shape[-1]
    scale = scale or (1.0 / math.sqrt(head_dim))
    bs = key_cache.shape[2]
    nblk = (context_len + bs - 1) // bs
    ks, vs = [], []
    for logical in range(nblk):
        phys = int(block_table[logical])
        n = min(bs, context_len - logical * bs)
        ks.append(key_cache[phys, :, :n, :].astype(np.float32))
        vs.append(value_cache[phys, :, :n, :].astype(np.float32))
    keys = np.concatenate(ks, axis=1)      # (Hc, ctx, D)
    values = np.concatenate(vs, axis=1)
    q = query[0].astype(np.float32)        # (H, q, D)
    group = q.shape[0] // keys.shape[0]
    if group > 1:
        keys = np.repeat(keys, group, axis=0)
        values = np.repeat(values, group, axis=0)
    s = np.matmul(q, np.transpose(keys, (0, 2, 1))) * np.float32(scale)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    p = to_f32(from_f32(p, probs_dtype), probs_dtype)
    o = np.matmul(p, values)               # (H, q, D)
    H, qlen, D = o.shape
    return np.transpose(o, (1, 0, 2)).reshape(1, qlen, H * D)


# --------------------------------------------------------------------------
# (f3) speculative acceptance — integer decision, exact given the uniforms
# --------------------------------------------------------------------------


def accepted_drafts(draft_tokens: Sequence[int], target_probs: Optional[np.ndarray] = None,
                    draft_probs: Optional[np.ndarray] = None,
                    uniforms: Optional[Sequence[float]] = None,
                    target_tokens: Optional[Sequence[int]] = None) -> int:
    """
    Number of leading accepted drafts of one sequence.

    Sampling (``RejectionSampler.verify_tokens``, ``rejection_sampler.py:46-66``):
    draft i is accepted when ``r_i <= min(1, p(x_i) / (q(x_i) + 1e-9))`` with the
    reference's Python-float (double) arithmetic; the uniforms ``r_i`` are given
    instead of drawn.  Greedy (temperature 0, ``batched_speculative.py:744-757``):
    point-mass distributions, so draft i is accepted while it equals the target's
    argmax at slot i.
    """
    n = 0
    for i, x in enumerate(draft_tokens):
        x = int(x)
        if target_probs is None:
            ok = x == int(target_tokens[i])
        else:
            p = float(target_probs[i][x])
            q = float(draft_probs[i][x])
            ok = float(uniforms[i]) <= min(1.0, p / (q + 1e-9))
        if not ok:
            break
        n += 1
    return n


def inverse_cdf_draw(weights: np.ndarray, u: float) -> Optional[int]:
    """
    Token drawn from unnormalised non-negative ``weights`` at uniform ``u``: the
    smallest v with ``cumsum(weights)[v] > u * sum(weights)`` (float64), or None
    when the weights sum to zero.  ``sample_from_probs``
    (``rejection_sampler.py:13-26``) draws from the same distribution with
    ``torch.multinomial``; a given ``u`` makes the draw reproducible.
    """
    w = np.maximum(np.asarray(weights, dtype=np.float64), 0.0)
    total = w.sum()
    if not total > 0:
        return None
    c = np.cumsum(w)
    return int(min(np.searchsorted(c, u * total, side="right"), len(w) - 1))


def next_token_after(accepted: int, num_drafts: int, target_probs: np.ndarray,
                     draft_probs: np.ndarray, u: float) -> int:
    """
    The token that follows the accepted drafts (``rejection_sampler.py:67-84``):
    after a rejection at slot a, a draw from ``clamp(p_a - q_a, 0)`` (from
    ``p_a`` when that is all zero); after all K accepted, the bonus draw from
    ``p_K``.
    """
    if accepted < num_drafts:
        tok = inverse_cdf_draw(target_probs[accepted] - draft_probs[accepted], u)
        if tok is None:
            tok = inverse_cdf_draw(target_probs[accepted], u)
    else:
        tok = inverse_cdf_draw(target_probs[num_drafts], u)
    if tok is None:
        tok = min(len(target_probs[0]) - 1, int(u * len(target_probs[0])))
    return tok
