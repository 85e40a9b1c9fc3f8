"""
Host-side planning of a packed varlen pass (pure Python/numpy; no GPU).

MemForge describes a packed pass per query row: the sequence it belongs to
(``seq_ids``), its absolute position (``positions``) and one block table per
sequence (``memforge_ml/kernels/varlen_attention.py:78-110``).  The kernels take
per-segment metadata instead: a segment is a run of rows of one sequence at
consecutive positions ``p0 .. p0+n-1``, which sees keys ``0 .. p0+i`` for its
row i.  This module validates the row form exactly as the reference does
(same exception types and messages, ``varlen_attention.py:111-158``) and cuts it
into segments:

* rows are grouped per sequence in first-seen order (``group_by_sequence``,
  ``varlen_attention.py:60-75``), sorted by position, and split wherever
  positions are not consecutive;
* ``row_map`` sends segment-ordered row r to its packed row (None when the
  packing already is segment order);
* each segment gets the sequence's block table, ``kv_len = last position + 1``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import numpy as np


def group_by_sequence(seq_ids: Sequence[int]) -> List[Tuple[int, List[int]]]:
    """Rows per sequence, first-seen order (``varlen_attention.py:60-75``)."""
    order: List[int] = []
    rows: dict = {}
    for row, seq_id in enumerate(seq_ids):
        if seq_id not in rows:
            rows[seq_id] = []
            order.append(seq_id)
        rows[seq_id].append(row)
    return [(s, rows[s]) for s in order]


@dataclass
class VarlenPlan:
    tables: np.ndarray        # int32 [S, W]
    cu_seqlens: np.ndarray    # int32 [S + 1]
    kv_lens: np.ndarray       # int32 [S]
    row_map: Optional[np.ndarray]  # int32 [T] or None (identity)
    max_q_len: int
    total: int

    @property
    def num_segments(self) -> int:
        return int(self.kv_lens.shape[0])

    def packed(self) -> Tuple[np.ndarray, dict]:
        """All arrays in one int32 buffer (one host->device copy) plus offsets."""
        parts = [("tables", self.tables.reshape(-1)), ("cu", self.cu_seqlens),
                 ("kv", self.kv_lens)]
        if self.row_map is not None:
            parts.append(("row_map", self.row_map))
        offs, at = {}, 0
        for name, arr in parts:
            offs[name] = (at, arr.size)
            at += arr.size
        buf = np.empty(at, dtype=np.int32)
        for name, arr in parts:
            o, n = offs[name]
            buf[o:o + n] = arr
        return buf, offs


def _table_list(block_tables) -> List[np.ndarray]:
    out = []
    for t in block_tables:
        if hasattr(t, "detach"):
            t = t.detach().cpu().numpy()
        out.append(np.asarray(t, dtype=np.int64).reshape(-1))
    return out


def plan_varlen(total: int, block_tables, seq_ids: Sequence[int], positions: Sequence[int],
                block_size: int, num_heads: int, num_kv_heads: int) -> VarlenPlan:
    """Validate a packed pass like the reference and cut it into segments."""
    if len(seq_ids) != total or len(positions) != total:
        raise ValueError(
            f"{total} query tokens but {len(seq_ids)} seq_ids and "
            f"{len(positions)} positions"
        )
    if total == 0:
        raise ValueError("paged_attention_varlen requires at least one query token")
    if any(p < 0 for p in positions):
        raise ValueError(f"negative query position in {list(positions)}")
    if num_heads % num_kv_heads != 0:
        raise ValueError(
            f"{num_heads} query heads is not a multiple of {num_kv_heads} kv heads"
        )
    tables = _table_list(block_tables)
    seg_tables: List[np.ndarray] = []
    seg_lens: List[int] = []
    kv_lens: List[int] = []
    order: List[int] = []
    for seq_id, rows in group_by_sequence(seq_ids):
        if seq_id < 0 or seq_id >= len(tables):
            raise IndexError(
                f"seq_id {seq_id} has no block table (got {len(tables)})"
            )
        table = tables[seq_id]
        last_key = max(positions[r] for r in rows)
        needed = (last_key + 1 + block_size - 1) // block_size
        if needed > table.size:
            raise IndexError(
                f"sequence {seq_id} reads up to position {last_key}, needing "
                f"{needed} blocks, but its block table has {table.size} entries"
            )
        rows_sorted = sorted(rows, key=lambda r: (positions[r], r))
        run: List[int] = []
        for r in rows_sorted:
            if run and positions[r] != positions[run[-1]] + 1:
                seg_tables.append(table)
                seg_lens.append(len(run))
                kv_lens.append(positions[run[-1]] + 1)
                order.extend(run)
                run = []
            run.append(r)
        seg_tables.append(table)
        seg_lens.append(len(run))
        kv_lens.append(positions[run[-1]] + 1)
        order.extend(run)
    width = max(1, max(t.size for t in seg_tables))
    tab = np.zeros((len(seg_tables), width), dtype=np.int32)
    for i, t in enumerate(seg_tables):
        tab[i, :t.size] = t
    cu = np.zeros(len(seg_lens) + 1, dtype=np.int32)
    cu[1:] = np.cumsum(seg_lens)
    row_map = np.asarray(order, dtype=np.int32)
    identity = bool(np.array_equal(row_map, np.arange(total, dtype=np.int32)))
    return VarlenPlan(tables=tab, cu_seqlens=cu, kv_lens=np.asarray(kv_lens, np.int32),
                      row_map=None if identity else row_map, max_q_len=max(seg_lens),
                      total=total)
