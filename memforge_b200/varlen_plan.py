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
* each segment gets its sequence's block table, ``kv_len = last position + 1``;
  ``table_index`` says where each segment's block ids sit in the concatenation
  of all tables, so device tables are assembled on the device (one gather).
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
    seg_seq: np.ndarray       # int32 [S]: the sequence each segment belongs to
    needed: np.ndarray        # int32 [S]: blocks segment s reads (its table prefix)
    cu_seqlens: np.ndarray    # int32 [S + 1]
    kv_lens: np.ndarray       # int32 [S]
    row_map: Optional[np.ndarray]  # int32 [T] or None (identity)
    max_q_len: int
    total: int

    @property
    def num_segments(self) -> int:
        return int(self.kv_lens.shape[0])

    @property
    def uniform_q(self) -> int:
        """
        The common query-run length when every segment has the same number of
        rows and the rows are already in segment order (no row map), else 0.
        Such a batch is passed as ``q_per_seq``: the attention call then needs
        no per-segment offsets, and a batch of long runs is one launch.
        """
        q = np.diff(self.cu_seqlens)
        if self.row_map is not None or q.size == 0 or (q != q[0]).any():
            return 0
        return int(q[0])

    @property
    def width(self) -> int:
        return max(1, int(self.needed.max()))

    def table_index(self, sizes: Sequence[int]) -> np.ndarray:
        """
        int64 ``[S, width]``: for the concatenation of every sequence's table
        (in sequence-id order, ``sizes`` entries each) followed by one zero, the
        position of segment s's j-th block id (the zero past its needed prefix).
        """
        offs = np.zeros(len(sizes) + 1, dtype=np.int64)
        offs[1:] = np.cumsum(sizes)
        idx = np.full((self.num_segments, self.width), offs[-1], dtype=np.int64)
        for i, (sq, n) in enumerate(zip(self.seg_seq, self.needed)):
            idx[i, :n] = offs[sq] + np.arange(n)
        return idx

    def host_tables(self, block_tables) -> np.ndarray:
        """int32 ``[S, width]`` block ids from host-side tables."""
        flat = [np.asarray(_host(t), dtype=np.int64).reshape(-1) for t in block_tables]
        cat = np.concatenate(flat + [np.zeros(1, np.int64)])
        return cat[self.table_index([f.size for f in flat])].astype(np.int32)

    def packed(self, block_tables) -> Tuple[np.ndarray, dict]:
        """Host tables and every other int32 array in one buffer, plus offsets."""
        parts = [("tables", self.host_tables(block_tables).reshape(-1)),
                 ("cu", self.cu_seqlens), ("kv", self.kv_lens)]
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


def _host(t):
    if hasattr(t, "detach"):
        return t.detach().cpu().numpy()
    return t


def _numel(t) -> int:
    if hasattr(t, "numel"):
        return int(t.numel())
    return int(np.asarray(t).size)


def plan_varlen(total: int, block_tables, seq_ids: Sequence[int], positions: Sequence[int],
                block_size: int, num_heads: int, num_kv_heads: int) -> VarlenPlan:
    """
    Validate a packed pass like the reference and cut it into segments.  Only
    the tables' lengths are read here, never their contents, so device tables
    cost no synchronisation.
    """
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
    sizes = [_numel(t) for t in block_tables]
    seg_seq: List[int] = []
    seg_lens: List[int] = []
    kv_lens: List[int] = []
    order: List[int] = []
    for seq_id, rows in group_by_sequence(seq_ids):
        if seq_id < 0 or seq_id >= len(sizes):
            raise IndexError(
                f"seq_id {seq_id} has no block table (got {len(sizes)})"
            )
        last_key = max(positions[r] for r in rows)
        needed = (last_key + 1 + block_size - 1) // block_size
        if needed > sizes[seq_id]:
            raise IndexError(
                f"sequence {seq_id} reads up to position {last_key}, needing "
                f"{needed} blocks, but its block table has {sizes[seq_id]} entries"
            )
        rows_sorted = sorted(rows, key=lambda r: (positions[r], r))
        run: List[int] = []
        for r in rows_sorted + [None]:
            if run and (r is None or positions[r] != positions[run[-1]] + 1):
                seg_seq.append(seq_id)
                seg_lens.append(len(run))
                kv_lens.append(positions[run[-1]] + 1)
                order.extend(run)
                run = []
            if r is not None:
                run.append(r)
    cu = np.zeros(len(seg_lens) + 1, dtype=np.int32)
    cu[1:] = np.cumsum(seg_lens)
    kv = np.asarray(kv_lens, np.int32)
    row_map = np.asarray(order, dtype=np.int32)
    identity = bool(np.array_equal(row_map, np.arange(total, dtype=np.int32)))
    return VarlenPlan(seg_seq=np.asarray(seg_seq, np.int32),
                      needed=((kv + block_size - 1) // block_size).astype(np.int32),
                      cu_seqlens=cu, kv_lens=kv,
                      row_map=None if identity else row_map, max_q_len=max(seg_lens),
                      total=total)
