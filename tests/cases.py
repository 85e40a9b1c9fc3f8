"""
Seeded synthetic inputs shared by the golden-fixture generator, the CPU tests,
the GPU parity tests and ``bench.py``.

Everything here is numpy (PCG64), so the same seed yields the same bytes on
any machine; the golden fixtures therefore store only outputs plus a checksum of
the inputs they were made from.

The five ``config*`` builders restate BASELINE.json's workloads:

1. decode, SmolLM2-360M layer: Hq 15, Hkv 5, D 64, fp32, B 8, ctx ~U[16,512]
2. KV write + decode, Llama-3-8B: Hq 32, Hkv 8, D 128, bf16, B 64,
   ctx ~U[256,4096], 16384-block pool
3. chunked prefill (16 seqs, prompt ~U[128,2048] in 512-token chunks over a
   prefix ~U[0,1024]) mixed with 48 decodes ctx ~U[256,4096]
4. speculative verify, Qwen2.5-14B: Hq 40, Hkv 8, B 32, ctx ~U[512,8192],
   5-token window, accepted ~U[0,4]
5. long-context decode, Llama-3-70B: Hq 64, Hkv 8, B 256,
   ctx log-uniform [4096,32768]
"""

from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

BLOCK = 16


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def checksum(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()[:16]


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 values rounded to the nearest bf16 (returned as fp32)."""
    from oracle.paged_oracle import bf16_to_f32, f32_to_bf16
    return bf16_to_f32(f32_to_bf16(x))


def normal(g: np.random.Generator, shape, std: float = 1.0) -> np.ndarray:
    return (g.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


def disjoint_tables(g: np.random.Generator, lengths: List[int], num_blocks: int,
                    block_size: int = BLOCK, pad_to: Optional[int] = None) -> np.ndarray:
    """
    One block table per sequence, a non-overlapping slice of a seeded
    permutation of the pool (BASELINE config 1's recipe).  Returns int32
    ``[B, max_blocks]`` padded with -1.
    """
    need = [(n + block_size - 1) // block_size for n in lengths]
    if sum(need) > num_blocks:
        raise ValueError(f"{sum(need)} blocks needed, pool has {num_blocks}")
    perm = g.permutation(num_blocks).astype(np.int32)
    width = pad_to if pad_to is not None else max(max(need), 1)
    tables = np.full((len(lengths), width), -1, dtype=np.int32)
    at = 0
    for i, n in enumerate(need):
        tables[i, :n] = perm[at:at + n]
        at += n
    return tables


@dataclass
class DecodeCase:
    """A batch of sequences with one or more query rows each, over one layer."""
    name: str
    dtype: str                      # 'f32' | 'bf16' | 'f16'
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    num_blocks: int
    ctx_lens: np.ndarray            # int32 [B]: keys visible to the last query row
    q_per_seq: int
    tables: np.ndarray              # int32 [B, max_blocks]
    q: np.ndarray                   # fp32 values (already rounded to dtype) [B*q_per_seq, Hq, D]
    k_pool: Optional[np.ndarray]    # fp32 values [NB, BS, Hkv, D] (None: generate on device)
    v_pool: Optional[np.ndarray]
    scale: float
    extra: dict = field(default_factory=dict)

    @property
    def batch(self) -> int:
        return int(self.ctx_lens.shape[0])


def _round(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return bf16_round(x)
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    return x


def config1(seed: int = 0) -> DecodeCase:
    g = rng(seed)
    B, Hq, Hkv, D, NB = 8, 15, 5, 64, 512
    ctx = g.integers(16, 512, size=B, endpoint=True).astype(np.int32)
    tables = disjoint_tables(g, ctx.tolist(), NB)
    std = 1.0 / math.sqrt(D)
    q = normal(g, (B, Hq, D), std)
    k = normal(g, (NB, BLOCK, Hkv, D), std)
    v = normal(g, (NB, BLOCK, Hkv, D), std)
    return DecodeCase("config1", "f32", Hq, Hkv, D, NB, ctx, 1, tables, q, k, v,
                      1.0 / math.sqrt(D))


def config2_meta(seed: int = 0, batch: int = 64, num_kv_heads: int = 8):
    """Lengths and tables for BASELINE config 2 (pool contents come from the device)."""
    g = rng(seed)
    NB = 16384
    ctx = g.integers(256, 4096, size=batch, endpoint=True).astype(np.int32)
    tables = disjoint_tables(g, ctx.tolist(), NB * max(1, batch // 64))
    return dict(num_blocks=NB * max(1, batch // 64), ctx=ctx, tables=tables,
                num_q_heads=32 * num_kv_heads // 8, num_kv_heads=num_kv_heads,
                head_dim=128)


def config4_meta(seed: int = 0):
    g = rng(seed)
    B, K = 32, 4
    ctx = g.integers(512, 8192, size=B, endpoint=True).astype(np.int32)
    accepted = g.integers(0, K, size=B, endpoint=True).astype(np.int32)
    # Tables cover the context plus the whole lookahead window.
    NB = int(sum((c + K + 1 + BLOCK - 1) // BLOCK for c in ctx)) + 64
    tables = disjoint_tables(g, (ctx + K + 1).tolist(), NB)
    return dict(num_blocks=NB, ctx=ctx, accepted=accepted, tables=tables,
                num_q_heads=40, num_kv_heads=8, head_dim=128, window=K + 1)


def config5_meta(seed: int = 0, batch: int = 256):
    g = rng(seed)
    lo, hi = math.log(4096), math.log(32768)
    ctx = np.exp(g.uniform(lo, hi, size=batch)).astype(np.int64)
    ctx = np.clip(ctx, 4096, 32768).astype(np.int32)
    NB = int(sum((c + BLOCK - 1) // BLOCK for c in ctx)) + 64
    tables = disjoint_tables(g, ctx.tolist(), NB)
    return dict(num_blocks=NB, ctx=ctx, tables=tables, num_q_heads=64,
                num_kv_heads=8, head_dim=128)


def config3_meta(seed: int = 0, chunk: int = 512):
    """
    One pass of chunked prefill mixed with decodes: 16 prefill sequences each
    contribute one chunk (the first chunk of a prompt ~U[128,2048] on top of a
    paged prefix ~U[0,1024]), plus 48 decode sequences with ctx ~U[256,4096].
    Later chunks of the same prompts are the same shape with a longer prefix;
    ``chunk_index`` selects which chunk of each prompt this pass carries.
    """
    g = rng(seed)
    P, Dn = 16, 48
    prompt = g.integers(128, 2048, size=P, endpoint=True).astype(np.int32)
    prefix = g.integers(0, 1024, size=P, endpoint=True).astype(np.int32)
    dctx = g.integers(256, 4096, size=Dn, endpoint=True).astype(np.int32)
    totals = (prefix + prompt).tolist() + dctx.tolist()
    NB = int(sum((t + BLOCK - 1) // BLOCK for t in totals)) + 64
    tables = disjoint_tables(g, totals, NB)
    return dict(num_blocks=NB, prompt=prompt, prefix=prefix, decode_ctx=dctx,
                tables=tables, num_q_heads=32, num_kv_heads=8, head_dim=128,
                chunk=chunk)


def config3_pass(meta: dict, chunk_index: int = 0):
    """
    (q_lens, kv_lens) per sequence for one pass: prefill sequence i carries
    tokens ``prefix+chunk_index*chunk .. +chunk`` of its prompt (0 rows once its
    prompt is done), decode sequences carry one row each.
    """
    chunk = meta["chunk"]
    q_lens, kv_lens = [], []
    for p, L in zip(meta["prefix"], meta["prompt"]):
        lo = chunk_index * chunk
        n = int(max(0, min(chunk, L - lo)))
        q_lens.append(n)
        kv_lens.append(int(p) + lo + n)
    for c in meta["decode_ctx"]:
        q_lens.append(1)
        kv_lens.append(int(c))
    return np.asarray(q_lens, np.int32), np.asarray(kv_lens, np.int32)


def small_decode_case(name: str, seed: int, dtype: str, Hq: int, Hkv: int, D: int,
                      ctx: List[int], q_per_seq: int = 1, NB: Optional[int] = None,
                      q_std: float = 1.0, kv_std: float = 1.0) -> DecodeCase:
    g = rng(seed)
    need = sum((c + BLOCK - 1) // BLOCK for c in ctx)
    NB = NB or need + 8
    ctx = np.asarray(ctx, np.int32)
    tables = disjoint_tables(g, ctx.tolist(), NB)
    q = _round(normal(g, (len(ctx) * q_per_seq, Hq, D), q_std), dtype)
    k = _round(normal(g, (NB, BLOCK, Hkv, D), kv_std), dtype)
    v = _round(normal(g, (NB, BLOCK, Hkv, D), kv_std), dtype)
    return DecodeCase(name, dtype, Hq, Hkv, D, NB, ctx, q_per_seq, tables, q, k, v,
                      1.0 / math.sqrt(D))


def rows_of(case: DecodeCase):
    """Reference-style packed metadata: (seq_ids, positions) per query row."""
    seq_ids, positions = [], []
    for s in range(case.batch):
        n = int(case.ctx_lens[s])
        for i in range(case.q_per_seq):
            seq_ids.append(s)
            positions.append(n - case.q_per_seq + i)
    return seq_ids, positions


def oracle_decode(case: DecodeCase, window: Optional[dict] = None) -> np.ndarray:
    """Oracle output for a DecodeCase, [B*q_per_seq, Hq, D] fp32."""
    from oracle.paged_oracle import varlen_attention
    seq_ids, positions = rows_of(case)
    tables = [case.tables[s][case.tables[s] >= 0] for s in range(case.batch)]
    qh = np.transpose(case.q, (1, 0, 2))                      # (H, T, D)
    out = varlen_attention(qh, case.k_pool[None], case.v_pool[None], 0, tables,
                           seq_ids, positions, BLOCK, scale=case.scale,
                           window=window)
    return np.transpose(out, (1, 0, 2))
