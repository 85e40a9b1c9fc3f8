"""
Helpers for the GPU parity tests: device copies of seeded cases and a plain
PyTorch fp32 reference of paged attention for full-size configs (itself checked
against the numpy oracle in ``test_torch_reference.py``).
"""

from __future__ import annotations

import math
from typing import Optional

import numpy as np
import torch

from oracle.paged_oracle import f32_to_bf16

TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
TOL = {"f32": dict(atol=1e-5, rtol=1e-5), "bf16": dict(atol=2e-2, rtol=1e-2),
       "f16": dict(atol=2e-2, rtol=1e-2)}


def to_dev(x: np.ndarray, dtype: str, device="cuda") -> torch.Tensor:
    """fp32 numpy values (already representable) -> device tensor of `dtype`."""
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    return t.to(TORCH_DT[dtype]).to(device)


def to_np32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def assert_close(got: np.ndarray, want: np.ndarray, dtype: str, what: str = ""):
    tol = TOL[dtype]
    err = np.abs(got - want)
    bound = tol["atol"] + tol["rtol"] * np.abs(want)
    bad = err > bound
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    assert not bad.any(), (f"{what}: {int(bad.sum())} elements out of tolerance, "
                           f"max |err| {float(err.max()):.3e}")


def torch_reference(q: torch.Tensor, k_layer: torch.Tensor, v_layer: torch.Tensor,
                    tables: torch.Tensor, kv_lens, q_lens, scale: float,
                    win_k: Optional[torch.Tensor] = None, win_v: Optional[torch.Tensor] = None,
                    causal: bool = True) -> torch.Tensor:
    """
    fp32 paged attention, one sequence at a time, on whatever device the inputs
    live: the materialised formulation of ``paged_attention_varlen_materialised``.
    q: (rows, Hq, D) sequence-major; k_layer: (NB, BS, Hkv, D).
    """
    rows, Hq, D = q.shape
    NB, BS, Hkv, _ = k_layer.shape
    G = Hq // Hkv
    out = torch.empty((rows, Hq, D), dtype=torch.float32, device=q.device)
    kflat = k_layer.reshape(NB * BS, Hkv, D)
    vflat = v_layer.reshape(NB * BS, Hkv, D)
    kv_lens = [int(x) for x in kv_lens]
    q_lens = [int(x) for x in q_lens]
    r0 = 0
    for s, (kv, ql) in enumerate(zip(kv_lens, q_lens)):
        if ql == 0:
            continue
        pos = torch.arange(kv, device=q.device)
        slots = tables[s, pos // BS].long() * BS + pos % BS
        keys = kflat[slots].float()
        vals = vflat[slots].float()
        if win_k is not None:
            keys[kv - ql:] = win_k[r0:r0 + ql].float()
            vals[kv - ql:] = win_v[r0:r0 + ql].float()
        keys = keys.permute(1, 0, 2).repeat_interleave(G, dim=0)    # (Hq, kv, D)
        vals = vals.permute(1, 0, 2).repeat_interleave(G, dim=0)
        qs = q[r0:r0 + ql].float().permute(1, 0, 2)                  # (Hq, ql, D)
        sc = torch.matmul(qs, keys.transpose(1, 2)) * scale
        if causal:
            limit = (kv - ql) + torch.arange(ql, device=q.device)
            vis = pos[None, :] <= limit[:, None]
            sc = sc.masked_fill(~vis[None], float("-inf"))
        w = torch.softmax(sc, dim=-1)
        out[r0:r0 + ql] = torch.matmul(w, vals).permute(1, 0, 2)
        r0 += ql
    return out


def randn_pool(num_blocks: int, heads: int, dim: int, dtype: torch.dtype, seed: int,
               device="cuda", block: int = 16):
    g = torch.Generator(device=device).manual_seed(seed)
    k = torch.randn((num_blocks, block, heads, dim), generator=g, device=device, dtype=dtype)
    v = torch.randn((num_blocks, block, heads, dim), generator=g, device=device, dtype=dtype)
    return k, v
