"""
Tensor-level wrappers over the C ABI.

PyTorch supplies device memory, streams and strides; every computation happens
in ``libmemforge_sm100.so``.  Tensors must be CUDA tensors: there is no CPU
implementation, and a CPU tensor is an error, not a reason to fall back.

Workspace and error word
------------------------
* The attention kernels keep split-K partials and arrival counters in a
  zero-initialised workspace they leave zeroed.  One is cached per device and
  grown on demand; make one warm-up call before capturing a CUDA graph so the
  capture does not allocate.  A workspace that is outgrown stays allocated, so
  graphs captured on it keep a valid address.  Launches on different streams
  that may overlap must pass their own ``workspace=``.
* Kernels report bad block ids, slots past the pool, too-short block tables and
  expired waits by OR-ing bits into a per-device int32 error word.  With
  ``MEMFORGE_CHECK=1`` (or ``set_checks(True)``) every call synchronises and
  raises on a non-zero word; otherwise ``check_device_errors()`` reads it.
"""

from __future__ import annotations

import os
import threading
from typing import Dict, Optional, Sequence

import torch

from . import _lib as L

DTYPES = {torch.float32: L.MF_F32, torch.float16: L.MF_F16, torch.bfloat16: L.MF_BF16}

_state_lock = threading.Lock()
_workspaces: Dict[int, torch.Tensor] = {}
_retired: list = []   # grown-out workspaces, kept alive for graphs that captured them
_err_words: Dict[int, torch.Tensor] = {}
_checks = os.environ.get("MEMFORGE_CHECK", "0") not in ("", "0")
launch_counter = {"reshape_and_cache": 0, "paged_attention": 0, "copy_blocks": 0,
                  "peer_barrier": 0, "commit_window": 0, "gather_kv": 0,
                  "accept_commit": 0}


def set_checks(enabled: bool) -> None:
    """Synchronise and check the device error word after every call."""
    global _checks
    _checks = bool(enabled)


def require_cuda(what: str, *tensors) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                f"{what}: memforge_b200 runs on CUDA tensors (sm_100a); got a tensor on {t.device}")


def dtype_code(dt: torch.dtype) -> int:
    if dt not in DTYPES:
        raise TypeError(f"unsupported dtype {dt}; expected float32, float16 or bfloat16")
    return DTYPES[dt]


def _dev_index(t: torch.Tensor) -> int:
    return t.device.index if t.device.index is not None else torch.cuda.current_device()


def err_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _err_words.get(idx)
    if w is None:
        with _state_lock:
            w = _err_words.get(idx)
            if w is None:
                w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
                _err_words[idx] = w
    return w


def check_device_errors(device: Optional[torch.device] = None, reset: bool = True) -> None:
    """Synchronise and raise if any kernel on `device` reported a violation."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    w = err_word(device)
    bits = int(w.item())
    if reset and bits:
        w.zero_()
        ws = _workspaces.get(device.index if device.index is not None else torch.cuda.current_device())
        if ws is not None:
            ws.zero_()   # an aborted launch may leave arrival counters behind
    if bits:
        raise IndexError(f"memforge_b200 kernel reported: {L.describe_err(bits)} (0x{bits:x})")


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _workspaces.get(idx)
    if ws is None or ws.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(
                "paged attention needs a larger workspace during CUDA graph capture: make one "
                "call with the same shapes before capturing")
        with _state_lock:
            ws = _workspaces.get(idx)
            if ws is None or ws.numel() < nbytes:
                size = max(nbytes, 1 << 20)
                if ws is not None:
                    _retired.append(ws)
                ws = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", idx))
                _workspaces[idx] = ws
    return ws


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _after(what: str, device: torch.device) -> None:
    if _checks:
        torch.cuda.synchronize(device)
        check_device_errors(device)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


# ------------------------------------------------------------------ KV write

def reshape_and_cache(key: torch.Tensor, value: torch.Tensor, key_pool: torch.Tensor,
                      value_pool: torch.Tensor, slot_mapping: torch.Tensor,
                      heads_major: bool = False) -> None:
    """
    Scatter ``key``/``value`` rows ``(T, H, D)`` (any strides, D contiguous)
    into one pool layer at ``slot_mapping[t]`` (int32/int64 CUDA tensor,
    -1 = skip).  ``key_pool`` is ``(blocks, block_size, H, D)``, or
    ``(blocks, H, block_size, D)`` with ``heads_major=True``.
    """
    require_cuda("reshape_and_cache", key, value, key_pool, value_pool, slot_mapping)
    if key.dim() != 3 or value.shape != key.shape:
        raise ValueError(f"keys/values must be (T, H, D) of one shape, got {tuple(key.shape)} "
                         f"and {tuple(value.shape)}")
    if key.stride(-1) != 1:
        key = key.contiguous()
    if value.stride(-1) != 1:
        value = value.contiguous()
    if key_pool.stride(-1) != 1 or value_pool.stride() != key_pool.stride():
        raise ValueError("pool layers must share strides and have a contiguous last dim")
    if slot_mapping.dtype not in (torch.int32, torch.int64):
        raise TypeError("slot_mapping must be int32 or int64")
    if not slot_mapping.is_contiguous():
        slot_mapping = slot_mapping.contiguous()
    T, H, D = key.shape
    if heads_major:
        nb, hp, bs, dp = key_pool.shape
        sb, sh, ss = key_pool.stride(0), key_pool.stride(1), key_pool.stride(2)
    else:
        nb, bs, hp, dp = key_pool.shape
        sb, ss, sh = key_pool.stride(0), key_pool.stride(1), key_pool.stride(2)
    if (hp, dp) != (H, D):
        raise ValueError(f"pool holds {hp} heads x {dp} dims, keys are {H} x {D}")
    if slot_mapping.numel() != T:
        raise ValueError(f"{T} tokens but {slot_mapping.numel()} slots")
    if T == 0:
        return
    lib = L.lib()
    dev = key.device
    rc = lib.mf_reshape_and_cache(
        key.data_ptr(), value.data_ptr(), dtype_code(key.dtype), key.stride(0), key.stride(1),
        value.stride(0), value.stride(1), key_pool.data_ptr(), value_pool.data_ptr(),
        dtype_code(key_pool.dtype), sb, ss, sh, nb, bs, slot_mapping.data_ptr(),
        1 if slot_mapping.dtype == torch.int64 else 0, T, H, D, err_word(dev).data_ptr(),
        _stream_ptr(dev))
    L.check(rc, "mf_reshape_and_cache")
    launch_counter["reshape_and_cache"] += 1
    _after("reshape_and_cache", dev)


def gather_kv(key_pool: torch.Tensor, value_pool: torch.Tensor, flat_index: torch.Tensor,
              heads_major: bool = False):
    """
    ``mf_gather_kv``: the pool slots ``flat_index`` (int32/int64 CUDA tensor) of
    one layer ``(blocks, block_size, H, D)`` (or ``(blocks, H, block_size, D)``
    with ``heads_major``) as contiguous ``(1, H, T, D)`` keys and values.
    """
    require_cuda("gather_kv", key_pool, value_pool)
    if flat_index.device != key_pool.device:
        flat_index = flat_index.to(key_pool.device)
    if key_pool.stride(-1) != 1 or value_pool.stride() != key_pool.stride():
        raise ValueError("pool layers must share strides and have a contiguous last dim")
    if flat_index.dtype not in (torch.int32, torch.int64):
        raise TypeError("flat_index must be int32 or int64")
    flat_index = flat_index.reshape(-1).contiguous()
    if heads_major:
        nb, H, bs, D = key_pool.shape
        sb, sh, ss = key_pool.stride(0), key_pool.stride(1), key_pool.stride(2)
    else:
        nb, bs, H, D = key_pool.shape
        sb, ss, sh = key_pool.stride(0), key_pool.stride(1), key_pool.stride(2)
    T = flat_index.numel()
    k = torch.empty((1, H, T, D), dtype=key_pool.dtype, device=key_pool.device)
    v = torch.empty_like(k)
    if T == 0:
        return k, v
    dev = key_pool.device
    rc = L.lib().mf_gather_kv(key_pool.data_ptr(), value_pool.data_ptr(),
                              dtype_code(key_pool.dtype), sb, ss, sh, nb, bs,
                              flat_index.data_ptr(), 1 if flat_index.dtype == torch.int64 else 0,
                              T, H, D, k.data_ptr(), v.data_ptr(), T * D, D,
                              err_word(dev).data_ptr(), _stream_ptr(dev))
    L.check(rc, "mf_gather_kv")
    launch_counter["gather_kv"] += 1
    _after("gather_kv", dev)
    return k, v


def commit_window(win_k: torch.Tensor, win_v: torch.Tensor, key_pool: torch.Tensor,
                  value_pool: torch.Tensor, block_tables: torch.Tensor, ctx_lens: torch.Tensor,
                  num_confirmed: torch.Tensor) -> None:
    """
    Write rows ``0 .. num_confirmed[b]-1`` of each sequence's window into the
    pool at positions ``ctx_lens[b] + j`` (one launch; the slot arithmetic runs
    on the device).  One layer: ``win_k``/``win_v`` ``(B*W, H, D)``
    sequence-major and ``key_pool`` ``(blocks, block_size, H, D)``; every layer
    at once: ``(L, B*W, H, D)`` windows and ``(L, blocks, block_size, H, D)``
    pools.  ``block_tables`` int32 ``[B, width]``, ``ctx_lens`` and
    ``num_confirmed`` int32 ``[B]``.  Rows past ``num_confirmed`` are not
    written.
    """
    require_cuda("commit_window", win_k, win_v, key_pool, value_pool, block_tables, ctx_lens,
                 num_confirmed)
    if win_v.shape != win_k.shape or win_k.dim() not in (3, 4):
        raise ValueError(f"window keys/values must be (B*W, H, D) or (L, B*W, H, D) of one "
                         f"shape, got {tuple(win_k.shape)} and {tuple(win_v.shape)}")
    layered = win_k.dim() == 4
    if key_pool.dim() != (5 if layered else 4) or value_pool.shape != key_pool.shape:
        raise ValueError("pools must be (blocks, block_size, H, D) for (B*W, H, D) windows and "
                         "(L, blocks, block_size, H, D) for (L, B*W, H, D) windows")
    wk = win_k if layered else win_k.unsqueeze(0)
    wv = win_v if layered else win_v.unsqueeze(0)
    kp = key_pool if layered else key_pool.unsqueeze(0)
    vp = value_pool if layered else value_pool.unsqueeze(0)
    B = ctx_lens.numel()
    if B == 0:
        return
    if num_confirmed.numel() != B:
        raise ValueError(f"{B} sequences but {num_confirmed.numel()} confirmed counts")
    L_, R, H, D = wk.shape
    W = R // B
    if W * B != R or W == 0:
        raise ValueError("window rows are not a whole number of windows")
    if kp.shape[0] != L_:
        raise ValueError(f"{L_} window layers but {kp.shape[0]} pool layers")
    if wk.stride(-1) != 1:
        wk = wk.contiguous()
    if wv.stride(-1) != 1:
        wv = wv.contiguous()
    if kp.stride(-1) != 1 or vp.stride() != kp.stride():
        raise ValueError("pools must share strides and have a contiguous last dim")
    _, nb, bs, hp, dp = kp.shape
    if (hp, dp) != (H, D):
        raise ValueError(f"pool holds {hp} heads x {dp} dims, window rows are {H} x {D}")
    if block_tables.dim() != 2 or block_tables.shape[0] != B:
        raise ValueError("block_tables must be [B, width]")
    tables = block_tables.to(torch.int32).contiguous()
    ctx = ctx_lens.to(torch.int32).contiguous()
    conf = num_confirmed.to(torch.int32).contiguous()
    dev = win_k.device
    rc = L.lib().mf_commit_window(
        wk.data_ptr(), wv.data_ptr(), dtype_code(wk.dtype), wk.stride(0), wk.stride(1),
        wk.stride(2), wv.stride(0), wv.stride(1), wv.stride(2), kp.data_ptr(), vp.data_ptr(),
        dtype_code(kp.dtype), kp.stride(0), kp.stride(1), kp.stride(2), kp.stride(3), L_, nb, bs,
        tables.data_ptr(), tables.stride(0), ctx.data_ptr(), conf.data_ptr(), B, W, H, D,
        err_word(dev).data_ptr(), _stream_ptr(dev))
    L.check(rc, "mf_commit_window")
    launch_counter["commit_window"] += 1
    _after("commit_window", dev)


def copy_blocks(key_pool: torch.Tensor, value_pool: torch.Tensor, pairs: torch.Tensor) -> None:
    """Copy block src -> dst in every layer; ``pairs`` is int32 ``[n, 2]`` on the device."""
    require_cuda("copy_blocks", key_pool, value_pool, pairs)
    if not (key_pool.is_contiguous() and value_pool.is_contiguous()):
        raise ValueError("copy_blocks needs contiguous pools")
    if pairs.dtype != torch.int32:
        pairs = pairs.to(torch.int32)
    pairs = pairs.contiguous()
    layers, nb = key_pool.shape[0], key_pool.shape[1]
    block_elems = key_pool[0, 0].numel()
    dev = key_pool.device
    rc = L.lib().mf_copy_blocks(key_pool.data_ptr(), value_pool.data_ptr(), layers, nb,
                                block_elems, key_pool.element_size(), pairs.data_ptr(),
                                pairs.shape[0], err_word(dev).data_ptr(), _stream_ptr(dev))
    L.check(rc, "mf_copy_blocks")
    launch_counter["copy_blocks"] += 1
    _after("copy_blocks", dev)


# ----------------------------------------------------------------- attention

def paged_attention(q: torch.Tensor, out: torch.Tensor, key_pool: torch.Tensor,
                    value_pool: torch.Tensor, block_tables: torch.Tensor,
                    kv_lens: torch.Tensor, *, cu_seqlens_q: Optional[torch.Tensor] = None,
                    q_per_seq: int = 1, max_q_len: Optional[int] = None, scale: float,
                    causal: bool = True, row_map: Optional[torch.Tensor] = None,
                    win_k: Optional[torch.Tensor] = None, win_v: Optional[torch.Tensor] = None,
                    heads_major: bool = False, workspace_tensor: Optional[torch.Tensor] = None,
                    out_peers: Optional[Sequence[int]] = None, out_head_offset: int = 0
                    ) -> torch.Tensor:
    """
    ``mf_paged_attention`` on torch tensors.

    q, out: ``(rows, Hq, D)`` views (any row/head strides, D contiguous).
    key_pool/value_pool: one layer, ``(blocks, block_size, Hkv, D)`` (or
    ``(blocks, Hkv, block_size, D)`` with ``heads_major``).
    block_tables: int32 ``[num_seqs, width]``; kv_lens: int32 ``[num_seqs]``;
    cu_seqlens_q: int32 ``[num_seqs+1]`` or None (uniform ``q_per_seq``);
    row_map: int32 ``[rows]`` or None; win_k/win_v: ``(rows, Hkv, D)`` or None.
    out_peers: device addresses of the full ``[rows, total heads, D]`` output on
    every GPU of a head-sharded step (``out`` gives their strides); the kernel
    stores this call's heads at ``out_head_offset`` into all of them.
    """
    require_cuda("paged_attention", q, out, key_pool, value_pool, block_tables, kv_lens,
                 cu_seqlens_q, row_map, win_k, win_v)
    for name, t in (("block_tables", block_tables), ("kv_lens", kv_lens),
                    ("cu_seqlens_q", cu_seqlens_q), ("row_map", row_map)):
        if t is not None and t.dtype != torch.int32:
            raise TypeError(f"{name} must be int32 (got {t.dtype})")
    if q.stride(-1) != 1 or out.stride(-1) != 1:
        raise ValueError("q/out need a contiguous head_dim")
    if key_pool.stride() != value_pool.stride() or key_pool.stride(-1) != 1:
        raise ValueError("pool layers must share strides and have a contiguous last dim")
    if q.dtype != key_pool.dtype or out.dtype != q.dtype or value_pool.dtype != q.dtype:
        raise TypeError("q, out and the pool must share a dtype")
    if block_tables.dim() != 2 or block_tables.stride(1) != 1:
        block_tables = block_tables.contiguous()
    kv_lens = kv_lens.contiguous()
    rows, hq, d = q.shape
    if heads_major:
        nb, hkv, bs, dp = key_pool.shape
        sb, sh, ss = key_pool.stride(0), key_pool.stride(1), key_pool.stride(2)
    else:
        nb, bs, hkv, dp = key_pool.shape
        sb, ss, sh = key_pool.stride(0), key_pool.stride(1), key_pool.stride(2)
    if dp != d:
        raise ValueError(f"query head_dim {d} but the pool holds {dp}")
    num_seqs = kv_lens.numel()
    a = L.AttentionArgs()
    a.struct_size = ctypes_sizeof_args()
    a.q, a.q_stride_row, a.q_stride_head = q.data_ptr(), q.stride(0), q.stride(1)
    a.out, a.out_stride_row, a.out_stride_head = out.data_ptr(), out.stride(0), out.stride(1)
    a.k_pool, a.v_pool = key_pool.data_ptr(), value_pool.data_ptr()
    a.pool_stride_block, a.pool_stride_slot, a.pool_stride_head = sb, ss, sh
    a.num_blocks, a.block_size = nb, bs
    a.block_tables, a.table_stride = block_tables.data_ptr(), block_tables.stride(0)
    a.cu_seqlens_q = _ptr(cu_seqlens_q)
    a.q_per_seq = q_per_seq
    a.kv_lens = kv_lens.data_ptr()
    a.row_map = _ptr(row_map)
    if win_k is not None:
        if win_k.stride() != win_v.stride() or win_k.stride(-1) != 1:
            raise ValueError("window K/V must share strides with a contiguous last dim")
        a.win_k, a.win_v = win_k.data_ptr(), win_v.data_ptr()
        a.win_stride_row, a.win_stride_head = win_k.stride(0), win_k.stride(1)
    a.num_seqs, a.total_q = num_seqs, rows
    a.max_q_len = max_q_len if max_q_len is not None else q_per_seq
    a.num_q_heads, a.num_kv_heads, a.head_dim = hq, hkv, d
    a.scale, a.causal, a.dtype = float(scale), 1 if causal else 0, dtype_code(q.dtype)
    if out_peers:
        if len(out_peers) > L.MF_MAX_OUT_PEERS:
            raise ValueError(f"at most {L.MF_MAX_OUT_PEERS} output peers")
        a.num_out_peers, a.out_head_offset = len(out_peers), int(out_head_offset)
        for i, ptr in enumerate(out_peers):
            a.out_peers[i] = int(ptr)
    lib = L.lib()
    dev = q.device
    idx = _dev_index(q)
    need = lib.mf_paged_attention_workspace_size(a, idx)
    ws = workspace_tensor if workspace_tensor is not None else (
        workspace(dev, need) if need else None)
    rc = lib.mf_paged_attention(a, _ptr(ws), 0 if ws is None else ws.numel(),
                                err_word(dev).data_ptr(), _stream_ptr(dev))
    L.check(rc, "mf_paged_attention")
    launch_counter["paged_attention"] += 1
    _after("paged_attention", dev)
    return out


_ARGS_SIZE = None


def ctypes_sizeof_args() -> int:
    global _ARGS_SIZE
    if _ARGS_SIZE is None:
        import ctypes
        _ARGS_SIZE = ctypes.sizeof(L.AttentionArgs)
    return _ARGS_SIZE


def peer_barrier(flag_ptrs: Sequence[int], rank: int, epoch: int,
                 device: torch.device) -> None:
    """``mf_peer_barrier``: completes a head-sharded step (see ``kv_shard.PeerOutput``)."""
    import ctypes
    arr = (ctypes.c_void_p * len(flag_ptrs))(*[int(p) for p in flag_ptrs])
    rc = L.lib().mf_peer_barrier(arr, len(flag_ptrs), int(rank), int(epoch),
                                 err_word(device).data_ptr(), _stream_ptr(device))
    L.check(rc, "mf_peer_barrier")
    launch_counter["peer_barrier"] += 1
