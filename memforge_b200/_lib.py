"""
ctypes binding of ``libmemforge_sm100.so`` (the C ABI in include/memforge_sm100.h).

This is the exact stub a MemForge maintainer would add on the reference side:
it loads the library, declares the prototypes and turns negative return codes
into exceptions.  Loading fails loudly: there is no CPU path behind it.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmemforge_sm100.so")

MF_F32, MF_F16, MF_BF16 = 0, 1, 2

MF_OK = 0
MF_EINVAL = -1
MF_EBOUNDS = -2
MF_ETIMEOUT = -3
MF_ECUDA = -4
MF_EUNSUPPORTED = -5
MF_EWORKSPACE = -6

MF_ERR_BLOCK_ID = 0x1
MF_ERR_SLOT = 0x2
MF_ERR_TABLE = 0x4
MF_ERR_LENGTH = 0x8
MF_ERR_TIMEOUT = 0x10

ERR_NAMES = {
    MF_ERR_BLOCK_ID: "block table entry outside the pool",
    MF_ERR_SLOT: "slot_mapping entry outside the pool",
    MF_ERR_TABLE: "context needs more blocks than the block table holds",
    MF_ERR_LENGTH: "length out of range (kv_len < q_len, or a confirmed count above the "
                   "window)",
    MF_ERR_TIMEOUT: "a bounded pipeline wait gave up",
}

# Every symbol include/memforge_sm100.h declares.
EXPORTED = (
    "mf_abi_version", "mf_last_error", "mf_device_info", "mf_reshape_and_cache",
    "mf_paged_attention_workspace_size", "mf_paged_attention", "mf_paged_decode",
    "mf_copy_blocks", "mf_paged_decode_noalloc", "mf_peer_barrier", "mf_ipc_export",
    "mf_ipc_open", "mf_ipc_close", "mf_commit_window", "mf_gather_kv", "mf_accept_commit",
)

MF_IPC_HANDLE_BYTES = 64

MF_MAX_OUT_PEERS = 8

c_i32, c_i64, c_f32, c_vp, c_sz = (ctypes.c_int32, ctypes.c_int64, ctypes.c_float,
                                   ctypes.c_void_p, ctypes.c_size_t)


class AttentionArgs(ctypes.Structure):
    """Mirror of ``mf_attention_args``."""
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("q", c_vp), ("q_stride_row", c_i64), ("q_stride_head", c_i64),
        ("out", c_vp), ("out_stride_row", c_i64), ("out_stride_head", c_i64),
        ("k_pool", c_vp), ("v_pool", c_vp),
        ("pool_stride_block", c_i64), ("pool_stride_slot", c_i64), ("pool_stride_head", c_i64),
        ("num_blocks", c_i32), ("block_size", c_i32),
        ("block_tables", c_vp), ("table_stride", c_i32),
        ("cu_seqlens_q", c_vp), ("q_per_seq", c_i32),
        ("kv_lens", c_vp), ("row_map", c_vp),
        ("win_k", c_vp), ("win_v", c_vp), ("win_stride_row", c_i64), ("win_stride_head", c_i64),
        ("num_seqs", c_i32), ("total_q", c_i32), ("max_q_len", c_i32),
        ("num_q_heads", c_i32), ("num_kv_heads", c_i32), ("head_dim", c_i32),
        ("scale", c_f32), ("causal", c_i32), ("dtype", ctypes.c_int),
        ("num_out_peers", c_i32), ("out_head_offset", c_i32),
        ("out_peers", c_vp * MF_MAX_OUT_PEERS),
    ]


class AcceptArgs(ctypes.Structure):
    """Mirror of ``mf_accept_args``."""
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("num_seqs", c_i32), ("num_drafts", c_i32),
        ("draft_tokens", c_vp), ("draft_tokens_stride", c_i64),
        ("target_tokens", c_vp), ("target_tokens_stride", c_i64),
        ("target_probs", c_vp), ("tp_stride_seq", c_i64), ("tp_stride_slot", c_i64),
        ("draft_probs", c_vp), ("dp_stride_seq", c_i64), ("dp_stride_slot", c_i64),
        ("vocab", c_i32),
        ("uniforms", c_vp), ("uniforms_stride", c_i64),
        ("resample_uniform", c_vp),
        ("num_accepted", c_vp), ("next_token", c_vp),
        ("win_k", c_vp), ("win_v", c_vp),
        ("win_stride_layer", c_i64), ("win_stride_row", c_i64), ("win_stride_head", c_i64),
        ("key_pool", c_vp), ("value_pool", c_vp),
        ("pool_stride_layer", c_i64), ("pool_stride_block", c_i64),
        ("pool_stride_slot", c_i64), ("pool_stride_head", c_i64),
        ("num_layers", c_i32), ("num_blocks", c_i32), ("block_size", c_i32),
        ("block_tables", c_vp), ("table_stride", c_i32),
        ("ctx_lens", c_vp),
        ("num_kv_heads", c_i32), ("head_dim", c_i32), ("elem_bytes", c_i32),
        ("err_flag", c_vp),
    ]


class MemforgeError(RuntimeError):
    """A negative return code from the library."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


_lock = threading.Lock()
_lib = None


def _declare(lib):
    lib.mf_abi_version.restype = ctypes.c_int
    lib.mf_last_error.restype = ctypes.c_char_p
    lib.mf_device_info.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                                   ctypes.POINTER(ctypes.c_int)]
    lib.mf_reshape_and_cache.argtypes = [
        c_vp, c_vp, ctypes.c_int, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, ctypes.c_int,
        c_i64, c_i64, c_i64, c_i32, c_i32, c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp]
    lib.mf_paged_attention_workspace_size.argtypes = [ctypes.POINTER(AttentionArgs), ctypes.c_int]
    lib.mf_paged_attention_workspace_size.restype = c_sz
    lib.mf_paged_attention.argtypes = [ctypes.POINTER(AttentionArgs), c_vp, c_sz, c_vp, c_vp]
    lib.mf_paged_decode.argtypes = [
        c_vp, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_i32, c_vp, c_i32, c_vp, c_i32,
        c_i32, c_i32, c_i32, c_i32, c_f32, ctypes.c_int, c_vp, c_vp, c_sz, c_vp, c_vp]
    lib.mf_gather_kv.argtypes = [
        c_vp, c_vp, ctypes.c_int, c_i64, c_i64, c_i64, c_i32, c_i32, c_vp, c_i32, c_i32, c_i32,
        c_i32, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp]
    lib.mf_accept_commit.argtypes = [ctypes.POINTER(AcceptArgs), c_vp]
    lib.mf_copy_blocks.argtypes = [c_vp, c_vp, c_i32, c_i32, c_i64, c_i32, c_vp, c_i32, c_vp, c_vp]
    lib.mf_commit_window.argtypes = [
        c_vp, c_vp, ctypes.c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp,
        ctypes.c_int, c_i64, c_i64, c_i64, c_i64, c_i32, c_i32, c_i32, c_vp, c_i32, c_vp, c_vp,
        c_i32, c_i32, c_i32, c_i32, c_vp, c_vp]
    lib.mf_peer_barrier.argtypes = [ctypes.POINTER(c_vp), c_i32, c_i32, ctypes.c_uint32, c_vp,
                                     c_vp]
    lib.mf_ipc_export.argtypes = [c_vp, c_vp, ctypes.POINTER(ctypes.c_uint64)]
    lib.mf_ipc_open.argtypes = [c_vp, ctypes.c_uint64, ctypes.POINTER(c_vp)]
    lib.mf_ipc_close.argtypes = [c_vp, ctypes.c_uint64]
    lib.mf_paged_decode_noalloc.argtypes = [
        c_vp, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_i32, c_vp, c_i32, c_vp, c_i32,
        c_i32, c_i32, c_i32, c_i32, c_f32, ctypes.c_int, c_vp, c_vp, c_vp]
    for name in EXPORTED:
        if name not in ("mf_last_error", "mf_paged_attention_workspace_size"):
            getattr(lib, name).restype = ctypes.c_int
    return lib


def lib():
    """The loaded library (loaded once).  Raises if it has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with `python -m memforge_b200.build` "
                        "(there is no CPU implementation of these kernels)")
                _lib = _declare(ctypes.CDLL(LIB_PATH))
                if _lib.mf_abi_version() != 1:
                    raise RuntimeError("libmemforge_sm100.so ABI version mismatch")
    return _lib


def check(rc: int, what: str) -> None:
    if rc != MF_OK:
        msg = lib().mf_last_error()
        raise MemforgeError(rc, f"{what} failed ({rc}): {msg.decode() if msg else ''}")


def describe_err(bits: int) -> str:
    return "; ".join(v for k, v in ERR_NAMES.items() if bits & k) or "no error"
