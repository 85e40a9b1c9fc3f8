"""The C ABI library loads and exports what include/memforge_sm100.h declares (no GPU)."""

import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from memforge_b200 import _lib as L
from tests.conftest import ROOT

HEADER = os.path.join(ROOT, "include", "memforge_sm100.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"MF_API\s+[\w\s\*]+?\b(mf_\w+)\s*\(", text)))


def test_library_builds_and_loads():
    from memforge_b200.build import build
    path = build()
    assert os.path.exists(path)
    lib = L.lib()
    assert lib.mf_abi_version() == 1


def test_every_declared_symbol_is_exported():
    syms = declared_symbols()
    assert set(syms) == set(L.EXPORTED), syms
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (mf_\w+)", out))
    assert set(syms) <= exported
    # nothing but the C ABI leaks out of the library
    assert exported == set(syms)


@pytest.mark.parametrize("cname,struct", [("mf_attention_args", L.AttentionArgs),
                                          ("mf_accept_args", L.AcceptArgs)])
def test_args_struct_layout_matches_the_header(cname, struct):
    """sizeof and offsets of the argument structs agree between C and ctypes."""
    fields = [f for f, _ in struct._fields_]
    src = ["#include <stdio.h>", "#include <stddef.h>", '#include "memforge_sm100.h"',
           "int main(void){",
           f'printf("%zu\\n", sizeof({cname}));']
    for f in fields:
        src.append(f'printf("%zu\\n", offsetof({cname}, {f}));')
    src.append("return 0;}")
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        exe = os.path.join(d, "t")
        open(c, "w").write("\n".join(src))
        subprocess.run(["gcc", "-I", os.path.dirname(HEADER), c, "-o", exe], check=True)
        vals = [int(x) for x in subprocess.run([exe], capture_output=True, text=True,
                                               check=True).stdout.split()]
    assert vals[0] == ctypes.sizeof(struct)
    for f, off in zip(fields, vals[1:]):
        assert getattr(struct, f).offset == off, f


def test_error_paths_without_a_gpu():
    """Argument validation happens before any CUDA call and returns MF_EINVAL."""
    lib = L.lib()
    a = L.AttentionArgs()
    a.struct_size = 3  # wrong ABI size
    rc = lib.mf_paged_attention(a, None, 0, None, None)
    assert rc == L.MF_EINVAL
    assert b"size mismatch" in lib.mf_last_error()
    a.struct_size = ctypes.sizeof(a)
    a.num_q_heads, a.num_kv_heads, a.head_dim = 6, 4, 64
    a.num_blocks, a.block_size, a.q_per_seq = 1, 16, 1
    rc = lib.mf_paged_attention(a, None, 0, None, None)
    assert rc == L.MF_EINVAL and b"multiple" in lib.mf_last_error()
    rc = lib.mf_reshape_and_cache(None, None, 2, 0, 0, 0, 0, None, None, 2, 0, 0, 0, 1, 16,
                                  None, 0, 4, 1, 64, None, None)
    assert rc == L.MF_EINVAL


def test_commit_window_validates_before_any_cuda_call():
    lib = L.lib()
    # win_k, win_v, src dtype, k/v layer/row/head strides, pools, pool dtype, pool strides,
    # layers, blocks, block size, tables, table stride, ctx, confirmed, seqs, window, heads, dim
    def call(src=2, pool=2, layers=1, seqs=2, window=5, heads=8, dim=128, ptr=None):
        return lib.mf_commit_window(ptr, ptr, src, 0, 0, 0, 0, 0, 0, ptr, ptr, pool, 0, 0, 0, 0,
                                    layers, 16, 16, ptr, 4, ptr, ptr, seqs, window, heads, dim,
                                    None, None)
    assert call(window=0) == L.MF_EINVAL
    assert call(layers=0) == L.MF_EINVAL
    assert call() == L.MF_EINVAL and b"null pointer" in lib.mf_last_error()
    assert call(seqs=0) == L.MF_OK  # nothing to commit
    buf = ctypes.create_string_buffer(64)
    p = ctypes.cast(buf, ctypes.c_void_p)
    assert call(src=L.MF_BF16, pool=L.MF_F32, ptr=p) == L.MF_EUNSUPPORTED
    assert b"dtype" in lib.mf_last_error()
