"""
Build ``libmemforge_sm100.so`` in-tree with nvcc for sm_100a.

    python -m memforge_b200.build            # build if sources changed
    python -m memforge_b200.build --force    # always rebuild
    python -m memforge_b200.build --ptxas-v  # print register / smem usage

The library is plain C ABI (include/memforge_sm100.h) with the CUDA runtime
linked statically, so it loads into any process (PyTorch, a cgo or JNI host,
ctypes) without version coupling to that process's own CUDA runtime.
"""

from __future__ import annotations

import argparse
import glob
import hashlib
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libmemforge_sm100.so")
STAMP = LIB + ".sha"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2,-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-shared", "-cudart", "static",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    return "nvcc"


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _digest() -> str:
    h = hashlib.sha256()
    files = sources() + sorted(glob.glob(os.path.join(CSRC, "*.h")) +
                               glob.glob(os.path.join(CSRC, "*.cuh")) +
                               glob.glob(os.path.join(INCLUDE, "*.h")))
    for f in files:
        h.update(f.encode())
        with open(f, "rb") as fh:
            h.update(fh.read())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def build(force: bool = False, ptxas_verbose: bool = False) -> str:
    digest = _digest()
    if not force and os.path.exists(LIB) and os.path.exists(STAMP):
        with open(STAMP) as fh:
            if fh.read().strip() == digest:
                return LIB
    cmd = [nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-o", LIB + ".tmp", *sources()]
    # Exported symbols: only the extern "C" mf_* API (everything else is hidden).
    cmd += ["-Xlinker", "--version-script=" + os.path.join(CSRC, "exports.map")]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + proc.stdout + proc.stderr)
    if ptxas_verbose:
        sys.stdout.write(proc.stdout + proc.stderr)
    os.replace(LIB + ".tmp", LIB)
    with open(STAMP, "w") as fh:
        fh.write(digest)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force or args.ptxas_v, ptxas_verbose=args.ptxas_v))


if __name__ == "__main__":
    main()
