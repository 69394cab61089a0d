"""Builds libltvqkv.so (the C-ABI CUDA library of the filtered-QKV hot path) in-tree.

The library is compiled with nvcc for sm_100a only; the .so lands next to this file so it
travels with the source tree. `python -m nanochat_filter_b200.build [--ptxas-info]`.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
LIB_NAME = "libltvqkv.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)

SOURCES = ["ltvqkv_abi.cu", "ltvqkv_scan.cu", "ltvqkv_gemm.cu", "ltvqkv_decode.cu", "ltvqkv_lookback.cu", "ltvqkv_rotary.cu"]
HEADERS = sorted(f for f in os.listdir(CSRC) if f.endswith(".cuh"))

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libltvqkv")
    return cand


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    lib_mtime = os.path.getmtime(LIB_PATH)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [os.path.join(INCLUDE, "ltvqkv.h")]
    return any(os.path.getmtime(d) > lib_mtime for d in deps)


def build(force: bool = False, ptxas_info: bool = False, verbose: bool = False) -> str:
    """Compiles every .cu source into libltvqkv.so (sm_100a). Returns the library path."""
    if not force and not ptxas_info and not _stale():
        return LIB_PATH
    nvcc = _nvcc()
    objs = []
    build_dir = os.path.join(HERE, "_build")
    os.makedirs(build_dir, exist_ok=True)
    for src in SOURCES:
        obj = os.path.join(build_dir, src.replace(".cu", ".o"))
        cmd = [nvcc, *NVCC_FLAGS, "-I", INCLUDE, "-c", os.path.join(CSRC, src), "-o", obj]
        if ptxas_info:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp, *objs]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, ptxas_info=a.ptxas_info, verbose=a.verbose))
