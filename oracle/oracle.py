"""CPU oracle of the filtered-QKV hot path — TEST INFRASTRUCTURE ONLY.

Python/numpy front end of ltv_oracle.c (a C restatement of the reference's own CPU oracle,
nanochat/ops/ltv_reference_ops.py:7-124 and :299-308). Only tests/, the smoke check of
__graft_entry__.py and the CPU-baseline / reference leg of bench.py use this module; the
product path (nanochat_filter_b200) never imports it.

All arrays are numpy float32. `bf16=True` means the inputs hold bfloat16 values and every
stored result is rounded to bfloat16, exactly where the reference's torch code rounds.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "ltv_oracle.c")
LIB = os.path.join(HERE, "liboracle.so")
NO_CHUNKING = (2147483647, 1, 1)  # (P, Q, K) of the plain scan, ltv_reference_ops.py:162-192

_lib = None


def build(force: bool = False) -> str:
    """Compiles ltv_oracle.c into liboracle.so next to it (gcc, OpenMP when available)."""
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    base = ["-O2", "-fPIC", "-ffp-contract=off", "-fvisibility=hidden", "-std=c11", "-shared", "-o", LIB, SRC, "-lm"]
    last = None
    for cc in ("/usr/bin/gcc", "gcc", "cc"):
        for omp in (["-fopenmp"], []):
            try:
                subprocess.run([cc, *omp, *base], check=True, capture_output=True)
                return LIB
            except (OSError, subprocess.CalledProcessError) as e:  # try the next compiler / no OpenMP
                last = e
    raise RuntimeError(f"could not build the oracle: {last}")


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(LIB)
        f = ctypes.POINTER(ctypes.c_float)
        i, ll = ctypes.c_int, ctypes.c_longlong
        lib.oracle_scan_fwd.argtypes = [f, f, f, f, f, f, i, i, i, i, i, i, i, i, ll, ll, ll]
        lib.oracle_scan_bwd.argtypes = [f, f, f, f, f, f, f, f, f, i, i, i, i, i, i, i, i, ll, ll, ll]
        lib.oracle_gemm_fwd.argtypes = [f, f, f, i, i, i, i, i]
        lib.oracle_gemm_bwd.argtypes = [f, f, f, f, f, i, i, i, i, i, i]
        lib.oracle_round_bf16.argtypes = [f, ll]
        lib.oracle_set_threads.argtypes = [i]
        lib.oracle_set_threads.restype = i
        _lib = lib
    return _lib


def set_threads(n: int) -> int:
    """Sets the oracle's OpenMP thread count (n > 0) and returns the count in effect."""
    return int(_load().oracle_set_threads(int(n)))


def _p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def round_bf16(a) -> np.ndarray:
    """Round-to-nearest-even to bfloat16 values (kept as float32)."""
    out = _f32(a).copy()
    _load().oracle_round_bf16(_p(out), out.size)
    return out


def scan_fwd(combined, inits, logit_bias, NH, NKVH, Da, r, use_sigmoid, bf16, pqk=NO_CHUNKING):
    """combined [B,T,F], inits [B,H,D], logit_bias [H,Da] -> (hq, hk, hv) head-major."""
    combined, inits, logit_bias = _f32(combined), _f32(inits), _f32(logit_bias)
    B, T, _ = combined.shape
    D = Da * r
    oq = np.zeros((B, NH, T, D), np.float32)
    ok = np.zeros((B, NKVH, T, D), np.float32)
    ov = np.zeros((B, NKVH, T, D), np.float32)
    P, Q, K = pqk
    _load().oracle_scan_fwd(_p(combined), _p(inits), _p(logit_bias), _p(oq), _p(ok), _p(ov), B, T, NH, NKVH, Da, r,
                            int(use_sigmoid), int(bf16), P, Q, K)
    return oq, ok, ov


def scan_bwd(combined, inits, logit_bias, gq, gk, gv, NH, NKVH, Da, r, use_sigmoid, bf16, pqk=NO_CHUNKING):
    """Returns (grad_combined [B,T,F], grad_inits [B,H,D], grad_logit_bias [H,Da])."""
    combined, inits, logit_bias = _f32(combined), _f32(inits), _f32(logit_bias)
    gq, gk, gv = _f32(gq), _f32(gk), _f32(gv)
    B, T, F = combined.shape
    H = NH + 2 * NKVH
    D = Da * r
    gc = np.zeros((B, T, F), np.float32)
    gi = np.zeros((B, H, D), np.float32)
    gb = np.zeros((H, Da), np.float32)
    P, Q, K = pqk
    _load().oracle_scan_bwd(_p(combined), _p(inits), _p(logit_bias), _p(gq), _p(gk), _p(gv), _p(gc), _p(gi), _p(gb),
                            B, T, NH, NKVH, Da, r, int(use_sigmoid), int(bf16), P, Q, K)
    return gc, gi, gb


def _qz(a, bf16):
    return round_bf16(a) if bf16 else _f32(a)


def gemm_fwd(x, w, bf16, acc=np.float64):
    """out[b,f,t] = sum_k x[b,t,k] w[f,k] (accumulated in `acc`, rounded to dtype): the reference's
    fused_linear_transpose_reference (ltv_reference_ops.py:299-308, matmul(x, W^T).transpose(1, 2)),
    contracted by numpy's BLAS one sequence at a time, then rounded once. acc=np.float64 is the
    oracle; acc=np.float32 is the reference's own arithmetic (torch / cuBLAS accumulate in fp32)."""
    x, w = _f32(x), _f32(w)
    B, T, K = x.shape
    F = w.shape[0]
    out = np.empty((B, F, T), np.float32)
    wa = w.astype(acc)
    for b in range(B):
        out[b] = _qz(wa @ x[b].astype(acc).T, bf16)
    return out


def gemm_bwd(x, w, g, bf16_x, bf16_w, acc=np.float64):
    """g [B,F,T] -> (grad_x [B,T,K] = sum_f g w, grad_w [F,K] = sum_b sum_t g x), the gradients of
    gemm_fwd, contracted in `acc` (numpy BLAS) and rounded once to their dtypes."""
    x, w, g = _f32(x), _f32(w), _f32(g)
    B, T, K = x.shape
    F = w.shape[0]
    gx = np.empty((B, T, K), np.float32)
    gw = np.zeros((F, K), acc)
    wa = w.astype(acc)
    for b in range(B):
        gb = g[b].astype(acc)
        gx[b] = _qz(gb.T @ wa, bf16_x)
        gw += gb @ x[b].astype(acc)
    return gx, _qz(gw, bf16_w)


def gemm_fwd_c(x, w, bf16):
    """gemm_fwd by ltv_oracle.c's loops (double accumulation; the pinned C restatement)."""
    x, w = _f32(x), _f32(w)
    B, T, K = x.shape
    F = w.shape[0]
    out = np.zeros((B, F, T), np.float32)
    _load().oracle_gemm_fwd(_p(x), _p(w), _p(out), B, T, K, F, int(bf16))
    return out


def gemm_bwd_c(x, w, g, bf16_x, bf16_w):
    """gemm_bwd by ltv_oracle.c's loops."""
    x, w, g = _f32(x), _f32(w), _f32(g)
    B, T, K = x.shape
    F = w.shape[0]
    gx = np.zeros((B, T, K), np.float32)
    gw = np.zeros((F, K), np.float32)
    _load().oracle_gemm_bwd(_p(x), _p(w), _p(g), _p(gx), _p(gw), B, T, K, F, int(bf16_x), int(bf16_w))
    return gx, gw


def layer_fwd_bwd(x, w, inits, logit_bias, gq, gk, gv, NH, NKVH, Da, r, bf16, use_sigmoid=True, acc=np.float64):
    """Whole filtered-QKV layer, forward and backward, as the reference composes it:
    combined = W x^T (rounded to dtype), scan, then the scan backward and the projection
    backward. Returns a dict of every output and gradient. `acc`: the GEMMs' accumulation type
    (float64: the oracle; float32: the reference's own fp32-accumulated arithmetic)."""
    comb = gemm_fwd(x, w, bf16, acc)                  # [B, F, T]
    comb_btf = np.ascontiguousarray(comb.transpose(0, 2, 1))
    hq, hk, hv = scan_fwd(comb_btf, inits, logit_bias, NH, NKVH, Da, r, use_sigmoid, bf16)
    gc, gi, gb = scan_bwd(comb_btf, inits, logit_bias, gq, gk, gv, NH, NKVH, Da, r, use_sigmoid, bf16)
    gx, gw = gemm_bwd(x, w, np.ascontiguousarray(gc.transpose(0, 2, 1)), bf16, False, acc)
    return dict(combined=comb, hq=hq, hk=hk, hv=hv, grad_combined=gc, grad_inits=gi, grad_logit_bias=gb,
                grad_x=gx, grad_w=gw)
