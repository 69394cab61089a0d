"""Generates the golden vectors of tests/golden/ from the reference's own CPU oracle.

Run in a container that has the reference checkout (read-only) at REFERENCE_ROOT:

    python tests/golden/make_golden.py [REFERENCE_ROOT]

It imports nanochat/ops/ltv_reference_ops.py by file path (that module needs only torch) and
records, for seeded or patterned inputs, the outputs and autograd gradients of
  - ltv_fused_concat_head_major_register_cast_blelloch_scan_minimal (ltv_reference_ops.py:162-192)
  - ltv_look_back_fused_concat_head_major_register_cast_sequential_scan_minimal (:37-124)
  - fused_linear_transpose_reference (:299-308)
The patterned inputs follow the reference's kernel tests (tests/ltv_scan_test_utils.py:84-131:
batch 4, 8 query + 8 kv heads, total head dim 2, every divisor r, seq_len 1, 2, 3, 31, 32, 33,
all-ones upstream gradients). Nothing here runs on the GPU box: the .npz files are the record.
"""

from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference_ops(root: str):
    path = os.path.join(root, "nanochat", "ops", "ltv_reference_ops.py")
    spec = importlib.util.spec_from_file_location("ref_ltv_reference_ops", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float32).contiguous().numpy()


def patterned_inputs(batch, nh, nkvh, seq_len, da, r, sigmoid, dtype):
    """Integer patterns of the reference's kernel tests (tests/ltv_scan_test_utils.py:84-131)."""
    total_h = nh + 2 * nkvh
    D = da * r
    fph = D + da
    b = torch.arange(batch).view(batch, 1, 1, 1)
    t = torch.arange(seq_len).view(1, seq_len, 1, 1)
    h = torch.arange(total_h).view(1, 1, total_h, 1)
    d = torch.arange(D).view(1, 1, 1, D)
    g = torch.arange(da).view(1, 1, 1, da)
    vals = ((9 * b + 7 * t + 3 * h + d) % 5) - 2
    logits = (b + t + h + g) % 2
    combined = torch.cat([vals.expand(batch, seq_len, total_h, D), logits.expand(batch, seq_len, total_h, da)], dim=3)
    combined = combined.reshape(batch, seq_len, total_h * fph).to(dtype)
    bi = torch.arange(batch).view(batch, 1, 1)
    hi = torch.arange(total_h).view(1, total_h, 1)
    di = torch.arange(D).view(1, 1, D)
    inits = (((13 * bi + 3 * hi + di) % 7) - 3).to(dtype)
    hh = torch.arange(total_h).view(total_h, 1)
    gg = torch.arange(da).view(1, da)
    bias = (((hh + 2 * gg) % 3) - 1).to(torch.float32) if sigmoid else torch.zeros(total_h, da)
    return combined, inits, bias


def random_inputs(gen, batch, nh, nkvh, seq_len, da, r, dtype, logit_shift=0.0):
    total_h = nh + 2 * nkvh
    D = da * r
    vals = torch.randn(batch, seq_len, total_h, D, generator=gen)
    logits = torch.randn(batch, seq_len, total_h, da, generator=gen) + logit_shift
    combined = torch.cat([vals, logits], dim=3).reshape(batch, seq_len, total_h * (D + da)).to(dtype)
    inits = (0.5 * torch.randn(batch, total_h, D, generator=gen)).to(dtype)
    bias = torch.randn(total_h, da, generator=gen)
    return combined, inits, bias


def run_scan(ops, combined, inits, bias, nh, nkvh, da, r, sigmoid, grads=None, gen=None, pqk=None):
    c = combined.clone().requires_grad_(True)
    i = inits.clone().requires_grad_(True)
    lb = bias.clone().requires_grad_(True)
    if pqk is None:
        q, k, v = ops.ltv_fused_concat_head_major_register_cast_blelloch_scan_minimal(
            c, i, lb, nh, nkvh, da, r, 2147483647, 1, 1, sigmoid)
    else:
        P, Q, K = pqk
        q, k, v = ops.ltv_look_back_fused_concat_head_major_register_cast_sequential_scan_minimal(
            c, i, lb, nh, nkvh, da, r, P, Q, K, sigmoid)
    if grads == "ones":
        gq, gk, gv = torch.ones_like(q), torch.ones_like(k), torch.ones_like(v)
    else:
        gq = torch.randn(q.shape, generator=gen).to(q.dtype)
        gk = torch.randn(k.shape, generator=gen).to(k.dtype)
        gv = torch.randn(v.shape, generator=gen).to(v.dtype)
    torch.autograd.backward([q, k, v], [gq, gk, gv])
    return dict(
        combined=to_np(combined), inits=to_np(inits), logit_bias=to_np(bias),
        hq=to_np(q), hk=to_np(k), hv=to_np(v), gq=to_np(gq), gk=to_np(gk), gv=to_np(gv),
        grad_combined=to_np(c.grad), grad_inits=to_np(i.grad), grad_logit_bias=to_np(lb.grad),
    )


def main(root: str) -> None:
    ops = load_reference_ops(root)
    torch.manual_seed(0)
    dtypes = {"f32": torch.float32, "bf16": torch.bfloat16}

    # 1) Patterned cases of the reference kernel tests.
    cases = {}
    for dname, dt in dtypes.items():
        for sigmoid in (True, False):
            for seq_len in (1, 2, 3, 31, 32, 33):
                for r in (1, 2):
                    da = 2 // r
                    combined, inits, bias = patterned_inputs(4, 8, 8, seq_len, da, r, sigmoid, dt)
                    res = run_scan(ops, combined, inits, bias, 8, 8, da, r, sigmoid, grads="ones")
                    key = f"{dname}_sig{int(sigmoid)}_T{seq_len}_r{r}"
                    for name, arr in res.items():
                        cases[f"{key}/{name}"] = arr
    np.savez_compressed(os.path.join(HERE, "scan_patterned.npz"), **cases)

    # 2) Random inputs at the production head dim (D = 128) with r = 128 and r = 64.
    gen = torch.Generator().manual_seed(1234)
    cases = {}
    for dname, dt in dtypes.items():
        for (batch, nh, nkvh, seq_len, da, r, shift) in ((2, 1, 1, 40, 1, 128, 0.0), (1, 2, 1, 67, 2, 64, -2.0)):
            combined, inits, bias = random_inputs(gen, batch, nh, nkvh, seq_len, da, r, dt, shift)
            res = run_scan(ops, combined, inits, bias, nh, nkvh, da, r, True, grads="randn", gen=gen)
            key = f"{dname}_B{batch}_NH{nh}_NKVH{nkvh}_T{seq_len}_Da{da}_r{r}"
            for name, arr in res.items():
                cases[f"{key}/{name}"] = arr
    np.savez_compressed(os.path.join(HERE, "scan_random.npz"), **cases)

    # 3) Look-back (P, Q, K) chunked scans (ltv_reference_ops.py:37-124).
    gen = torch.Generator().manual_seed(77)
    cases = {}
    for (P, Q, K) in ((2147483647, 1, 1), (64, 60, 5), (16, 12, 5), (8, 6, 3)):
        for dname, dt in dtypes.items():
            combined, inits, bias = random_inputs(gen, 2, 1, 1, 70, 1, 32, dt)
            res = run_scan(ops, combined, inits, bias, 1, 1, 1, 32, True, grads="randn", gen=gen, pqk=(P, Q, K))
            key = f"{dname}_P{P}_Q{Q}_K{K}"
            for name, arr in res.items():
                cases[f"{key}/{name}"] = arr
    np.savez_compressed(os.path.join(HERE, "scan_lookback.npz"), **cases)

    # 4) Projection (fused linear transpose) and its gradients, reference GEMM test shapes
    #    (tests/test_fused_linear_transpose.py:36-41) minus the large one.
    gen = torch.Generator().manual_seed(4321)
    cases = {}
    for dname, dt in dtypes.items():
        for (B, T, K, F) in ((1, 16, 32, 128), (4, 128, 128, 256), (2, 31, 63, 127), (2, 24, 96, 387)):
            x = (torch.randn(B, T, K, generator=gen) / K**0.5).to(dt).requires_grad_(True)
            w = (torch.randn(F, K, generator=gen) / K**0.5).to(dt).requires_grad_(True)
            out = ops.fused_linear_transpose_reference(x, w)
            g = torch.randn(out.shape, generator=gen).to(dt)
            out.backward(g)
            key = f"{dname}_B{B}_T{T}_K{K}_F{F}"
            cases[f"{key}/x"] = to_np(x)
            cases[f"{key}/w"] = to_np(w)
            cases[f"{key}/out"] = to_np(out)
            cases[f"{key}/g"] = to_np(g)
            cases[f"{key}/grad_x"] = to_np(x.grad)
            cases[f"{key}/grad_w"] = to_np(w.grad)
    np.savez_compressed(os.path.join(HERE, "gemm.npz"), **cases)


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py REFERENCE_ROOT (the nanochat-filter checkout)")
    main(root)
