"""Pins the CPU oracle (oracle/ltv_oracle.c) to golden vectors of the reference's own oracle.

The .npz files were produced by tests/golden/make_golden.py from the reference's
nanochat/ops/ltv_reference_ops.py (torch autograd on CPU). The oracle must reproduce them:
forward outputs bit-exactly; gradients bit-exactly except where fp32 summation order differs
(the reference sums group reductions and the bias gradient in torch's own order), bounded below.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import load_golden, max_rel_err
from oracle import oracle as O


def _parse(key):
    parts = key.split("_")
    return parts[0], {p.rstrip("0123456789"): int(p[len(p.rstrip("0123456789")):]) for p in parts[1:]}


PATTERNED = load_golden("scan_patterned.npz")
RANDOM = load_golden("scan_random.npz")
LOOKBACK = load_golden("scan_lookback.npz")
GEMM = load_golden("gemm.npz")


@pytest.mark.parametrize("key", sorted(PATTERNED))
def test_oracle_patterned_exact(key):
    """Integer-pattern cases of the reference kernel tests: exact for every output and grad."""
    c = PATTERNED[key]
    dt, p = _parse(key)
    bf16 = dt == "bf16"
    sig = bool(p["sig"])
    r = p["r"]
    da = 2 // r
    hq, hk, hv = O.scan_fwd(c["combined"], c["inits"], c["logit_bias"], 8, 8, da, r, sig, bf16)
    np.testing.assert_array_equal(hq, c["hq"])
    np.testing.assert_array_equal(hk, c["hk"])
    np.testing.assert_array_equal(hv, c["hv"])
    gc, gi, gb = O.scan_bwd(c["combined"], c["inits"], c["logit_bias"], c["gq"], c["gk"], c["gv"], 8, 8, da, r, sig,
                            bf16)
    np.testing.assert_array_equal(gc, c["grad_combined"])
    np.testing.assert_array_equal(gi, c["grad_inits"])
    assert max_rel_err(gb, c["grad_logit_bias"]) <= 1e-6


def _grad_tols(bf16):
    # fp32: summation order of the r-channel group sums (reference: torch reduction order).
    # bf16: additionally a different fp32 sum can round to the neighbouring bfloat16 value.
    return (2e-2, 1e-2) if bf16 else (1e-4, 1e-2)


@pytest.mark.parametrize("key", sorted(RANDOM))
def test_oracle_random_d128(key):
    c = RANDOM[key]
    dt, p = _parse(key)
    bf16 = dt == "bf16"
    NH, NKVH, Da, r = p["NH"], p["NKVH"], p["Da"], p["r"]
    hq, hk, hv = O.scan_fwd(c["combined"], c["inits"], c["logit_bias"], NH, NKVH, Da, r, True, bf16)
    for a, n in ((hq, "hq"), (hk, "hk"), (hv, "hv")):
        np.testing.assert_array_equal(a, c[n])
    gc, gi, gb = O.scan_bwd(c["combined"], c["inits"], c["logit_bias"], c["gq"], c["gk"], c["gv"], NH, NKVH, Da, r,
                            True, bf16)
    tol, floor = _grad_tols(bf16)
    assert max_rel_err(gc, c["grad_combined"], floor) <= tol
    np.testing.assert_array_equal(gi, c["grad_inits"])
    assert max_rel_err(gb, c["grad_logit_bias"]) <= 1e-5


@pytest.mark.parametrize("key", sorted(LOOKBACK))
def test_oracle_lookback_chunks(key):
    c = LOOKBACK[key]
    dt, p = _parse(key)
    bf16 = dt == "bf16"
    pqk = (p["P"], p["Q"], p["K"])
    hq, hk, hv = O.scan_fwd(c["combined"], c["inits"], c["logit_bias"], 1, 1, 1, 32, True, bf16, pqk)
    for a, n in ((hq, "hq"), (hk, "hk"), (hv, "hv")):
        np.testing.assert_array_equal(a, c[n])
    gc, gi, gb = O.scan_bwd(c["combined"], c["inits"], c["logit_bias"], c["gq"], c["gk"], c["gv"], 1, 1, 1, 32, True,
                            bf16, pqk)
    tol, floor = _grad_tols(bf16)
    assert max_rel_err(gc, c["grad_combined"], floor) <= tol
    assert max_rel_err(gi, c["grad_inits"]) <= 1e-5
    assert max_rel_err(gb, c["grad_logit_bias"]) <= 2e-5


@pytest.mark.parametrize("key", sorted(GEMM))
def test_oracle_gemm(key):
    c = GEMM[key]
    bf16 = key.startswith("bf16")
    # The reference accumulates in fp32 (torch CPU matmul), the oracle in double; the bounds
    # are the reference's own GEMM test tolerances (tests/test_fused_linear_transpose.py:74-76).
    # Both forms of the oracle's contraction (numpy float64 BLAS, and ltv_oracle.c's loops) are
    # pinned, and they agree with each other to float64 summation noise before the final rounding.
    tol = 5e-2 if bf16 else 1e-4
    out = O.gemm_fwd(c["x"], c["w"], bf16)
    gx, gw = O.gemm_bwd(c["x"], c["w"], c["g"], bf16, bf16)
    out_c = O.gemm_fwd_c(c["x"], c["w"], bf16)
    gx_c, gw_c = O.gemm_bwd_c(c["x"], c["w"], c["g"], bf16, bf16)
    for a, ac, n in ((out, out_c, "out"), (gx, gx_c, "grad_x"), (gw, gw_c, "grad_w")):
        assert max_rel_err(a, c[n], 1e-2) <= tol, n
        assert max_rel_err(ac, c[n], 1e-2) <= tol, n
        assert max_rel_err(a, ac, 1e-2) <= (8e-3 if bf16 else 1e-6), n  # at most one rounding flip apart


def test_oracle_layer_composition_small():
    """layer_fwd_bwd composes projection and scan exactly as the reference filter does."""
    rng = np.random.default_rng(0)
    B, T, C, NH, NKVH, Da, r = 2, 9, 16, 1, 1, 1, 4
    H, D = NH + 2 * NKVH, Da * r
    F = H * (D + Da)
    x = rng.standard_normal((B, T, C)).astype(np.float32)
    w = (rng.standard_normal((F, C)) / 4).astype(np.float32)
    inits = rng.standard_normal((B, H, D)).astype(np.float32)
    bias = rng.standard_normal((H, Da)).astype(np.float32)
    gq = rng.standard_normal((B, NH, T, D)).astype(np.float32)
    gk = rng.standard_normal((B, NKVH, T, D)).astype(np.float32)
    gv = rng.standard_normal((B, NKVH, T, D)).astype(np.float32)
    res = O.layer_fwd_bwd(x, w, inits, bias, gq, gk, gv, NH, NKVH, Da, r, bf16=False)
    comb = np.einsum("btc,fc->bft", x.astype(np.float64), w.astype(np.float64))
    np.testing.assert_allclose(res["combined"], comb, rtol=1e-6, atol=1e-6)
    # grad_x / grad_w against a direct contraction of grad_combined
    gcomb = res["grad_combined"].transpose(0, 2, 1).astype(np.float64)  # [B, F, T]
    np.testing.assert_allclose(res["grad_x"], np.einsum("bft,fc->btc", gcomb, w), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(res["grad_w"], np.einsum("bft,btc->fc", gcomb, x), rtol=1e-5, atol=1e-5)
