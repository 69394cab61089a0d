"""GPU parity of the scan operator against the reference's golden vectors and the oracle.

Ports the reference's kernel tests (tests/test_ltv_cuda_fused_concat_head_major_register_cast_blelloch_scan.py:28-261):
patterned integer inputs, seq_len 1, 2, 3, 31, 32, 33, every divisor r of head dim 2, every dense
stride layout of `combined` (with and without gaps), all-ones upstream gradients, tolerance
exact without sigmoid and atol = rtol = 0.025 with sigmoid (tests/ltv_scan_test_utils.py:134-140).
Beyond that: production head dim 128 with several look-back chunks, the benchmark shapes at full
size against the CPU oracle (max relative error with an absolute floor: <= 1e-5 fp32,
<= 2e-2 bf16), transposed q/k gradient layouts, and the bounded-wait failure path.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import nanochat_filter_b200  # noqa: F401  (registers torch.ops.nanochat_cuda)
from conftest import load_golden, max_rel_err, storage_size, stride_layouts
from nanochat_filter_b200 import _lib
from oracle import oracle as O

pytestmark = pytest.mark.gpu

SCAN = torch.ops.nanochat_cuda.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_op
DT = {"f32": torch.float32, "bf16": torch.bfloat16}
PATTERNED = load_golden("scan_patterned.npz")
RANDOM = load_golden("scan_random.npz")
# Relative errors are taken against max(|expected|, FLOOR * max|expected|): the group sums of the
# logit gradient cancel, and fp32 summation order alone moves entries near zero.
FLOOR = 1e-2


def strided_copy(arr: np.ndarray, dtype, device, stride):
    """Device tensor holding `arr` with the given strides; gaps are filled with NaN so that a
    kernel reading outside the view shows up in the results."""
    shape = arr.shape
    base = torch.full((storage_size(shape, stride),), float("nan"), dtype=dtype, device=device)
    view = torch.as_strided(base, shape, stride)
    view.copy_(torch.from_numpy(arr).to(dtype))
    return view


def run_scan(combined, inits, bias, NH, NKVH, da, r, sig, gq, gk, gv):
    combined = combined.detach().requires_grad_(True)
    inits = inits.detach().requires_grad_(True)
    bias = bias.detach().requires_grad_(True)
    q, k, v = SCAN(combined, inits, bias, NH, NKVH, da, r, 8, 8, 4, 32, 2, 8, sig)
    torch.autograd.backward([q, k, v], [gq, gk, gv])
    return q, k, v, combined.grad, inits.grad, bias.grad


def _np(t):
    return t.detach().float().cpu().numpy()


def _patterned_keys():
    return sorted(PATTERNED)


@pytest.mark.parametrize("key", _patterned_keys())
def test_scan_patterned_all_stride_layouts(cuda_device, key):
    c = PATTERNED[key]
    dname, sig_s, T_s, r_s = key.split("_")
    dtype = DT[dname]
    sig = sig_s == "sig1"
    r = int(r_s[1:])
    da = 2 // r
    tol = dict(rtol=0.025, atol=0.025) if sig else dict(rtol=0, atol=0)
    dev = cuda_device
    inits = torch.from_numpy(c["inits"]).to(dev, dtype)
    bias = torch.from_numpy(c["logit_bias"]).to(dev)
    gq, gk, gv = (torch.from_numpy(c[n]).to(dev, dtype) for n in ("gq", "gk", "gv"))
    for stride in stride_layouts(c["combined"].shape):
        comb = strided_copy(c["combined"], dtype, dev, stride)
        q, k, v, gc, gi, gb = run_scan(comb, inits, bias, 8, 8, da, r, sig, gq, gk, gv)
        case = f"{key} stride={stride}"
        for a, n in ((q, "hq"), (k, "hk"), (v, "hv"), (gc, "grad_combined"), (gi, "grad_inits"),
                     (gb, "grad_logit_bias")):
            np.testing.assert_allclose(_np(a), c[n], err_msg=f"{n} {case}", **tol)
    assert _lib.all_workspace_errors() == 0


@pytest.mark.parametrize("key", sorted(RANDOM))
def test_scan_random_d128_vs_reference(cuda_device, key):
    c = RANDOM[key]
    p = dict((s.rstrip("0123456789"), int(s[len(s.rstrip("0123456789")):])) for s in key.split("_")[1:])
    dtype = DT[key.split("_")[0]]
    dev = cuda_device
    comb = torch.from_numpy(c["combined"]).to(dev, dtype)
    # the production layout: the transposed view of a [B, F, T] projection buffer
    comb = comb.transpose(1, 2).contiguous().transpose(1, 2)
    inits = torch.from_numpy(c["inits"]).to(dev, dtype)
    bias = torch.from_numpy(c["logit_bias"]).to(dev)
    gq, gk, gv = (torch.from_numpy(c[n]).to(dev, dtype) for n in ("gq", "gk", "gv"))
    q, k, v, gc, gi, gb = run_scan(comb, inits, bias, p["NH"], p["NKVH"], p["Da"], p["r"], True, gq, gk, gv)
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
    for a, n in ((q, "hq"), (k, "hk"), (v, "hv"), (gc, "grad_combined"), (gi, "grad_inits"),
                 (gb, "grad_logit_bias")):
        assert max_rel_err(_np(a), c[n], FLOOR) <= tol, n


def _random_case(seed, B, T, NH, NKVH, Da, r, bias_shift=0.0, logit_scale=1.0):
    rng = np.random.default_rng(seed)
    H, D = NH + 2 * NKVH, Da * r
    vals = rng.standard_normal((B, T, H, D)).astype(np.float32)
    logits = (logit_scale * rng.standard_normal((B, T, H, Da))).astype(np.float32)
    comb = np.concatenate([vals, logits], axis=3).reshape(B, T, H * (D + Da))
    inits = (0.5 * rng.standard_normal((B, H, D))).astype(np.float32)
    bias = (rng.standard_normal((H, Da)) * 0.5 + bias_shift).astype(np.float32)
    gq = rng.standard_normal((B, NH, T, D)).astype(np.float32)
    gk = rng.standard_normal((B, NKVH, T, D)).astype(np.float32)
    gv = rng.standard_normal((B, NKVH, T, D)).astype(np.float32)
    return comb, inits, bias, gq, gk, gv


def _check_vs_oracle(dev, dtype, B, T, NH, NKVH, Da, r, seed, bias_shift=0.0, layout="bft", transposed_qk=False):
    bf16 = dtype == torch.bfloat16
    comb, inits, bias, gq, gk, gv = _random_case(seed, B, T, NH, NKVH, Da, r, bias_shift)
    if bf16:
        comb, inits, gq, gk, gv = (O.round_bf16(a) for a in (comb, inits, gq, gk, gv))
    tc = torch.from_numpy(comb).to(dev, dtype)
    if layout == "bft":
        tc = tc.transpose(1, 2).contiguous().transpose(1, 2)
    ti = torch.from_numpy(inits).to(dev, dtype)
    tb = torch.from_numpy(bias).to(dev)
    tg = [torch.from_numpy(a).to(dev, dtype) for a in (gq, gk, gv)]
    if transposed_qk:
        # gradients as the attention layer hands them back: [B, T, H, D] storage viewed [B, H, T, D]
        tg[0] = tg[0].transpose(1, 2).contiguous().transpose(1, 2)
        tg[1] = tg[1].transpose(1, 2).contiguous().transpose(1, 2)
    q, k, v, gc, gi, gb = run_scan(tc, ti, tb, NH, NKVH, Da, r, True, *tg)
    eq, ek, ev = O.scan_fwd(comb, inits, bias, NH, NKVH, Da, r, True, bf16)
    # the oracle replays its own forward for the backward (QuantizedStateUpdate semantics); a
    # one-ulp difference in a stored bf16 h_{t-1} stays far inside the bf16 bound
    egc, egi, egb = O.scan_bwd(comb, inits, bias, gq, gk, gv, NH, NKVH, Da, r, True, bf16)
    tol = 2e-2 if bf16 else 1e-5
    errs = {n: max_rel_err(_np(a), e, FLOOR) for a, e, n in (
        (q, eq, "hq"), (k, ek, "hk"), (v, ev, "hv"), (gc, egc, "grad_combined"), (gi, egi, "grad_inits"),
        (gb, egb, "grad_logit_bias"))}
    assert _lib.all_workspace_errors() == 0
    bad = {n: e for n, e in errs.items() if e > tol}
    assert not bad, f"max rel err above {tol}: {bad} (all: {errs})"


# T = 700 takes the generic chunked kernels (T not a multiple of 8), T = 704 and 1000 the
# vectorised bf16 kernels (704: eleven full 64-token chunks; 1000: a partial last chunk).
@pytest.mark.parametrize("T", [700, 704, 1000])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("Da,r", [(1, 128), (2, 64), (4, 32)])
def test_scan_multichunk_vs_oracle(cuda_device, dtype, Da, r, T):
    _check_vs_oracle(cuda_device, dtype, B=3, T=T, NH=2, NKVH=1, Da=Da, r=r, seed=Da)


@pytest.mark.parametrize("T", [333, 336])
@pytest.mark.parametrize("layout", ["bft", "btf"])
def test_scan_layouts_and_transposed_grads(cuda_device, layout, T):
    _check_vs_oracle(cuda_device, torch.bfloat16, B=2, T=T, NH=2, NKVH=2, Da=1, r=128, seed=5, layout=layout,
                     transposed_qk=True)


def test_scan_head_dim_64_and_256(cuda_device):
    _check_vs_oracle(cuda_device, torch.bfloat16, B=2, T=256, NH=1, NKVH=1, Da=1, r=64, seed=6)
    _check_vs_oracle(cuda_device, torch.bfloat16, B=2, T=256, NH=1, NKVH=1, Da=2, r=128, seed=7)


def test_scan_baseline_config2_full_size(cuda_device):
    """d=12 training shape (B=32, T=1024, 6+6+6 heads x 128, r=128), bf16, against the oracle."""
    _check_vs_oracle(cuda_device, torch.bfloat16, B=32, T=1024, NH=6, NKVH=6, Da=1, r=128, seed=2)


def test_scan_baseline_config3_long_sequence(cuda_device):
    """Long-sequence stress (B=4, T=16384, 8+8+8 heads x 128), decay a ~= 0.95 (logit bias -3),
    many chained look-back chunks, against the oracle."""
    _check_vs_oracle(cuda_device, torch.bfloat16, B=4, T=16384, NH=8, NKVH=8, Da=1, r=128, seed=3, bias_shift=-3.0)


def test_scan_config1_fp32(cuda_device):
    """Config-1 shape (B=2, T=256, 6+6+6 heads x 128) in fp32 against the oracle at 1e-5."""
    _check_vs_oracle(cuda_device, torch.float32, B=2, T=256, NH=6, NKVH=6, Da=1, r=128, seed=1)


def test_scan_empty_sequence(cuda_device):
    dev = cuda_device
    comb = torch.empty(2, 0, 3 * 3, device=dev, dtype=torch.bfloat16, requires_grad=True)
    inits = torch.randn(2, 3, 2, device=dev, dtype=torch.bfloat16, requires_grad=True)
    bias = torch.zeros(3, 1, device=dev, requires_grad=True)
    q, k, v = SCAN(comb, inits, bias, 1, 1, 1, 2, 8, 8, 4, 32, 2, 8, True)
    assert q.shape == (2, 1, 0, 2)
    (q.sum() + k.sum() + v.sum()).backward()
    assert torch.all(inits.grad == 0)


def test_scan_repeated_calls_reuse_workspace(cuda_device):
    """Back-to-back launches on one workspace (epoch-tagged flags, self-resetting counters)."""
    for i in range(3):
        _check_vs_oracle(cuda_device, torch.bfloat16, B=2, T=200, NH=1, NKVH=1, Da=1, r=128, seed=10 + i)


def test_bounded_wait_reports_timeout(cuda_device):
    """A device-side wait on a flag nothing sets gives up after its limit, records
    LTVQKV_ERR_TIMEOUT for the host, and the context stays usable."""
    L = _lib.load()
    ws = torch.zeros(4096, dtype=torch.uint8, device=cuda_device)
    rc = L.ltvqkv_debug_wait_timeout(ws.data_ptr(), 50_000_000, _lib.stream_handle(cuda_device))
    assert rc == 0
    assert _lib.workspace_error(ws) == 7  # LTVQKV_ERR_TIMEOUT
    assert _lib.workspace_error(ws) == 0  # cleared by the read
    _check_vs_oracle(cuda_device, torch.bfloat16, B=1, T=100, NH=1, NKVH=1, Da=1, r=128, seed=9)


def test_scan_is_deterministic_run_to_run(cuda_device):
    """Carries are composed in a fixed association (anchored look-back), so repeated runs —
    whatever the tile timing — give identical bits, forward and backward."""
    dev = cuda_device
    comb, inits, bias, gq, gk, gv = _random_case(11, 4, 4096, 2, 2, 1, 128, -3.0)
    tc = torch.from_numpy(O.round_bf16(comb)).to(dev, torch.bfloat16).transpose(1, 2).contiguous().transpose(1, 2)
    ti = torch.from_numpy(O.round_bf16(inits)).to(dev, torch.bfloat16)
    tb = torch.from_numpy(bias).to(dev)
    tg = [torch.from_numpy(O.round_bf16(a)).to(dev, torch.bfloat16) for a in (gq, gk, gv)]
    first = run_scan(tc, ti, tb, 2, 2, 1, 128, True, *tg)
    for _ in range(3):
        again = run_scan(tc, ti, tb, 2, 2, 1, 128, True, *tg)
        for a, e in zip(again, first):
            assert torch.equal(a, e)


# Many (batch, head) rows (>= 2 per SM slot) take the row-streaming kernels: a CTA walks whole
# rows chunk by chunk with the carry in registers.
@pytest.mark.parametrize("T", [64, 200, 520])
@pytest.mark.parametrize("Da,r", [(1, 128), (2, 64), (4, 32), (1, 64), (2, 128), (1, 256)])
def test_scan_row_streaming_path_vs_oracle(cuda_device, T, Da, r):
    _check_vs_oracle(cuda_device, torch.bfloat16, B=64, T=T, NH=2, NKVH=2, Da=Da, r=r, seed=T + Da,
                     transposed_qk=True)


# A ragged last chunk (1000 = 15 * 64 + 40) on the row-streaming path, head dim 128.
def test_scan_row_streaming_ragged_tail(cuda_device):
    _check_vs_oracle(cuda_device, torch.bfloat16, B=60, T=1000, NH=3, NKVH=1, Da=1, r=128, seed=5,
                     transposed_qk=False)

