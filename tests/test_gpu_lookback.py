"""GPU parity of the look-back (chunk-restarting) scan operators.

Ports the reference's look-back kernel tests
(tests/test_ltv_cuda_look_back_fused_concat_head_major_register_cast_{blelloch,sequential}_scan.py):
patterned integer inputs, seq_len 1, 2, 3, 31, 32, 33, every divisor r of head dim 2, every dense
stride layout of `combined`, the reference's (P, Q, K) configurations
(tests/ltv_scan_test_utils.py:11-19), all-ones upstream gradients, exact without sigmoid and
atol = rtol = 0.025 with sigmoid. At those lengths every configuration is a single chunk, so the
expected values are the plain scan's golden vectors. Chunking proper is pinned by the golden
vectors of the reference's sequential oracle (ltv_reference_ops.py:37-124; P/Q/K with warm-up
prefixes, T = 70) and by the CPU oracle at head dim 128 with long, overlapping prefixes.
Tolerances: fp32 max relative error (absolute floor 1e-2 of the largest value) 1e-5 on outputs and
on grad_inits / grad_logit_bias, and on grad_combined the oracle pinning bound; bf16 2e-2.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import nanochat_filter_b200  # noqa: F401
from conftest import load_golden, max_rel_err, stride_layouts
from nanochat_filter_b200 import _lib
from oracle import oracle as O
from test_gpu_scan import strided_copy

pytestmark = pytest.mark.gpu

OPS = torch.ops.nanochat_cuda
LB = "ltv_look_back_fused_concat_head_major_register_cast_{}_scan_cuda_op"
KINDS = ("blelloch", "sequential")
DT = {"f32": torch.float32, "bf16": torch.bfloat16}
PATTERNED = load_golden("scan_patterned.npz")
LOOKBACK = load_golden("scan_lookback.npz")
SUPPORTED_PQK = [(2147483647, 1, 1), (1024, 1024, 1), (64, 60, 5), (128, 112, 17), (160, 108, 53),
                 (192, 104, 89), (224, 100, 125)]
FLOOR = 1e-2


def run_lb(kind, combined, inits, bias, NH, NKVH, da, r, P, Q, K, sig, grads):
    combined = combined.detach().requires_grad_(True)
    inits = inits.detach().requires_grad_(True)
    bias = bias.detach().requires_grad_(True)
    op = getattr(OPS, LB.format(kind))
    tuning = (8, 8, 4, 32, 2, 8) if kind == "blelloch" else (2, 4, 2, 8)
    q, k, v = op(combined, inits, bias, NH, NKVH, da, r, P, Q, K, *tuning, sig)
    torch.autograd.backward([q, k, v], list(grads))
    return q, k, v, combined.grad, inits.grad, bias.grad


def _np(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("pqk", SUPPORTED_PQK[:4])
@pytest.mark.parametrize("key", sorted(k for k in PATTERNED if "_T3" in k or "_T33" in k or "_T1_" in k))
def test_lookback_reference_port(cuda_device, kind, pqk, key):
    c = PATTERNED[key]
    dname, sig_s, _, r_s = key.split("_")
    dtype = DT[dname]
    sig = sig_s == "sig1"
    r = int(r_s[1:])
    da = 2 // r
    tol = dict(rtol=0.025, atol=0.025) if sig else dict(rtol=0, atol=0)
    dev = cuda_device
    inits = torch.from_numpy(c["inits"]).to(dev, dtype)
    bias = torch.from_numpy(c["logit_bias"]).to(dev)
    grads = [torch.from_numpy(c[n]).to(dev, dtype) for n in ("gq", "gk", "gv")]
    for stride in stride_layouts(c["combined"].shape)[::5]:
        comb = strided_copy(c["combined"], dtype, dev, stride)
        res = run_lb(kind, comb, inits, bias, 8, 8, da, r, *pqk, sig, grads)
        for a, n in zip(res, ("hq", "hk", "hv", "grad_combined", "grad_inits", "grad_logit_bias")):
            np.testing.assert_allclose(_np(a), c[n], err_msg=f"{n} {key} {pqk} stride={stride}", **tol)
    assert _lib.all_workspace_errors() == 0


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("key", sorted({k.split("/")[0] for k in LOOKBACK}))
def test_lookback_golden_chunks(cuda_device, kind, key):
    """Chunked cases (P < T) against the reference's sequential look-back oracle."""
    c = LOOKBACK[key]
    dname = key.split("_")[0]
    P, Q, K = (int(s[1:]) for s in key.split("_")[1:])
    dtype = DT[dname]
    dev = cuda_device
    comb = torch.from_numpy(c["combined"]).to(dev, dtype)
    inits = torch.from_numpy(c["inits"]).to(dev, dtype)
    bias = torch.from_numpy(c["logit_bias"]).to(dev)
    grads = [torch.from_numpy(c[n]).to(dev, dtype) for n in ("gq", "gk", "gv")]
    res = run_lb(kind, comb, inits, bias, 1, 1, 1, 32, P, Q, K, True, grads)
    bf16 = dtype == torch.bfloat16
    for a, n in zip(res, ("hq", "hk", "hv", "grad_combined", "grad_inits", "grad_logit_bias")):
        tol = 2e-2 if bf16 else (2e-5 if n == "grad_logit_bias" else 1e-5)
        if n == "grad_combined" and not bf16:
            tol = 1e-4  # the reference sums overlapping prefixes through autograd in its own order
        assert max_rel_err(_np(a), c[n], FLOOR) <= tol, n


def _random(seed, B, T, NH, NKVH, Da, r):
    rng = np.random.default_rng(seed)
    H, D = NH + 2 * NKVH, Da * r
    vals = rng.standard_normal((B, T, H, D)).astype(np.float32)
    logits = rng.standard_normal((B, T, H, Da)).astype(np.float32)
    comb = np.concatenate([vals, logits], axis=3).reshape(B, T, H * (D + Da))
    inits = (0.5 * rng.standard_normal((B, H, D))).astype(np.float32)
    bias = (rng.standard_normal((H, Da)) * 0.5).astype(np.float32)
    gq = rng.standard_normal((B, NH, T, D)).astype(np.float32)
    gk = rng.standard_normal((B, NKVH, T, D)).astype(np.float32)
    gv = rng.standard_normal((B, NKVH, T, D)).astype(np.float32)
    return comb, inits, bias, gq, gk, gv


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,T,NH,NKVH,Da,r,P,Q,K", [
    (2, 300, 1, 1, 1, 128, 64, 60, 5),
    (2, 300, 1, 1, 1, 128, 224, 100, 125),   # prefixes longer than the chunks they precede
    (1, 257, 2, 1, 2, 64, 16, 12, 40),        # each token in the prefixes of several chunks
    (3, 130, 1, 0, 4, 32, 32, 32, 1),         # restarts without a prefix
    (2, 100, 1, 1, 1, 128, 1024, 1024, 1),    # P >= T: the plain scan
])
def test_lookback_vs_oracle(cuda_device, dtype, B, T, NH, NKVH, Da, r, P, Q, K):
    bf16 = dtype == torch.bfloat16
    comb, inits, bias, gq, gk, gv = _random(B * 100 + T, B, T, NH, NKVH, Da, r)
    if bf16:
        comb, inits, gq, gk, gv = (O.round_bf16(a) for a in (comb, inits, gq, gk, gv))
    dev = cuda_device
    tc = torch.from_numpy(comb).to(dev, dtype).transpose(1, 2).contiguous().transpose(1, 2)
    res = run_lb("blelloch", tc, torch.from_numpy(inits).to(dev, dtype), torch.from_numpy(bias).to(dev), NH, NKVH,
                 Da, r, P, Q, K, True, [torch.from_numpy(a).to(dev, dtype) for a in (gq, gk, gv)])
    eq, ek, ev = O.scan_fwd(comb, inits, bias, NH, NKVH, Da, r, True, bf16, (P, Q, K))
    egc, egi, egb = O.scan_bwd(comb, inits, bias, gq, gk, gv, NH, NKVH, Da, r, True, bf16, (P, Q, K))
    tol = 2e-2 if bf16 else 1e-5
    for a, e, n in zip(res, (eq, ek, ev, egc, egi, egb), ("hq", "hk", "hv", "grad_combined", "grad_inits",
                                                          "grad_logit_bias")):
        if e.size == 0:
            continue
        assert max_rel_err(_np(a), e, FLOOR) <= tol, n
    assert _lib.all_workspace_errors() == 0


def test_lookback_plain_equals_scan_op(cuda_device):
    """P >= T is the plain scan: outputs equal the scan operator's within the bf16 bound."""
    comb, inits, bias, gq, gk, gv = _random(5, 2, 200, 2, 1, 1, 128)
    dev = cuda_device
    tc = torch.from_numpy(comb).to(dev, torch.bfloat16)
    ti = torch.from_numpy(inits).to(dev, torch.bfloat16)
    tb = torch.from_numpy(bias).to(dev)
    q1, k1, v1 = getattr(OPS, LB.format("sequential"))(tc, ti, tb, 2, 1, 1, 128, 2147483647, 1, 1, 2, 4, 2, 8, True)
    q2, k2, v2 = OPS.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_op(
        tc, ti, tb, 2, 1, 1, 128, 8, 8, 4, 32, 2, 8, True)
    for a, b in ((q1, q2), (k1, k2), (v1, v2)):
        assert max_rel_err(_np(a), _np(b), FLOOR) <= 2e-2


@pytest.mark.parametrize("variant", ["blelloch", "sequential"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_lookback_filter_decode_equals_batch(cuda_device, variant, dtype):
    """The look-back filter on the CUDA operators: token-by-token decode through the cache
    (advance_kv_cache) equals the chunked batch forward (bf16: within the bf16 bound, since the
    decode restarts from states stored in bf16)."""
    import nanochat_filter_b200 as nf

    spec = nf.ChunksAndHistory(p=16, q=12, k=5)
    cls = (nf.LtvLookBackFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter if variant == "blelloch"
           else nf.LtvLookBackFusedConcatHeadMajorRegisterCastSequentialScanQkvFilter)
    torch.manual_seed(0)
    filt = cls(2, 1, 128, 128, spec).to(cuda_device)
    filt.init_weights(2.0, 0.05, 0.5, 0.5)
    x = torch.randn(2, 40, 256, device=cuda_device).to(dtype)
    inits = filt.init_param.unsqueeze(0).expand(2, -1, -1)
    # bf16 as in training: fp32 parameters under autocast (the sequential variant's nn.Linear
    # projection then yields bf16)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16, enabled=dtype == torch.bfloat16):
        batch = filt(x, inits, full_recurrence=False)
        cache = nf.KVCache(2, 2, 1, 64, 128, num_layers=1, layer_specs=[spec])
        steps = [nf.advance_kv_cache(x[:, t:t + 1], 0, filt, inits, cache) for t in range(40)]
    for i in range(3):
        dec = torch.cat([s[i] for s in steps], dim=1)
        if dtype == torch.float32:
            torch.testing.assert_close(dec, batch[i], rtol=1e-5, atol=1e-5)
        else:
            # every decode step restarts from a state stored in bf16, so rounding accumulates over
            # the 40 steps: norm-wise bound, as for the whole bf16 layer
            d, e = _np(dec), _np(batch[i])
            assert np.abs(d - e).max() <= 2e-2 * np.abs(e).max()


def _bwd_abi(comb, inits, bias, outs, grads, NH, NKVH, Da, r, P, Q, K, ws_bytes):
    """ltvqkv_lookback_scan_bwd through the C-ABI with a workspace of ws_bytes (fresh, zeroed)."""
    L = _lib.load()
    B, T, _ = comb.shape
    gc = torch.zeros(comb.shape[0], comb.shape[2], comb.shape[1], dtype=comb.dtype,
                     device=comb.device).transpose(1, 2)  # the production (transposed) layout
    gi = torch.empty_like(inits)
    gb = torch.zeros_like(bias)
    ws = torch.zeros(max(ws_bytes, 4096), dtype=torch.uint8, device=comb.device)
    S = _lib.strides
    sc, gs = comb.stride(), gc.stride()
    rc = L.ltvqkv_lookback_scan_bwd(
        _lib.dtype_code(comb.dtype), comb.data_ptr(), sc[0], sc[1], sc[2], inits.data_ptr(), bias.data_ptr(),
        *[x for o in outs for x in (o.data_ptr(), S(o.stride()))],
        *[x for o in grads for x in (o.data_ptr(), S(o.stride()))],
        gc.data_ptr(), gs[0], gs[1], gs[2], gi.data_ptr(), gb.data_ptr(),
        B, T, NH, NKVH, Da, r, P, Q, K, 1, ws.data_ptr(), ws.numel(), _lib.stream_handle(comb.device))
    _lib.check(rc, "ltvqkv_lookback_scan_bwd")
    torch.cuda.synchronize()
    return gc, gi, gb


@pytest.mark.parametrize("B,T,NH,NKVH,Da,r,P,Q,K", [
    (2, 304, 1, 1, 1, 128, 64, 60, 5),        # chunk edges off the 8-token grid
    (2, 512, 2, 1, 1, 128, 128, 112, 17),     # the reference's production chunking
    (1, 256, 1, 1, 2, 64, 32, 16, 17),        # prefix as long as a chunk, two gate groups
    (2, 200, 1, 1, 4, 32, 24, 24, 9),         # four gate groups per head
    (3, 136, 1, 0, 1, 128, 32, 32, 1),        # restarts without a prefix
    (2, 256, 1, 1, 2, 32, 32, 28, 5),         # head dim 64 (the kernel's runtime head-dim form)
    (1, 128, 1, 0, 3, 32, 16, 16, 9),         # head dim 96, three gate groups
])
def test_lookback_chunk_parallel_backward(cuda_device, B, T, NH, NKVH, Da, r, P, Q, K):
    """The chunk-parallel backward (bf16, production layout, T % 8 == 0, taken when the workspace holds
    its slots) against the one-CTA-per-row form (the minimal workspace) and the oracle: grad_combined
    and grad_inits bit for bit, the logit-bias gradient within fp32 reassociation (per-chunk partials)."""
    comb, inits, bias, gq, gk, gv = _random(B * 1000 + T, B, T, NH, NKVH, Da, r)
    comb, inits, gq, gk, gv = (O.round_bf16(a) for a in (comb, inits, gq, gk, gv))
    dev, bf = cuda_device, torch.bfloat16
    tc = torch.from_numpy(comb).to(dev, bf).transpose(1, 2).contiguous().transpose(1, 2)
    ti, tb = torch.from_numpy(inits).to(dev, bf), torch.from_numpy(bias).to(dev)
    grads = [torch.from_numpy(a).to(dev, bf) for a in (gq, gk, gv)]
    outs = getattr(OPS, LB.format("blelloch"))(tc, ti, tb, NH, NKVH, Da, r, P, Q, K, 8, 8, 4, 32, 2, 8, True)
    L = _lib.load()
    small = L.ltvqkv_lookback_workspace_bytes(B, NH, NKVH, Da)
    full = L.ltvqkv_lookback_bwd_workspace_bytes(B, T, NH, NKVH, Da, r, P, Q, K)
    assert full > small  # eligible shape: the query asks for the chunk slots
    seq = _bwd_abi(tc, ti, tb, outs, grads, NH, NKVH, Da, r, P, Q, K, small)
    par = _bwd_abi(tc, ti, tb, outs, grads, NH, NKVH, Da, r, P, Q, K, full)
    assert torch.equal(par[0], seq[0]), "grad_combined"
    assert torch.equal(par[1], seq[1]), "grad_inits"
    assert max_rel_err(_np(par[2]), _np(seq[2]), FLOOR) <= 1e-5, "grad_logit_bias"
    egc, egi, egb = O.scan_bwd(comb, inits, bias, gq, gk, gv, NH, NKVH, Da, r, True, True, (P, Q, K))
    for a, e, n in zip(par, (egc, egi, egb), ("grad_combined", "grad_inits", "grad_logit_bias")):
        if e.size:
            assert max_rel_err(_np(a), e, FLOOR) <= 2e-2, n
