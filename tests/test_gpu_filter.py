"""Drop-in behaviour of the filter module, the QKV computer module and the decode step on GPU.

The module composes projection + scan exactly as the reference's
LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter does; it is compared with the
oracle's composition of the reference algorithm (oracle.layer_fwd_bwd). Decode follows the
reference's integration tests (tests/test_gpt_ltv_integration.py:215: token-by-token decode
with the KV cache equals the batch forward).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import max_rel_err, max_rel_err_rms
from nanochat_filter_b200 import (
    KVCache,
    LtvCombinedQkvComputerModule,
    LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter,
    LtvInitValues,
)
from oracle import oracle as O

pytestmark = pytest.mark.gpu

FLOOR = 1e-2


def make_filter(dev, dtype, NH=2, NKVH=1, D=128, r=128, seed=0):
    torch.manual_seed(seed)
    f = LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter(NH, NKVH, D, r)
    f.init_weights(alpha_mlp_bias_init=-1.0, weight_s=0.05, bias_s=0.5, init_s=0.5)
    return f.to(dev, dtype if dtype == torch.float32 else torch.float32)


def _np(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_filter_forward_backward_vs_oracle(cuda_device, dtype):
    dev = cuda_device
    NH, NKVH, D, r, B, T = 2, 1, 128, 64, 2, 96
    f = make_filter(dev, dtype, NH, NKVH, D, r)
    if dtype == torch.bfloat16:
        f = f.to(torch.bfloat16)
        f.logit_bias.data = f.logit_bias.data.float()
    C = NH * D
    gen = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn(B, T, C, device=dev, generator=gen).to(dtype).requires_grad_(True)
    q, k, v = f(x, LtvInitValues())
    assert q.shape == (B, T, NH, D) and k.shape == (B, T, NKVH, D) and v.shape == (B, T, NKVH, D)
    assert q.transpose(1, 2).is_contiguous()  # [B, T, H, D] views of head-major storage
    gq = torch.randn(q.shape, device=dev, generator=gen).to(dtype)
    gk = torch.randn(k.shape, device=dev, generator=gen).to(dtype)
    gv = torch.randn(v.shape, device=dev, generator=gen).to(dtype)
    torch.autograd.backward([q, k, v], [gq, gk, gv])

    bf16 = dtype == torch.bfloat16
    H = NH + 2 * NKVH
    inits = f.init_param.detach().float().cpu().numpy()[None].repeat(B, 0)
    if bf16:
        inits = O.round_bf16(inits)
    ref = O.layer_fwd_bwd(_np(x), _np(f.c.weight), inits, _np(f.logit_bias),
                          _np(gq.transpose(1, 2)), _np(gk.transpose(1, 2)), _np(gv.transpose(1, 2)),
                          NH, NKVH, D // r, r, bf16=bf16)
    # fp32: elementwise relative error (floor 1% of the tensor's max) <= 1e-5.
    # bf16: elementwise relative error with the floor at the tensor's RMS <= 2e-2: the layer rounds
    # three times in sequence (projection buffer, scan output, gradient buffer) and a one-ulp flip at
    # any of them (fp32 vs float64 accumulation) moves its dependents by a fraction of that ulp, which
    # is not small next to entries far below the data's scale (test_gpu_configs.py measures it).
    tol = 2e-2 if bf16 else 1e-5

    def err(a, e):
        return max_rel_err_rms(a, e) if bf16 else max_rel_err(a, e, FLOOR)

    errs = {
        "q": err(_np(q.transpose(1, 2)), ref["hq"]),
        "k": err(_np(k.transpose(1, 2)), ref["hk"]),
        "v": err(_np(v.transpose(1, 2)), ref["hv"]),
        "dx": err(_np(x.grad), ref["grad_x"]),
        "dW": err(_np(f.c.weight.grad), ref["grad_w"]),
        "dbias": err(_np(f.logit_bias.grad), ref["grad_logit_bias"]),
        "dinit": err(_np(f.init_param.grad), ref["grad_inits"].sum(0)),
    }
    bad = {k2: e for k2, e in errs.items() if e > tol}
    assert not bad, f"above {tol}: {bad} (all {errs})"


def test_state_dict_layout_matches_reference_names(cuda_device):
    f = make_filter(cuda_device, torch.float32)
    sd = f.state_dict()
    assert set(sd) == {"c.weight", "init_param", "logit_bias"}
    assert sd["c.weight"].shape == (4 * 129, 256)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_decode_token_by_token_equals_batch_forward(cuda_device, dtype):
    """Prefill + one-token decode steps through the module and KV cache reproduce the batch
    forward over the whole sequence (the decode step uses the one-launch kernel)."""
    dev = cuda_device
    NH, NKVH, D, r, B, T, prompt = 2, 2, 128, 128, 3, 12, 5
    f = make_filter(dev, dtype, NH, NKVH, D, r, seed=4).to(dtype)
    f.logit_bias.data = f.logit_bias.data.float()
    mod = LtvCombinedQkvComputerModule(0, f)
    C = NH * D
    x = torch.randn(B, T, C, device=dev).to(dtype)
    with torch.no_grad():
        qf, kf, vf = mod(x, None)
        cache = KVCache(B, NH, NKVH, T, D, num_layers=1)
        qs, ks, vs = [], [], []
        q0, k0, v0 = mod(x[:, :prompt].contiguous(), cache)
        qs.append(q0); ks.append(k0); vs.append(v0)
        for t in range(prompt, T):
            q1, k1, v1 = mod(x[:, t:t + 1].contiguous(), cache)
            qs.append(q1); ks.append(k1); vs.append(v1)
    qd, kd, vd = torch.cat(qs, 1), torch.cat(ks, 1), torch.cat(vs, 1)
    # fp32: the same arithmetic (elementwise, floor 1% of max). bf16: the cache holds the rounded
    # state (as the reference's does) while the batch scan carries fp32, so each decode step
    # restarts from a value one rounding away; compared norm-wise.
    tol, floor = (1e-5, FLOOR) if dtype == torch.float32 else (3e-2, 1.0)
    for a, e in ((qd, qf), (kd, kf), (vd, vf)):
        assert max_rel_err(_np(a), _np(e), floor) <= tol
    # the cache holds the last step
    torch.testing.assert_close(cache.last_qkv.q.special[0], qd[:, -1], rtol=0, atol=0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("with_state", [False, True])
def test_decode_kernel_vs_oracle(cuda_device, dtype, with_state):
    """One decode step against the oracle's T == 1 projection + scan (reference semantics:
    projection rounded to the storage dtype, fp32 gate and update, rounded state)."""
    dev = cuda_device
    NH, NKVH, Da, r, B, C = 6, 6, 1, 128, 64, 768
    H, D = NH + 2 * NKVH, Da * r
    F = H * (D + Da)
    rng = np.random.default_rng(7)
    bf16 = dtype == torch.bfloat16
    rd = O.round_bf16 if bf16 else (lambda a: a)
    x = rd(rng.standard_normal((B, 1, C)).astype(np.float32))
    w = rd((rng.standard_normal((F, C)) / np.sqrt(C)).astype(np.float32))
    bias = rng.standard_normal((H, Da)).astype(np.float32)
    init = rd((0.5 * rng.standard_normal((H, D))).astype(np.float32))
    prev = rd(rng.standard_normal((B, H, D)).astype(np.float32))
    start = prev if with_state else np.repeat(init[None], B, 0)
    comb = O.gemm_fwd(x, w, bf16)                                  # [B, F, 1]
    eq, ek, ev = O.scan_fwd(comb.transpose(0, 2, 1), start, bias, NH, NKVH, Da, r, True, bf16)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev, dtype)
    pq = pk = pv = None
    if with_state:
        tp = T(prev)
        pq, pk, pv = tp[:, :NH], tp[:, NH:NH + NKVH], tp[:, NH + NKVH:]
    q, k, v = torch.ops.nanochat_cuda.ltv_decode_step(T(x), T(w), torch.from_numpy(bias).to(dev), pq, pk, pv,
                                                      T(init), NH, NKVH, Da, r, True)
    # fp32: elementwise, floor 1% of max|e|. bf16: elementwise with the floor at the tensor's RMS (a
    # projection value that rounds to the neighbouring bf16 value under a different fp32 summation
    # order moves its output by alpha * ulp(u), not small next to near-zero states)
    tol = 2e-2 if bf16 else 1e-5
    for a, e in ((q, eq[:, :, 0]), (k, ek[:, :, 0]), (v, ev[:, :, 0])):
        assert (max_rel_err_rms(_np(a), e) if bf16 else max_rel_err(_np(a), e, FLOOR)) <= tol


@pytest.mark.parametrize("B,C", [(64, 768), (70, 256), (3, 200)])
def test_decode_step_inplace_equals_out_of_place(cuda_device, B, C):
    """ltv_decode_step_ (states updated in place, as a cache update) equals ltv_decode_step."""
    NH, NKVH, Da, r = 2, 1, 1, 128
    H, D = NH + 2 * NKVH, Da * r
    g = torch.Generator(device=cuda_device).manual_seed(B + C)
    x = torch.randn(B, C, generator=g, device=cuda_device).to(torch.bfloat16)
    w = (torch.randn(H * (D + Da), C, generator=g, device=cuda_device) * C ** -0.5).to(torch.bfloat16)
    bias = torch.randn(H, Da, generator=g, device=cuda_device)
    init = torch.zeros(H, D, device=cuda_device, dtype=torch.bfloat16)
    st = [torch.randn(B, n, D, generator=g, device=cuda_device).to(torch.bfloat16) for n in (NH, NKVH, NKVH)]
    ref = torch.ops.nanochat_cuda.ltv_decode_step(x, w, bias, *st, init, NH, NKVH, Da, r, True)
    torch.ops.nanochat_cuda.ltv_decode_step_(x, w, bias, *st, NH, NKVH, Da, r, True)
    for a, b in zip(st, ref):
        assert torch.equal(a, b)
