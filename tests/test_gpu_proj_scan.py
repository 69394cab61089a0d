"""GPU parity of the one-call projection + scan forward (`ltv_proj_scan_cuda_op`).

The op must equal the reference filter's two-op composition
(nanochat/ltv_cuda_fused_concat_head_major_register_cast_blelloch_scan_qkv_filter.py:24-73:
fused_linear_transpose, then the scan op on combined^T) bit for bit — both the projection
`combined` it writes and q/k/v — so the comparison here is exact equality with this library's
own two operators, whose parity with the reference is covered by the GEMM and scan tests; the
oracle check below anchors the fused path to the CPU restatement directly as well. Shapes cover
the fused case (bf16, D = 128, Da = 1, T % 32 == 0) with T not a multiple of the 256-token tile,
C not a multiple of the 64-wide k block, heads without K/V, and the sequential fallback cases
(fp32, T % 32 != 0, Da > 1).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import nanochat_filter_b200  # noqa: F401
from nanochat_filter_b200.filters import LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter
from nanochat_filter_b200.util import LtvInitValues
from conftest import max_rel_err
from oracle import oracle as O

pytestmark = pytest.mark.gpu

OPS = torch.ops.nanochat_cuda


def _inputs(dev, B, T, C, NH, NKVH, Da, r, dtype, seed):
    H = NH + 2 * NKVH
    D = Da * r
    F = H * (D + Da)
    g = torch.Generator(device=dev).manual_seed(seed)
    x = (torch.randn((B, T, C), generator=g, device=dev) * 0.5).to(dtype)
    w = (torch.rand((F, C), generator=g, device=dev) * 2 - 1).mul(C ** -0.5).to(dtype)
    inits = (torch.rand((B, H, D), generator=g, device=dev) * 2 - 1).mul(0.5).to(dtype)
    bias = torch.rand((H, Da), generator=g, device=dev) * 2 - 1
    return x, w, inits, bias


def _two_ops(x, w, inits, bias, NH, NKVH, Da, r, use_sigmoid):
    comb = OPS.fused_linear_transpose_cuda_op(x, w)
    q, k, v = OPS.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_op(
        comb.transpose(1, 2), inits, bias, NH, NKVH, Da, r, 8, 8, 4, 32, 2, 8, use_sigmoid)
    return comb, q, k, v


# The fused kernel runs when B * H >= 2 * SMs (296 (batch, head) rows on a 148-SM B200), the
# shapes for which the scan operator takes its row-streaming kernel; other cases run the two
# entry points in sequence and must equal them trivially.
CASES = [
    # B, T, C, NH, NKVH, Da, r
    (32, 1024, 768, 6, 6, 1, 128),    # the d=12 training shape (config 2)
    (17, 544, 200, 6, 6, 1, 128),     # T % 256 != 0, C % 64 != 0
    (150, 32, 64, 2, 0, 1, 128),      # one token tile, Q heads only
    (60, 96, 136, 1, 2, 1, 128),      # K/V-heavy
    (2, 2048, 768, 6, 6, 1, 128),     # few rows: sequential
    (20, 1000, 256, 6, 6, 1, 128),    # T % 32 != 0: sequential
    (40, 256, 128, 6, 6, 2, 64),      # Da > 1: sequential
]


@pytest.mark.parametrize("B,T,C,NH,NKVH,Da,r", CASES)
@pytest.mark.parametrize("use_sigmoid", [True, False])
def test_proj_scan_equals_two_ops(cuda_device, B, T, C, NH, NKVH, Da, r, use_sigmoid):
    x, w, inits, bias = _inputs(cuda_device, B, T, C, NH, NKVH, Da, r, torch.bfloat16, B * 131 + T + C)
    if not use_sigmoid:
        bias = bias * 0.05 + 0.3  # raw alphas in (0.25, 0.35) keep the recurrence bounded
        w = w * 0.05
    ref = _two_ops(x, w, inits, bias, NH, NKVH, Da, r, use_sigmoid)
    got = OPS.ltv_proj_scan_cuda_op(x, w, inits, bias, NH, NKVH, Da, r, use_sigmoid)
    torch.cuda.synchronize()
    for a, b, n in zip(got, ref, ("combined", "q", "k", "v")):
        assert a.shape == b.shape, n
        assert torch.equal(a, b), f"{n}: {(a.float() - b.float()).abs().max().item()}"
    ckpt = got[4]
    if ckpt.numel():
        # entry j is the fp32 state after token 32 j + 31, whose bf16 rounding is that token's output
        H = NH + 2 * NKVH
        assert tuple(ckpt.shape) == (B, H, T // 32, 128)
        outs = torch.cat([o for o, n in zip(got[1:4], (NH, NKVH, NKVH)) if n], dim=1)
        last = outs[:, :, 31::32][:, :, :-1]
        assert torch.equal(ckpt[:, :, :-1].to(torch.bfloat16), last)


def test_proj_scan_fp32_fallback(cuda_device):
    x, w, inits, bias = _inputs(cuda_device, 2, 256, 128, 2, 1, 1, 128, torch.float32, 7)
    ref = _two_ops(x, w, inits, bias, 2, 1, 1, 128, True)
    got = OPS.ltv_proj_scan_cuda_op(x, w, inits, bias, 2, 1, 1, 128, True)
    for a, b in zip(got, ref):
        assert torch.equal(a, b)


def test_proj_scan_against_oracle(cuda_device):
    """The fused path against the CPU restatement of the scan on the kernel's own `combined`."""
    B, T, C, NH, NKVH, Da, r = 300, 64, 192, 1, 0, 1, 128   # 300 rows: the fused kernel
    x, w, inits, bias = _inputs(cuda_device, B, T, C, NH, NKVH, Da, r, torch.bfloat16, 99)
    comb, q, k, v, _ = OPS.ltv_proj_scan_cuda_op(x, w, inits, bias, NH, NKVH, Da, r, True)
    # projection: fp32 contraction of the same bf16 values, rounded once
    ref_comb = torch.matmul(w.float(), x.float().transpose(1, 2))
    np.testing.assert_allclose(comb.float().cpu().numpy(), ref_comb.cpu().numpy(), rtol=1e-2, atol=1e-2)
    # scan: the oracle fed the kernel's bf16 projection (bf16 state rounding, same bound as the
    # scan operator's own oracle test)
    f32 = lambda t: t.float().contiguous().cpu().numpy()  # noqa: E731
    oq, ok, ov = O.scan_fwd(f32(comb.transpose(1, 2)), f32(inits), f32(bias), NH, NKVH, Da, r, True, True)
    for got, want, n in ((q, oq, "q"), (k, ok, "k"), (v, ov, "v")):
        err = max_rel_err(f32(got), want, 1e-2)
        assert err <= 2e-2, f"{n}: {err}"


def test_proj_scan_autograd_equals_two_ops(cuda_device):
    B, T, C, NH, NKVH, Da, r = 100, 288, 192, 2, 1, 1, 128
    x, w, inits, bias = _inputs(cuda_device, B, T, C, NH, NKVH, Da, r, torch.bfloat16, 5)
    wf = w.float()
    gen = torch.Generator(device=cuda_device).manual_seed(3)
    grads = [torch.randn((B, n, T, 128), generator=gen, device=cuda_device).to(torch.bfloat16)
             for n in (NH, NKVH, NKVH)]

    def run(fused):
        xx = x.clone().requires_grad_(True)
        ww = wf.clone().requires_grad_(True)
        ii = inits.clone().requires_grad_(True)
        bb = bias.clone().requires_grad_(True)
        if fused:
            _, q, k, v, _ = OPS.ltv_proj_scan_cuda_op(xx, ww, ii, bb, NH, NKVH, Da, r, True)
        else:
            comb = OPS.fused_linear_transpose_cuda_op(xx, ww)  # fp32 master weight, as the filter passes it
            q, k, v = OPS.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_op(
                comb.transpose(1, 2), ii, bb, NH, NKVH, Da, r, 8, 8, 4, 32, 2, 8, True)
        torch.autograd.backward((q, k, v), grads)
        return (q, k, v, xx.grad, ww.grad, ii.grad, bb.grad)

    got, ref = run(True), run(False)
    names = ("q", "k", "v", "grad_x", "grad_w", "grad_inits", "grad_bias")
    for a, b, n in zip(got, ref, names):
        assert a.dtype == b.dtype and torch.equal(a, b), n


def test_filter_module_fused_forward(cuda_device):
    """The module's bf16 forward (one-call path) equals its fp32-free two-op composition."""
    torch.manual_seed(0)
    f = LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter(6, 6, 128, 128).to(cuda_device)
    f.init_weights(2.0, 0.05, 0.5, 0.5)
    B = 17
    x = (torch.randn(B, 320, 768, device=cuda_device) * 0.5).to(torch.bfloat16)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        q, k, v = f(x, LtvInitValues())
    inits = f.init_param.to(torch.bfloat16).unsqueeze(0).expand(B, -1, -1).contiguous()
    _, rq, rk, rv = _two_ops(x, f.c.weight.to(torch.bfloat16), inits, f.logit_bias.detach(), 6, 6, 1, 128, True)
    for a, b in ((q, rq), (k, rk), (v, rv)):
        assert torch.equal(a, b.transpose(1, 2))


@pytest.mark.parametrize("B,T,C,NH,NKVH,layout", [
    (32, 1024, 768, 6, 6, "contiguous"),   # config 2
    (100, 288, 192, 2, 1, "transposed"),   # upstream grads as [B, T, heads, D] storage
    (300, 64, 128, 1, 0, "contiguous"),    # Q-only, two chunks per row
])
def test_scan_ckpt_backward_equals_backward_kernel(cuda_device, B, T, C, NH, NKVH, layout):
    """The scan backward from the forward's state checkpoints equals the backward kernel that reads
    the forward's outputs, bit for bit (grad_combined, grad_inits, grad_logit_bias)."""
    x, w, inits, bias = _inputs(cuda_device, B, T, C, NH, NKVH, 1, 128, torch.bfloat16, B + T)
    comb, q, k, v, ckpt = OPS.ltv_proj_scan_cuda_op(x, w, inits, bias, NH, NKVH, 1, 128, True)
    assert ckpt.numel() > 0
    gen = torch.Generator(device=cuda_device).manual_seed(B)

    def grad(n):
        g = torch.randn((B, n, T, 128), generator=gen, device=cuda_device).to(torch.bfloat16)
        return g.transpose(1, 2).contiguous().transpose(1, 2) if layout == "transposed" else g

    gq, gk, gv = grad(NH), grad(NKVH), grad(NKVH)
    combined = comb.transpose(1, 2)
    res = []
    for use_ckpt in (True, False):
        gc = torch.full_like(combined, float("nan"))
        gi = torch.full_like(inits, float("nan"))
        gb = torch.zeros_like(bias)
        if use_ckpt:
            OPS.ltv_scan_ckpt_backward_kernel(combined, inits, bias, ckpt, gq, gk, gv, gc, gi, gb, NH, NKVH, 1, 128,
                                              True)
        else:
            OPS.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_backward_kernel(
                combined, inits, bias, q, k, v, gq, gk, gv, gc, gi, gb, NH, NKVH, 1, 128, 32, 2, 8, True)
        res.append((gc, gi, gb))
    torch.cuda.synchronize()
    for a, b, n in zip(res[0], res[1], ("grad_combined", "grad_inits", "grad_logit_bias")):
        assert torch.equal(a, b), n


def test_scan_ckpt_backward_unsupported_shape(cuda_device):
    """Shapes the row-streaming kernel does not take raise instead of running something else."""
    B, T, NH, NKVH = 2, 64, 1, 0   # 2 rows
    combined = torch.randn(B, T, 129, device=cuda_device).to(torch.bfloat16)
    inits = torch.zeros(B, 1, 128, device=cuda_device, dtype=torch.bfloat16)
    bias = torch.zeros(1, 1, device=cuda_device)
    ckpt = torch.zeros(B, 1, 2, 128, device=cuda_device)
    g = torch.zeros(B, 1, T, 128, device=cuda_device, dtype=torch.bfloat16)
    e = torch.zeros(B, 0, T, 128, device=cuda_device, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="not implement|unsupported|Unsupported"):
        OPS.ltv_scan_ckpt_backward_kernel(combined, inits, bias, ckpt, g, e, e, torch.empty_like(combined),
                                          torch.empty_like(inits), torch.zeros_like(bias), NH, NKVH, 1, 128, True)


@pytest.mark.parametrize("B,T,C,NH,NKVH", [(32, 1024, 768, 6, 6), (300, 64, 128, 1, 0)])
def test_shared_initial_state(cuda_device, B, T, C, NH, NKVH):
    """One initial state [H, D] for every sequence (the training case): outputs equal those of the
    same state expanded over the batch bit for bit; the checkpoint backward's grad_combined and
    grad_logit_bias equal the per-sequence form's bit for bit, and its [H, D] float32 initial-state
    gradient is the per-sequence bf16 gradients summed over the batch (fp32; summation order only)."""
    H = NH + 2 * NKVH
    x, w, _, bias = _inputs(cuda_device, B, T, C, NH, NKVH, 1, 128, torch.bfloat16, B * 7 + T)
    gen = torch.Generator(device=cuda_device).manual_seed(11)
    init = ((torch.rand((H, 128), generator=gen, device=cuda_device) * 2 - 1) * 0.5).to(torch.bfloat16)
    expanded = init.unsqueeze(0).expand(B, -1, -1).contiguous()
    shared = OPS.ltv_proj_scan_cuda_op(x, w, init, bias, NH, NKVH, 1, 128, True)
    per_seq = OPS.ltv_proj_scan_cuda_op(x, w, expanded, bias, NH, NKVH, 1, 128, True)
    assert shared[4].numel() > 0
    for a, b, n in zip(shared, per_seq, ("combined", "q", "k", "v")):
        assert torch.equal(a, b), n
    assert torch.equal(shared[4][:, :, :-1], per_seq[4][:, :, :-1])  # the last entry is not written
    comb, q, k, v, ckpt = shared
    combined = comb.transpose(1, 2)
    grads = [torch.randn((B, n, T, 128), generator=gen, device=cuda_device).to(torch.bfloat16)
             for n in (NH, NKVH, NKVH)]
    gc1, gi1 = torch.empty_like(combined), torch.full((H, 128), float("nan"), device=cuda_device)
    gb1 = torch.full_like(bias, float("nan"))  # overwritten, not added to
    OPS.ltv_scan_ckpt_backward_kernel(combined, init, bias, ckpt, *grads, gc1, gi1, gb1, NH, NKVH, 1, 128, True)
    gc2, gi2, gb2 = torch.empty_like(combined), torch.empty_like(expanded), torch.zeros_like(bias)
    OPS.ltv_scan_ckpt_backward_kernel(combined, expanded, bias, ckpt, *grads, gc2, gi2, gb2, NH, NKVH, 1, 128, True)
    torch.cuda.synchronize()
    assert torch.equal(gc1, gc2) and torch.equal(gb1, gb2)
    want = gi2.float().sum(0)
    torch.testing.assert_close(gi1, want, rtol=1e-5, atol=1e-5 * want.abs().max().item())


def test_shared_initial_state_autograd(cuda_device):
    """ltv_proj_scan_cuda_op with the fp32 [H, D] parameter as the initial state: gradients equal the
    expanded-state composition's bit for bit, except the [H, D] one, which the composition's expand
    backward sums as a bf16 tensor (one bf16 rounding of the batch sum, <= 2^-9 relative) while the
    shared form keeps the fp32 sum."""
    B, T, C, NH, NKVH = 100, 288, 192, 2, 1
    H = NH + 2 * NKVH
    x, w, _, bias = _inputs(cuda_device, B, T, C, NH, NKVH, 1, 128, torch.bfloat16, 21)
    gen = torch.Generator(device=cuda_device).manual_seed(4)
    init = (torch.rand((H, 128), generator=gen, device=cuda_device) * 2 - 1) * 0.5
    grads = [torch.randn((B, n, T, 128), generator=gen, device=cuda_device).to(torch.bfloat16)
             for n in (NH, NKVH, NKVH)]

    def run(shared):
        xx = x.clone().requires_grad_(True)
        ww = w.float().clone().requires_grad_(True)
        ii = init.clone().requires_grad_(True)
        bb = bias.clone().requires_grad_(True)
        inits = ii if shared else ii.to(torch.bfloat16).unsqueeze(0).expand(B, -1, -1)
        _, q, k, v, ckpt = OPS.ltv_proj_scan_cuda_op(xx, ww, inits, bb, NH, NKVH, 1, 128, True)
        assert ckpt.numel() > 0
        torch.autograd.backward((q, k, v), grads)
        return (q, k, v, xx.grad, ww.grad, bb.grad), ii.grad

    (got, gi_got), (ref, gi_ref) = run(True), run(False)
    for a, b, n in zip(got, ref, ("q", "k", "v", "grad_x", "grad_w", "grad_bias")):
        assert a.dtype == b.dtype and torch.equal(a, b), n
    assert gi_got.dtype == torch.float32
    torch.testing.assert_close(gi_got, gi_ref, rtol=2 ** -8, atol=1e-5 * gi_ref.abs().max().item())


@pytest.mark.parametrize("C,offset", [(124, 0), (128, 0), (128, 8)])
def test_proj_scan_fake_and_real_checkpoint_shapes_agree(cuda_device, C, offset):
    """The fake kernel's checkpoint shape equals the real op's: C % 8 != 0 (no one-kernel form, empty
    checkpoint), and x at an 8-element (16-byte) offset and at a 2-element (4-byte) one (the op
    realigns it, so the checkpoints the fake promises are written)."""
    B, T, NH, NKVH = 32, 64, 6, 6
    H, F = NH + 2 * NKVH, (NH + 2 * NKVH) * 129
    gen = torch.Generator(device=cuda_device).manual_seed(C + offset)
    for off in (offset, 2):
        buf = torch.randn(B * T * C + off, generator=gen, device=cuda_device).to(torch.bfloat16)
        x = buf[off:].view(B, T, C)
        w = (torch.randn(F, C, generator=gen, device=cuda_device) / C ** 0.5).to(torch.bfloat16)
        init = torch.zeros(H, 128, device=cuda_device)
        bias = torch.zeros(H, 1, device=cuda_device)
        real = OPS.ltv_proj_scan_cuda_op(x, w, init, bias, NH, NKVH, 1, 128, True)
        with torch.device("meta"):
            fake = OPS.ltv_proj_scan_cuda_op(torch.empty(B, T, C, dtype=torch.bfloat16),
                                             torch.empty(F, C, dtype=torch.bfloat16), torch.empty(H, 128),
                                             torch.empty(H, 1), NH, NKVH, 1, 128, True)
        for a, b in zip(real, fake):
            assert tuple(a.shape) == tuple(b.shape) and a.dtype == b.dtype
        assert (real[4].numel() > 0) == (C % 8 == 0)
