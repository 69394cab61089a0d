"""GPU parity of the attention's q / k prologue folded into the filter's kernels
(`ltv_proj_scan_rope_norm_cuda_op`, `ltv_rotary_qk_norm_ckpt_backward`, `ops.ltv_proj_scan_rope_norm`,
`forward_rotary_norm` of the filter and of the computer module).

The prologue is the reference attention's `apply_rotary_emb` then `norm` on the filter's q and k
(nanochat/gpt.py:96-111, 224-230). On the one-kernel shapes the forward rotates and normalises q and
k in the scan's epilogue (the raw q / k are never stored) and the backward takes their gradients back
through the norm and the rotation from raw outputs replayed out of the scan's checkpoints, chunk by
chunk in parallel, before the checkpoint scan backward. Both must equal this library's own
composition — ltv_proj_scan_cuda_op, then ltv_rotary_qk_norm — bit for bit: outputs, and through
autograd every parameter gradient. That composition's parity is covered elsewhere (the projection +
scan against the oracle in test_gpu_proj_scan.py / test_gpu_configs.py, the prologue against the
reference's torch chain in test_gpu_rotary.py); the fused outputs are also checked against the torch
chain directly here (bf16 elementwise, relative with a floor of 1e-2 of the largest value, 2e-2).
"""

from __future__ import annotations

import pytest
import torch

import nanochat_filter_b200 as nf
from nanochat_filter_b200 import LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter, LtvInitValues
from nanochat_filter_b200.module import LtvCombinedQkvComputerModule
from conftest import max_rel_err
from test_gpu_rotary import rotary_cache, torch_chain

pytestmark = pytest.mark.gpu

OPS = torch.ops.nanochat_cuda
D, R = 128, 128

# B * H >= 2 * 148 rows take the one-kernel path on a 148-SM B200; the last case runs the two
# operators in sequence (too few rows) and must match trivially.
CASES = [
    # B, T, C, NH, NKVH, position offset of the rotary tables
    (32, 1024, 768, 6, 6, 0),     # the d=12 training shape (config 2)
    (17, 544, 200, 6, 6, 37),     # T % 256 != 0, C % 64 != 0, tables sliced at an odd position
    (150, 64, 128, 2, 0, 0),      # Q heads only
    (60, 96, 136, 1, 2, 5),       # K/V-heavy
    (2, 256, 128, 6, 6, 0),       # few rows: two operators in sequence
]


def _inputs(dev, B, T, C, NH, NKVH, off, seed, shared):
    H = NH + 2 * NKVH
    F = H * (D + 1)
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn((B, T, C), generator=g, device=dev).to(torch.bfloat16)
    w = (torch.rand((F, C), generator=g, device=dev) * 2 - 1).mul(C ** -0.5)  # fp32 master weight
    if shared:
        inits = (torch.rand((H, D), generator=g, device=dev) * 2 - 1).mul(0.5)
    else:
        inits = (torch.rand((B, H, D), generator=g, device=dev) * 2 - 1).mul(0.5).to(torch.bfloat16)
    bias = torch.rand((H, 1), generator=g, device=dev) * 2 - 1
    cos, sin = rotary_cache(T + off, D, torch.bfloat16, dev)
    cos, sin = cos[:, off:off + T], sin[:, off:off + T]  # the model's per-position slice: [1, T, 1, D/2] views
    grads = [torch.randn((B, n, T, D), generator=g, device=dev).to(torch.bfloat16) for n in (NH, NKVH, NKVH)]
    return x, w, inits, bias, cos, sin, grads


def _written(ckpt):
    """The checkpoints a forward writes: all but the last chunk's (no chunk follows it)."""
    return ckpt[:, :, :-1] if ckpt.dim() == 4 else ckpt


def _leaves(*ts):
    return [t.detach().clone().requires_grad_(True) for t in ts]


@pytest.mark.parametrize("B,T,C,NH,NKVH,off", CASES)
@pytest.mark.parametrize("shared", [True, False])
def test_fused_prologue_equals_composition(cuda_device, B, T, C, NH, NKVH, off, shared):
    x0, w0, i0, b0, cos, sin, (gq, gk, gv) = _inputs(cuda_device, B, T, C, NH, NKVH, off, B + T + C, shared)

    # fused: projection + scan + rotary + norm in one forward, the prologue's backward in the replay
    x, w, inits, bias = _leaves(x0, w0, i0, b0)
    comb_f, qf, kf, vf, ck_f = OPS.ltv_proj_scan_rope_norm_cuda_op(x, w, inits, bias, cos, sin, NH, NKVH, 1, R, True)
    torch.autograd.backward([qf, kf, vf], [gq, gk, gv])
    fused = [t.detach() for t in (comb_f, qf, kf, vf, _written(ck_f))] + [x.grad, w.grad, bias.grad, inits.grad]

    # composition: the one-call projection + scan, then the standalone prologue on its raw outputs
    x, w, inits, bias = _leaves(x0, w0, i0, b0)
    comb, q, k, v, ck = OPS.ltv_proj_scan_cuda_op(x, w, inits, bias, NH, NKVH, 1, R, True)
    qn, kn = OPS.ltv_rotary_qk_norm(q.transpose(1, 2), k.transpose(1, 2), cos, sin)
    torch.autograd.backward([qn, kn, v], [gq.transpose(1, 2), gk.transpose(1, 2), gv])
    comp = [t.detach() for t in (comb, qn.transpose(1, 2), kn.transpose(1, 2), v, _written(ck))] + \
        [x.grad, w.grad, bias.grad, inits.grad]

    one_kernel = len(nf.ops._ckpt_shape(x0, NH, NKVH, 1, R)) == 4
    assert (ck_f.numel() > 0) == one_kernel
    names = ("combined", "q", "k", "v", "ckpt", "dx", "dW", "dbias", "dinit")
    for n, a, e in zip(names, fused, comp):
        assert a.shape == e.shape and a.dtype == e.dtype, n
        assert torch.equal(a, e), f"{n}: fused differs from the composition (max {(a.float() - e.float()).abs().max()})"

    # the reference's torch chain on the raw filter outputs
    with torch.no_grad():
        for a, raw in ((qf, q), (kf, k)):
            if raw.numel():
                ref = torch_chain(raw.detach().transpose(1, 2), cos, sin).transpose(1, 2)
                assert max_rel_err(a.float().cpu().numpy(), ref.float().cpu().numpy(), 1e-2) <= 2e-2


def _filter(dev, C, NH, NKVH, seed=0):
    torch.manual_seed(seed)
    f = LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter(NH, NKVH, D, R)
    f.c = torch.nn.Linear(C, f.c.out_features, bias=False)
    f.init_weights(alpha_mlp_bias_init=-1.0, weight_s=0.05, bias_s=0.5, init_s=0.5)
    return f.to(dev)


@pytest.mark.parametrize("B,T,C", [(32, 256, 256), (2, 64, 128)])
def test_module_forward_rotary_norm(cuda_device, B, T, C):
    """The computer module's forward_rotary_norm (no KV cache: the fused filter path; with a cache: the
    raw states cached, the prologue as its own operator) equals forward() followed by the fused
    rotary + norm operator, outputs and gradients."""
    dev = cuda_device
    NH, NKVH = 6, 6
    f = _filter(dev, C, NH, NKVH)
    m = LtvCombinedQkvComputerModule(0, f)
    g = torch.Generator(device=dev).manual_seed(3)
    x0 = torch.randn(B, T, C, device=dev, generator=g).to(torch.bfloat16)
    cos, sin = rotary_cache(T, D, torch.bfloat16, dev)
    grads = [torch.randn(B, T, n, D, device=dev, generator=g).to(torch.bfloat16) for n in (NH, NKVH, NKVH)]

    def run(fn):
        f.zero_grad(set_to_none=True)
        x = x0.clone().requires_grad_(True)
        outs = fn(x)
        torch.autograd.backward(list(outs), grads)
        return [t.detach().clone() for t in outs] + [x.grad, f.c.weight.grad, f.logit_bias.grad, f.init_param.grad]

    fused = run(lambda x: m.forward_rotary_norm(x, None, (cos, sin)))

    def composed(x):
        q, k, v = m(x, None)
        q, k = nf.ops.rotary_qk_norm(q, k, cos, sin)
        return q, k, v

    comp = run(composed)
    for n, a, e in zip(("q", "k", "v", "dx", "dW", "dbias", "dinit"), fused, comp):
        assert a.shape == e.shape, n
        assert torch.equal(a, e), f"{n}: max {(a.float() - e.float()).abs().max()}"


def test_filter_forward_rotary_norm_fp32(cuda_device):
    """fp32 activations take the two-operator form inside the operator; the result is still forward()
    followed by the prologue operator, outputs and gradients."""
    dev = cuda_device
    f = _filter(dev, 128, 2, 1)
    x0 = torch.randn(2, 40, 128, device=dev)
    cos, sin = rotary_cache(40, D, torch.float32, dev)
    grads = [torch.randn(2, 40, n, D, device=dev) for n in (2, 1, 1)]

    def run(fn):
        f.zero_grad(set_to_none=True)
        x = x0.clone().requires_grad_(True)
        outs = fn(x)
        torch.autograd.backward(list(outs), grads)
        return [t.detach().clone() for t in outs] + [x.grad, f.c.weight.grad, f.logit_bias.grad, f.init_param.grad]

    def composed(x):
        q, k, v = f(x, LtvInitValues())
        q, k = nf.ops.rotary_qk_norm(q, k, cos, sin)
        return q, k, v

    a = run(lambda x: f.forward_rotary_norm(x, LtvInitValues(), (cos, sin)))
    e = run(composed)
    for n, u, w in zip(("q", "k", "v", "dx", "dW", "dbias", "dinit"), a, e):
        assert torch.equal(u, w), n
