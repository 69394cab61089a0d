"""GPU parity of the fused rotary + QK RMS-norm prologue (`ltv_rotary_qk_norm`) against the
reference attention's torch chain (nanochat/gpt.py:96-111, 224-230: apply_rotary_emb, then norm =
F.rms_norm over the head dim), forward and autograd backward. q/k come as the filter returns them
([B, T, heads, D] views of head-major storage) or contiguous; outputs are head-major so that the
attention's transpose(1, 2) is contiguous. The forward is checked against the torch chain in the
storage dtype (elementwise, relative with a floor of 1e-2 of the largest value: 2e-2 bf16, 1e-5
fp32); values and gradients against the plain fp32 reference of the same op (bf16 inputs upcast):
fp32 elementwise 1e-5 forward, 1e-4 backward (reduction order); bf16 norm-wise, max |a - e| <=
2e-2 max |e| (the rotation's bf16 roundings, which the torch chain makes too, cancel in sums near
zero).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import nanochat_filter_b200 as nf  # noqa: F401
from conftest import max_rel_err

pytestmark = pytest.mark.gpu


def torch_chain(x, cos, sin):
    d = x.shape[3] // 2
    if x.shape[3] % 2 == 0:
        x1, x2 = x[..., :d], x[..., d:]
        x = torch.cat([x1 * cos + x2 * sin, x1 * (-sin) + x2 * cos], 3)
    return F.rms_norm(x, (x.size(-1),))


def rotary_cache(T, D, dtype, dev):
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, dtype=torch.float32, device=dev) / D))
    f = torch.outer(torch.arange(T, dtype=torch.float32, device=dev), inv)
    return f.cos().to(dtype)[None, :, None, :], f.sin().to(dtype)[None, :, None, :]


def _np(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,T,NH,NKVH,D,head_major", [(2, 64, 6, 6, 128, True), (3, 33, 2, 1, 64, False),
                                                       (1, 17, 1, 2, 256, True), (2, 9, 2, 2, 63, False)])
def test_rotary_qk_norm_matches_torch_chain(cuda_device, dtype, B, T, NH, NKVH, D, head_major):
    g = torch.Generator(device=cuda_device).manual_seed(B * 31 + T + D)

    def mk(n):
        if head_major:  # the filter's output: [B, T, heads, D] view of [B, heads, T, D] storage
            return torch.randn(B, n, T, D, generator=g, device=cuda_device).to(dtype).transpose(1, 2)
        return torch.randn(B, T, n, D, generator=g, device=cuda_device).to(dtype)

    q, k = mk(NH), mk(NKVH)
    cos, sin = rotary_cache(T, D - D % 2 if D % 2 == 0 else D + 1, dtype, cuda_device)
    gq = torch.randn(B, T, NH, D, generator=g, device=cuda_device).to(dtype)
    gk = torch.randn(B, T, NKVH, D, generator=g, device=cuda_device).to(dtype)
    qa, ka = q.detach().requires_grad_(True), k.detach().requires_grad_(True)
    oq, ok = nf.ops.rotary_qk_norm(qa, ka, cos, sin)
    torch.autograd.backward([oq, ok], [gq, gk])
    bf16 = dtype == torch.bfloat16
    # the reference chain in the storage dtype (the forward matches it to one storage ulp) ...
    with torch.no_grad():
        sq, sk = torch_chain(q, cos, sin), torch_chain(k, cos, sin)
    # ... and the plain fp32 reference of the same op for values and gradients
    qr, kr = q.detach().float().requires_grad_(True), k.detach().float().requires_grad_(True)
    rq, rk = torch_chain(qr, cos.float(), sin.float()), torch_chain(kr, cos.float(), sin.float())
    torch.autograd.backward([rq, rk], [gq.float(), gk.float()])
    checks = [(oq, sq, "q vs chain", 2e-2 if bf16 else 1e-5), (ok, sk, "k vs chain", 2e-2 if bf16 else 1e-5),
              (oq, rq, "q", 2e-2 if bf16 else 1e-5), (ok, rk, "k", 2e-2 if bf16 else 1e-5),
              (qa.grad, qr.grad, "dq", 2e-2 if bf16 else 1e-4), (ka.grad, kr.grad, "dk", 2e-2 if bf16 else 1e-4)]
    for a, e, n, tol in checks:
        assert a.shape == e.shape, n
        if bf16 and "chain" not in n:
            # against fp32: the rotation's bf16 roundings cancel in sums near zero, so norm-wise
            d, ref = _np(a), _np(e)
            assert np.abs(d - ref).max() <= tol * np.abs(ref).max(), n
        else:
            assert max_rel_err(_np(a), _np(e), 1e-2) <= tol, n
    assert oq.transpose(1, 2).is_contiguous() and ok.transpose(1, 2).is_contiguous()
