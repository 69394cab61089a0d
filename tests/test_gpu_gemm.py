"""GPU parity of the projection operator (fused linear transpose) and its backward.

Ports the reference's GEMM test (tests/test_fused_linear_transpose.py:32-86): shapes
(1,16,32,128), (4,128,128,256), (4,1024,1024,3096), (2,31,63,127); tolerance 1e-4 (fp32) and
5e-2 (bf16) for out, grad_x and grad_weight. The small shapes compare with the reference's golden
vectors; the large ones (incl. the d=12 training shape of config 2) with an fp32 contraction of the
same bf16 values. Both grad_out layouts the reference accepts are exercised, and fp32 master
weights with bf16 activations (grad_weight in fp32).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import nanochat_filter_b200  # noqa: F401
from conftest import load_golden, max_rel_err

pytestmark = pytest.mark.gpu

FLT = torch.ops.nanochat_cuda.fused_linear_transpose_cuda_op
BWD = torch.ops.nanochat_cuda.fused_linear_transpose_backward_kernel
GEMM = load_golden("gemm.npz")


@pytest.fixture(autouse=True)
def _no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


@pytest.mark.parametrize("key", sorted(GEMM))
def test_gemm_golden(cuda_device, key):
    c = GEMM[key]
    dtype = torch.bfloat16 if key.startswith("bf16") else torch.float32
    x = torch.from_numpy(c["x"]).to(cuda_device, dtype).requires_grad_(True)
    w = torch.from_numpy(c["w"]).to(cuda_device, dtype).requires_grad_(True)
    g = torch.from_numpy(c["g"]).to(cuda_device, dtype)
    out = FLT(x, w)
    out.backward(g)
    tol = 5e-2 if dtype == torch.bfloat16 else 1e-4
    for a, n in ((out, "out"), (x.grad, "grad_x"), (w.grad, "grad_w")):
        np.testing.assert_allclose(a.detach().float().cpu().numpy(), c[n], rtol=tol, atol=tol, err_msg=n)


def _reference(x, w, g):
    xf, wf, gf = x.detach().float(), w.detach().float(), g.detach().float()
    out = torch.matmul(wf, xf.transpose(1, 2))                 # [B, F, T]
    gx = torch.matmul(gf.transpose(1, 2), wf)                  # [B, T, K]
    gw = torch.einsum("bft,btk->fk", gf, xf)                   # [F, K]
    return out, gx, gw


@pytest.mark.parametrize("B,T,K,F", [(4, 1024, 1024, 3096), (32, 1024, 768, 2322), (3, 200, 64, 72)])
@pytest.mark.parametrize("grad_layout", ["contiguous", "transposed"])
def test_gemm_large_bf16(cuda_device, B, T, K, F, grad_layout):
    gen = torch.Generator(device=cuda_device).manual_seed(B * 7 + T)
    x = (torch.randn(B, T, K, device=cuda_device, generator=gen) / K**0.5).to(torch.bfloat16)
    w = (torch.randn(F, K, device=cuda_device, generator=gen) / K**0.5).to(torch.bfloat16)
    g = torch.randn(B, F, T, device=cuda_device, generator=gen).to(torch.bfloat16)
    if grad_layout == "transposed":
        g = g.transpose(1, 2).contiguous().transpose(1, 2)    # strides (F*T, 1, F)
    out = FLT(x, w)
    gx = torch.empty_like(x)
    gw = torch.empty_like(w)
    BWD(x, w, g, gx, gw)
    eo, egx, egw = _reference(x, w, g)
    # bf16 outputs: rounding of the result (2^-8 relative) plus fp32 summation order.
    assert max_rel_err(out.float().cpu().numpy(), eo.cpu().numpy()) <= 2e-2
    assert max_rel_err(gx.float().cpu().numpy(), egx.cpu().numpy()) <= 2e-2
    assert max_rel_err(gw.float().cpu().numpy(), egw.cpu().numpy()) <= 2e-2


def test_gemm_fp32_master_weight_grad(cuda_device):
    """bf16 activations with an fp32 weight: compute in bf16, grad_weight written in fp32."""
    B, T, K, F = 8, 512, 768, 2322
    gen = torch.Generator(device=cuda_device).manual_seed(11)
    x = (torch.randn(B, T, K, device=cuda_device, generator=gen) / K**0.5).to(torch.bfloat16).requires_grad_(True)
    w = (torch.randn(F, K, device=cuda_device, generator=gen) / K**0.5).requires_grad_(True)  # fp32
    g = torch.randn(B, F, T, device=cuda_device, generator=gen).to(torch.bfloat16)
    out = FLT(x, w)
    assert out.dtype == torch.bfloat16
    out.backward(g)
    assert w.grad.dtype == torch.float32
    eo, egx, egw = _reference(x, w.detach().to(torch.bfloat16), g)
    assert max_rel_err(out.detach().float().cpu().numpy(), eo.cpu().numpy()) <= 2e-2
    assert max_rel_err(x.grad.float().cpu().numpy(), egx.cpu().numpy()) <= 2e-2
    # fp32 (tensor-core) accumulation over 4096 tokens, written in fp32: norm-wise bound, since
    # entries that cancel to near zero carry the accumulation noise of the whole sum
    assert max_rel_err(w.grad.cpu().numpy(), egw.cpu().numpy(), 1.0) <= 1e-5


# Ragged tile edges: token counts and channel counts that are not multiples of the 256-row tiles
# or 64-wide k-blocks, head-dim totals F that leave a narrow last column tile, odd batch counts
# (the fp32 weight gradient is then reduced in one pass instead of two halves), both layouts.
@pytest.mark.parametrize("B,T,K,F,grad_layout", [(5, 264, 200, 130, "contiguous"), (6, 136, 72, 40, "transposed"),
                                                 (2, 1024, 768, 2322, "transposed"), (1, 8, 8, 8, "contiguous")])
def test_gemm_ragged_shapes_fp32_weight_grad(cuda_device, B, T, K, F, grad_layout):
    gen = torch.Generator(device=cuda_device).manual_seed(B + T + K + F)
    x = (torch.randn(B, T, K, device=cuda_device, generator=gen) / K**0.5).to(torch.bfloat16)
    w = (torch.randn(F, K, device=cuda_device, generator=gen) / K**0.5).to(torch.bfloat16)
    g = torch.randn(B, F, T, device=cuda_device, generator=gen).to(torch.bfloat16)
    if grad_layout == "transposed":
        g = g.transpose(1, 2).contiguous().transpose(1, 2)
    out = FLT(x, w)
    gx = torch.empty_like(x)
    gw = torch.full((F, K), float("nan"), device=cuda_device)  # fp32: every entry must be written
    BWD(x, w, g, gx, gw)
    eo, egx, egw = _reference(x, w, g)
    assert max_rel_err(out.float().cpu().numpy(), eo.cpu().numpy()) <= 2e-2
    assert max_rel_err(gx.float().cpu().numpy(), egx.cpu().numpy()) <= 2e-2
    assert max_rel_err(gw.cpu().numpy(), egw.cpu().numpy(), 1.0) <= 1e-5


def test_gemm_weight_grad_deterministic(cuda_device):
    """The fp32 weight gradient taken in two batch halves is the same on every run."""
    B, T, K, F = 8, 512, 768, 2322
    gen = torch.Generator(device=cuda_device).manual_seed(3)
    x = (torch.randn(B, T, K, device=cuda_device, generator=gen) / K**0.5).to(torch.bfloat16)
    w = (torch.randn(F, K, device=cuda_device, generator=gen) / K**0.5).to(torch.bfloat16)
    g = torch.randn(B, F, T, device=cuda_device, generator=gen).to(torch.bfloat16)
    gx = torch.empty_like(x)
    first = torch.empty(F, K, device=cuda_device)
    BWD(x, w, g, gx, first)
    for _ in range(3):
        again = torch.empty(F, K, device=cuda_device)
        BWD(x, w, g, gx, again)
        assert torch.equal(again, first)


def test_gemm_fp32_config1(cuda_device):
    """Config-1 projection shape in fp32 (CUDA-core fp32 products): max rel err <= 1e-5."""
    B, T, K, F = 2, 256, 768, 2322
    gen = torch.Generator(device=cuda_device).manual_seed(1)
    x = torch.randn(B, T, K, device=cuda_device, generator=gen, requires_grad=True)
    w = (torch.randn(F, K, device=cuda_device, generator=gen) / K**0.5).requires_grad_(True)
    g = torch.randn(B, F, T, device=cuda_device, generator=gen)
    out = FLT(x, w)
    out.backward(g)
    xd, wd, gd = x.detach().double(), w.detach().double(), g.double()
    eo = torch.matmul(wd, xd.transpose(1, 2))
    egx = torch.matmul(gd.transpose(1, 2), wd)
    egw = torch.einsum("bft,btk->fk", gd, xd)
    assert max_rel_err(out.detach().cpu().numpy(), eo.cpu().numpy()) <= 1e-5
    assert max_rel_err(x.grad.cpu().numpy(), egx.cpu().numpy()) <= 1e-5
    assert max_rel_err(w.grad.cpu().numpy(), egw.cpu().numpy()) <= 1e-5


def test_gemm_rejects_bad_layouts(cuda_device):
    x = torch.randn(2, 16, 32, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(40, 32, device=cuda_device, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="contiguous"):
        FLT(x.transpose(1, 2).contiguous().transpose(1, 2), w)
    g = torch.randn(2, 16, 40, device=cuda_device, dtype=torch.bfloat16).permute(0, 2, 1)[:, ::2]
    with pytest.raises(RuntimeError):
        BWD(x, w, g, torch.empty_like(x), torch.empty_like(w))
