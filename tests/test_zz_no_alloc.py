"""The allocation-free forward-scan entry point, ltvqkv_scan_fwd_noalloc, and its error query.

Some callers cannot allocate device memory or hand the library a workspace on the call path
(plugin hosts and serving runtimes that own all device memory under a fixed plan, foreign-language
callers without an allocator). For them the library keeps the forward scan's scratch in a fixed
32 MiB device array of its own. These tests call that entry point through the C ABI, twice in a
row with different inputs each time, on the three kernel families it can reach:

* the chunked three-pass kernels (few long rows, t-contiguous `combined`): equal to the
  workspace-taking entry point bit for bit, and to the oracle within the bf16 / fp32 bounds;
* the row-streaming kernel (B * heads >= 2 * SMs, the training layout);
* the generic kernel whose CTAs hand carries to each other through look-back flags and the
  header's epoch (T not a multiple of the chunk, token-major `combined`): the state the
  per-call clearing must reset, checked against the oracle.

After each call the array's error word is read through ltvqkv_scan_noalloc_error and must be 0.
A bounded wait that gives up (the library's failure-path check, pointed at the array) must be
reported by that query, even across a later allocation-free call, and cleared by the read.
A problem too large for the array is refused with LTVQKV_ERR_TOO_LARGE.
This file is collected last so that a run stopping at the first failure has run everything else.
"""

from __future__ import annotations

import pytest
import torch

import nanochat_filter_b200  # noqa: F401
from conftest import max_rel_err
from nanochat_filter_b200 import _lib
from oracle import oracle as O

pytestmark = pytest.mark.gpu

LTVQKV_ERR_TIMEOUT = 7
LTVQKV_ERR_TOO_LARGE = 10
FLOOR = 1e-2


def _inputs(dev, seed, B, T, NH, NKVH, Da, r, dtype, t_contiguous=True):
    g = torch.Generator(device="cpu").manual_seed(seed)
    H, D = NH + 2 * NKVH, Da * r
    F = H * (D + Da)
    if t_contiguous:
        comb = torch.randn(B, F, T, generator=g).to(dev, dtype).transpose(1, 2)  # [B, T, F] view, strides (F*T, 1, T)
    else:
        comb = torch.randn(B, T, F, generator=g).to(dev, dtype)  # token-major [B, T, F]
    inits = (0.5 * torch.randn(B, H, D, generator=g)).to(dev, dtype)
    bias = torch.randn(H, Da, generator=g).to(dev)
    return comb, inits, bias


def _noalloc(comb, inits, bias, NH, NKVH, Da, r):
    L = _lib.load()
    B, T, _ = comb.shape
    D = Da * r
    kw = dict(device=comb.device, dtype=comb.dtype)
    oq, ok, ov = torch.empty(B, NH, T, D, **kw), torch.empty(B, NKVH, T, D, **kw), torch.empty(B, NKVH, T, D, **kw)
    sc = comb.stride()
    rc = L.ltvqkv_scan_fwd_noalloc(_lib.dtype_code(comb.dtype), comb.data_ptr(), sc[0], sc[1], sc[2],
                                   inits.data_ptr(), bias.data_ptr(), oq.data_ptr(), ok.data_ptr(), ov.data_ptr(),
                                   B, T, NH, NKVH, Da, r, 1, _lib.stream_handle(comb.device))
    _lib.check(rc, "ltvqkv_scan_fwd_noalloc")
    return oq, ok, ov


def _oracle(comb, inits, bias, NH, NKVH, Da, r):
    bf16 = comb.dtype == torch.bfloat16
    return O.scan_fwd(comb.float().cpu().numpy(), inits.float().cpu().numpy(), bias.cpu().numpy(), NH, NKVH, Da, r,
                      True, bf16)


def _check_vs_oracle(got, comb, inits, bias, NH, NKVH, Da, r):
    tol = 2e-2 if comb.dtype == torch.bfloat16 else 1e-5
    exp = _oracle(comb, inits, bias, NH, NKVH, Da, r)
    for name, a, e in zip("qkv", got, exp):
        err = max_rel_err(a.float().cpu().numpy(), e, FLOOR)
        assert err <= tol, f"{name}: max relative error {err:.3g} > {tol}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_workspace_entry_point_on_two_calls(cuda_device, dtype):
    """Chunked shape (B * heads = 72): same kernels as the workspace entry, so equal to the bit."""
    NH, NKVH, Da, r, B, T = 6, 6, 1, 128, 4, 1024
    for seed in (101, 202):  # two calls in a row; the second must not see the first's state
        comb, inits, bias = _inputs(cuda_device, seed, B, T, NH, NKVH, Da, r, dtype)
        ref = torch.ops.nanochat_cuda.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_op(
            comb, inits, bias, NH, NKVH, Da, r, 8, 8, 4, 32, 2, 8, True)
        got = _noalloc(comb, inits, bias, NH, NKVH, Da, r)
        torch.cuda.synchronize()
        for a, e in zip(got, ref):
            assert torch.equal(a, e)
        _check_vs_oracle(got, comb, inits, bias, NH, NKVH, Da, r)
        assert _lib.noalloc_error(cuda_device) == 0


def test_noalloc_row_streaming_shape_on_two_calls(cuda_device):
    """The training layout with B * heads >= 2 * SMs (row-streaming kernel: tickets from the header)."""
    NH, NKVH, Da, r, B, T = 6, 6, 1, 128, 32, 256
    for seed in (303, 404):
        comb, inits, bias = _inputs(cuda_device, seed, B, T, NH, NKVH, Da, r, torch.bfloat16)
        ref = torch.ops.nanochat_cuda.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_op(
            comb, inits, bias, NH, NKVH, Da, r, 8, 8, 4, 32, 2, 8, True)
        got = _noalloc(comb, inits, bias, NH, NKVH, Da, r)
        torch.cuda.synchronize()
        for a, e in zip(got, ref):
            assert torch.equal(a, e)
        _check_vs_oracle(got, comb, inits, bias, NH, NKVH, Da, r)
        assert _lib.noalloc_error(cuda_device) == 0


def test_noalloc_generic_lookback_kernel_on_two_calls(cuda_device):
    """Token-major `combined` and T = 1000 (not a multiple of the chunk): the generic kernel, whose
    chunks wait on look-back flags tagged with the header's epoch. Two calls against the oracle."""
    NH, NKVH, Da, r, B, T = 2, 1, 2, 64, 3, 1000
    for seed in (505, 606):
        comb, inits, bias = _inputs(cuda_device, seed, B, T, NH, NKVH, Da, r, torch.bfloat16, t_contiguous=False)
        got = _noalloc(comb, inits, bias, NH, NKVH, Da, r)
        torch.cuda.synchronize()
        _check_vs_oracle(got, comb, inits, bias, NH, NKVH, Da, r)
        assert _lib.noalloc_error(cuda_device) == 0


def test_noalloc_timeout_is_reported_by_the_error_query(cuda_device):
    """A bounded wait that gives up on the array (the library's failure-path check with no workspace
    targets it) is reported by ltvqkv_scan_noalloc_error even after another allocation-free call,
    and the read clears it. The wait ends by itself after 50 ms; the context stays usable."""
    L = _lib.load()
    assert _lib.noalloc_error(cuda_device) == 0
    rc = L.ltvqkv_debug_wait_timeout(None, 50_000_000, _lib.stream_handle(cuda_device))
    _lib.check(rc, "ltvqkv_debug_wait_timeout")
    NH, NKVH, Da, r, B, T = 2, 1, 1, 128, 2, 256
    comb, inits, bias = _inputs(cuda_device, 707, B, T, NH, NKVH, Da, r, torch.bfloat16)
    got = _noalloc(comb, inits, bias, NH, NKVH, Da, r)  # a later call leaves the recorded error in place
    torch.cuda.synchronize()
    assert _lib.noalloc_error(cuda_device) == LTVQKV_ERR_TIMEOUT
    assert _lib.noalloc_error(cuda_device) == 0  # cleared by the read
    _check_vs_oracle(got, comb, inits, bias, NH, NKVH, Da, r)


def test_noalloc_refuses_problems_beyond_its_scratch(cuda_device):
    L = _lib.load()
    fake = 0x10000  # never dereferenced: the size check comes before any launch
    rc = L.ltvqkv_scan_fwd_noalloc(_lib.DTYPE_BF16, fake, 0, 1, 1, fake, fake, fake, fake, fake,
                                   64, 16384, 8, 8, 1, 128, 1, _lib.stream_handle(cuda_device))
    assert rc == LTVQKV_ERR_TOO_LARGE
    assert "32 MiB" in L.ltvqkv_status_string(rc).decode()
