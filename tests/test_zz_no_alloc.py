"""The allocation-free forward-scan entry point, ltvqkv_scan_fwd_noalloc.

Some callers cannot allocate device memory or hand the library a workspace on the call path
(plugin hosts and serving runtimes that own all device memory under a fixed plan, foreign-language
callers without an allocator). For them the library keeps the forward scan's look-back scratch in
a fixed 32 MiB device array of its own. This test calls that entry point through the C ABI and
checks that its results equal those of the workspace-taking entry point (same kernel, so equal to
the bit; the bf16 bound of the other tests is asserted as well), on two consecutive calls with
different inputs, and that a problem too large for the array is refused with LTVQKV_ERR_TOO_LARGE.
This file is collected last so that a run stopping at the first failure has run everything else.
"""

from __future__ import annotations

import pytest
import torch

import nanochat_filter_b200  # noqa: F401
from conftest import max_rel_err
from nanochat_filter_b200 import _lib

pytestmark = pytest.mark.gpu

LTVQKV_ERR_TOO_LARGE = 10


def _inputs(dev, seed, B, T, NH, NKVH, Da, r, dtype):
    g = torch.Generator(device="cpu").manual_seed(seed)
    H, D = NH + 2 * NKVH, Da * r
    F = H * (D + Da)
    comb = torch.randn(B, F, T, generator=g).to(dev, dtype).transpose(1, 2)  # [B, T, F] view, t contiguous
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


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_workspace_entry_point_on_two_calls(cuda_device, dtype):
    NH, NKVH, Da, r, B, T = 6, 6, 1, 128, 4, 1024
    for seed in (101, 202):  # two calls in a row; the second must not see the first's state
        comb, inits, bias = _inputs(cuda_device, seed, B, T, NH, NKVH, Da, r, dtype)
        ref = torch.ops.nanochat_cuda.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_op(
            comb, inits, bias, NH, NKVH, Da, r, 8, 8, 4, 32, 2, 8, True)
        got = _noalloc(comb, inits, bias, NH, NKVH, Da, r)
        torch.cuda.synchronize()
        tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
        for a, e in zip(got, ref):
            assert torch.equal(a, e)
            assert max_rel_err(a.float().cpu().numpy(), e.float().cpu().numpy(), 1e-2) <= tol


def test_noalloc_refuses_problems_beyond_its_scratch(cuda_device):
    L = _lib.load()
    fake = 0x10000  # never dereferenced: the size check comes before any launch
    rc = L.ltvqkv_scan_fwd_noalloc(_lib.DTYPE_BF16, fake, 0, 1, 1, fake, fake, fake, fake, fake,
                                   64, 16384, 8, 8, 1, 128, 1, _lib.stream_handle(cuda_device))
    assert rc == LTVQKV_ERR_TOO_LARGE
    assert "32 MiB" in L.ltvqkv_status_string(rc).decode()
