"""C-ABI checks that need no GPU: the library loads, exports every entry point include/ltvqkv.h
declares, and validates arguments before touching the device."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import ROOT
from nanochat_filter_b200 import _lib

HEADER = os.path.join(ROOT, "include", "ltvqkv.h")


def declared_symbols():
    text = open(HEADER).read()
    return re.findall(r"LTVQKV_API\s+[\w\s\*]+?\b(ltvqkv_\w+)\s*\(", text)


def test_header_declares_all_bound_symbols():
    syms = declared_symbols()
    assert len(syms) == len(set(syms))
    assert set(syms) == set(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for s in declared_symbols():
        assert hasattr(lib, s), s
        assert ctypes.cast(getattr(lib, s), ctypes.c_void_p).value


def test_version_and_status_strings():
    lib = _lib.load()
    assert lib.ltvqkv_abi_version() == 1
    for code, text in ((0, "ok"), (2, "shape"), (7, "timed out"), (8, "workspace")):
        assert text in lib.ltvqkv_status_string(code).decode()
    assert lib.ltvqkv_status_string(999).decode() == "unknown status"


def test_workspace_sizes():
    lib = _lib.load()
    small = lib.ltvqkv_scan_workspace_bytes(1, 16, 1, 1, 1, 2)
    big = lib.ltvqkv_scan_workspace_bytes(32, 1024, 6, 6, 1, 128)
    assert 256 < small < big
    assert lib.ltvqkv_scan_workspace_bytes(1, 16, 1, 1, 0, 2) == 0  # invalid shape
    assert lib.ltvqkv_scan_workspace_bytes(1, 16, 1, 1, 1, 2048) == 0  # head dim beyond 1024
    assert lib.ltvqkv_gemm_workspace_bytes() >= 256


def test_lookback_bwd_workspace_sizes():
    """The look-back backward's workspace query asks for the chunk-parallel slots exactly when that
    form applies (bf16, K - 1 <= min(P, Q) and <= 64, more than one chunk, D + Da <= 256, r % 32 == 0);
    otherwise it returns the one-CTA-per-row form's size."""
    lib = _lib.load()
    r256 = lambda n: (n + 255) // 256 * 256
    base = lib.ltvqkv_lookback_workspace_bytes(32, 6, 6, 1)
    full = lib.ltvqkv_lookback_bwd_workspace_bytes(32, 1024, 6, 6, 1, 128, 128, 112, 17)
    # 576 rows x 9 chunks; two slot arrays of 16 token rows of 136 entries (129 padded to 16 bytes),
    # the chunks' fp32 initial-state gradients and logit-bias partials
    slots = 32 * 18 * 9
    assert full == r256(base) + 2 * r256(slots * 16 * 136 * 2) + slots * 128 * 4 + r256(slots * 4)
    for args in ((2, 300, 1, 1, 1, 128, 224, 100, 125),   # warm-up prefix longer than a chunk
                 (2, 100, 1, 1, 1, 128, 1024, 1024, 1),   # one chunk
                 (2, 256, 1, 1, 2, 2, 32, 32, 5),          # r not a multiple of 32
                 (2, 256, 1, 1, 2, 128, 32, 32, 5),        # D + Da > 256
                 (2, 1024, 1, 1, 1, 128, 128, 112, 66)):   # prefix beyond 64 tokens
        B, T, NH, NKVH, Da = args[:5]
        assert lib.ltvqkv_lookback_bwd_workspace_bytes(*args) == lib.ltvqkv_lookback_workspace_bytes(B, NH, NKVH, Da), args


def test_argument_validation_without_device():
    lib = _lib.load()
    # bad dtype code
    assert lib.ltvqkv_scan_fwd(7, None, 0, 0, 0, None, None, None, None, None, 1, 1, 1, 1, 1, 1, 1, None, 0,
                               None) == 4
    # empty batch / sequence: nothing to do
    assert lib.ltvqkv_scan_fwd(1, None, 0, 0, 0, None, None, None, None, None, 0, 5, 1, 1, 1, 1, 1, None, 0,
                               None) == 0
    assert lib.ltvqkv_scan_fwd(1, None, 0, 0, 0, None, None, None, None, None, 3, 0, 1, 1, 1, 1, 1, None, 0,
                               None) == 0
    # missing data pointers
    assert lib.ltvqkv_scan_fwd(1, None, 0, 0, 0, None, None, None, None, None, 1, 4, 1, 1, 1, 1, 1, None, 0,
                               None) == 1
    # workspace too small (checked before any launch)
    fake = ctypes.c_void_p(0x10000)
    assert lib.ltvqkv_scan_fwd(1, fake, 12, 1, 4, fake, fake, fake, fake, fake, 1, 4, 1, 1, 1, 1, 1, fake, 16,
                               None) == 8
    # negative / inconsistent shapes
    assert lib.ltvqkv_gemm_fwd(1, None, None, None, -1, 4, 4, 4, None, 0, None) == 2
    assert lib.ltvqkv_gemm_fwd(1, None, None, None, 0, 4, 4, 4, None, 0, None) == 0
    assert lib.ltvqkv_gemm_bwd(1, None, None, None, 12, 1, 4, None, None, 0, 1, 4, 4, 3, None, 0, None) == 3
    assert lib.ltvqkv_decode_step(1, None, None, None, None, None, None, None, None, None, None, None, None,
                                  None, None, None, None, 0, 8, 1, 1, 1, 1, 1, None) == 0
    assert lib.ltvqkv_decode_step(1, None, None, None, None, None, None, None, None, None, None, None, None,
                                  None, None, None, None, 2, 8, 1, 1, 1, 1, 1, None) == 1
    # checkpoint forms: a missing or misaligned checkpoint buffer, or an initial-state stride other
    # than H * D or 0, is rejected before any device work
    assert lib.ltvqkv_proj_scan_fwd_ckpt(1, fake, fake, fake, 0, fake, fake, fake, fake, fake, None, 2, 64, 64, 1, 1,
                                         1, 128, 1, fake, 4096, None) == 1
    assert lib.ltvqkv_proj_scan_fwd_ckpt(1, fake, fake, fake, 0, fake, fake, fake, fake, fake,
                                         ctypes.c_void_p(0x10004), 2, 64, 64, 1, 1, 1, 128, 1, fake, 4096, None) == 1
    assert lib.ltvqkv_proj_scan_fwd_ckpt(1, fake, fake, fake, 5, fake, fake, fake, fake, fake, fake, 2, 64, 64, 1, 1,
                                         1, 128, 1, fake, 4096, None) == 3
    st = _lib.strides([0, 0, 0, 1])
    assert lib.ltvqkv_scan_bwd_ckpt(1, fake, 0, 1, 64, fake, 0, fake, None, fake, st, fake, st, fake, st,
                                    fake, 0, 1, 64, fake, fake, 2, 64, 1, 1, 1, 128, 1, fake, 4096, None) == 1
    assert lib.ltvqkv_scan_bwd_ckpt(1, fake, 0, 1, 64, fake, 7, fake, fake, fake, st, fake, st, fake, st,
                                    fake, 0, 1, 64, fake, fake, 2, 64, 1, 1, 1, 128, 1, fake, 4096, None) == 3


def test_check_raises_runtime_error():
    with pytest.raises(RuntimeError, match="ltvqkv_scan_fwd failed: invalid argument"):
        _lib.check(1, "ltvqkv_scan_fwd")
    with pytest.raises(TypeError):
        import torch

        _lib.dtype_code(torch.float16)
