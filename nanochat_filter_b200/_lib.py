"""ctypes binding of libltvqkv.so, the C ABI declared in include/ltvqkv.h.

Every call passes raw device pointers, element strides and sizes plus the current CUDA stream
of the calling thread. A non-zero status raises RuntimeError naming the entry point, the
status text and the last CUDA error — the same error class the reference's TORCH_CHECK
produces (cpp_ewma/src/*.cu). A missing library raises ImportError on first use; there is no
fallback implementation.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional, Sequence

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libltvqkv.so")

DTYPE_F32 = 0
DTYPE_BF16 = 1
ERR_UNSUPPORTED = 9  # LTVQKV_ERR_UNSUPPORTED: a valid request this entry point does not take

EXPORTED_SYMBOLS = (
    "ltvqkv_abi_version",
    "ltvqkv_status_string",
    "ltvqkv_last_cuda_error",
    "ltvqkv_scan_workspace_bytes",
    "ltvqkv_scan_fwd",
    "ltvqkv_scan_bwd",
    "ltvqkv_scan_bwd_ckpt",
    "ltvqkv_gemm_workspace_bytes",
    "ltvqkv_gemm_fwd",
    "ltvqkv_gemm_bwd",
    "ltvqkv_decode_step",
    "ltvqkv_workspace_error",
    "ltvqkv_debug_wait_timeout",
    "ltvqkv_scan_fwd_noalloc",
    "ltvqkv_scan_noalloc_error",
    "ltvqkv_proj_scan_fwd",
    "ltvqkv_proj_scan_fwd_ckpt",
    "ltvqkv_proj_scan_fwd_ckpt_rope",
    "ltvqkv_lookback_workspace_bytes",
    "ltvqkv_lookback_bwd_workspace_bytes",
    "ltvqkv_lookback_scan_fwd",
    "ltvqkv_lookback_scan_bwd",
    "ltvqkv_rotary_qk_norm_fwd",
    "ltvqkv_rotary_qk_norm_bwd",
    "ltvqkv_rotary_qk_norm_bwd_ckpt",
)

_lib: Optional[ctypes.CDLL] = None
_lib_lock = threading.Lock()

_vp = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_sz = ctypes.c_size_t
_pi64 = ctypes.POINTER(ctypes.c_int64)
_pf = ctypes.c_void_p


def _declare(lib: ctypes.CDLL) -> None:
    lib.ltvqkv_abi_version.restype = _i
    lib.ltvqkv_abi_version.argtypes = []
    lib.ltvqkv_status_string.restype = ctypes.c_char_p
    lib.ltvqkv_status_string.argtypes = [_i]
    lib.ltvqkv_last_cuda_error.restype = ctypes.c_char_p
    lib.ltvqkv_last_cuda_error.argtypes = []
    lib.ltvqkv_scan_workspace_bytes.restype = _sz
    lib.ltvqkv_scan_workspace_bytes.argtypes = [_i, _i, _i, _i, _i, _i]
    lib.ltvqkv_scan_fwd.restype = _i
    lib.ltvqkv_scan_fwd.argtypes = [_i, _vp, _i64, _i64, _i64, _vp, _pf, _vp, _vp, _vp,
                                    _i, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]
    lib.ltvqkv_scan_bwd.restype = _i
    lib.ltvqkv_scan_bwd.argtypes = [_i, _vp, _i64, _i64, _i64, _vp, _pf,
                                    _vp, _pi64, _vp, _pi64, _vp, _pi64,
                                    _vp, _pi64, _vp, _pi64, _vp, _pi64,
                                    _vp, _i64, _i64, _i64, _vp, _pf,
                                    _i, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]
    lib.ltvqkv_scan_bwd_ckpt.restype = _i
    lib.ltvqkv_scan_bwd_ckpt.argtypes = [_i, _vp, _i64, _i64, _i64, _vp, _i64, _pf, _pf,
                                         _vp, _pi64, _vp, _pi64, _vp, _pi64,
                                         _vp, _i64, _i64, _i64, _vp, _pf,
                                         _i, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]
    lib.ltvqkv_rotary_qk_norm_bwd_ckpt.restype = _i
    lib.ltvqkv_rotary_qk_norm_bwd_ckpt.argtypes = [_i, _vp, _vp, _i64, _pf, _pf, _vp, _vp, _i64, ctypes.c_float,
                                                   _vp, _pi64, _vp, _pi64, _vp, _pi64, _vp, _pi64,
                                                   _i, _i, _i, _i, _i, _i, _i, _vp]
    lib.ltvqkv_lookback_workspace_bytes.restype = _sz
    lib.ltvqkv_lookback_workspace_bytes.argtypes = [_i, _i, _i, _i]
    lib.ltvqkv_lookback_bwd_workspace_bytes.restype = _sz
    lib.ltvqkv_lookback_bwd_workspace_bytes.argtypes = [_i, _i, _i, _i, _i, _i, _i64, _i64, _i64]
    lib.ltvqkv_lookback_scan_fwd.restype = _i
    lib.ltvqkv_lookback_scan_fwd.argtypes = [_i, _vp, _i64, _i64, _i64, _vp, _pf, _vp, _vp, _vp,
                                             _i, _i, _i, _i, _i, _i, _i64, _i64, _i64, _i, _vp]
    lib.ltvqkv_lookback_scan_bwd.restype = _i
    lib.ltvqkv_lookback_scan_bwd.argtypes = [_i, _vp, _i64, _i64, _i64, _vp, _pf,
                                             _vp, _pi64, _vp, _pi64, _vp, _pi64,
                                             _vp, _pi64, _vp, _pi64, _vp, _pi64,
                                             _vp, _i64, _i64, _i64, _vp, _pf,
                                             _i, _i, _i, _i, _i, _i, _i64, _i64, _i64, _i, _vp, _sz, _vp]
    lib.ltvqkv_rotary_qk_norm_fwd.restype = _i
    lib.ltvqkv_rotary_qk_norm_fwd.argtypes = [_i, _vp, _pi64, _vp, _pi64, _vp, _vp, _pi64, _vp, _pi64, _vp, _pi64,
                                              _i, _i, _i, _i, _i, ctypes.c_float, _vp]
    lib.ltvqkv_rotary_qk_norm_bwd.restype = _i
    lib.ltvqkv_rotary_qk_norm_bwd.argtypes = [_i, _vp, _pi64, _vp, _pi64, _vp, _vp, _pi64, _vp, _pi64, _vp, _pi64,
                                              _vp, _pi64, _vp, _pi64, _i, _i, _i, _i, _i, ctypes.c_float, _vp]
    lib.ltvqkv_gemm_workspace_bytes.restype = _sz
    lib.ltvqkv_gemm_workspace_bytes.argtypes = []
    lib.ltvqkv_gemm_fwd.restype = _i
    lib.ltvqkv_gemm_fwd.argtypes = [_i, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz, _vp]
    lib.ltvqkv_proj_scan_fwd.restype = _i
    lib.ltvqkv_proj_scan_fwd.argtypes = [_i, _vp, _vp, _vp, _pf, _vp, _vp, _vp, _vp,
                                         _i, _i, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]
    lib.ltvqkv_proj_scan_fwd_ckpt.restype = _i
    lib.ltvqkv_proj_scan_fwd_ckpt.argtypes = [_i, _vp, _vp, _vp, _i64, _pf, _vp, _vp, _vp, _vp, _pf,
                                              _i, _i, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]
    lib.ltvqkv_proj_scan_fwd_ckpt_rope.restype = _i
    lib.ltvqkv_proj_scan_fwd_ckpt_rope.argtypes = [_i, _vp, _vp, _vp, _i64, _pf, _vp, _vp, _vp, _vp, _pf,
                                                   _vp, _vp, _i64, ctypes.c_float,
                                                   _i, _i, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]
    lib.ltvqkv_gemm_bwd.restype = _i
    lib.ltvqkv_gemm_bwd.argtypes = [_i, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp, _i,
                                    _i, _i, _i, _i, _vp, _sz, _vp]
    lib.ltvqkv_decode_step.restype = _i
    lib.ltvqkv_decode_step.argtypes = [_i, _vp, _vp, _pf,
                                       _vp, _pi64, _vp, _pi64, _vp, _pi64, _vp,
                                       _vp, _pi64, _vp, _pi64, _vp, _pi64,
                                       _i, _i, _i, _i, _i, _i, _i, _vp]
    lib.ltvqkv_workspace_error.restype = _i
    lib.ltvqkv_workspace_error.argtypes = [_vp, _vp, ctypes.POINTER(ctypes.c_uint32)]
    lib.ltvqkv_scan_fwd_noalloc.restype = _i
    lib.ltvqkv_scan_fwd_noalloc.argtypes = [_i, _vp, _i64, _i64, _i64, _vp, _pf, _vp, _vp, _vp,
                                            _i, _i, _i, _i, _i, _i, _i, _vp]
    lib.ltvqkv_scan_noalloc_error.restype = _i
    lib.ltvqkv_scan_noalloc_error.argtypes = [_vp, ctypes.POINTER(ctypes.c_uint32)]
    lib.ltvqkv_debug_wait_timeout.restype = _i
    lib.ltvqkv_debug_wait_timeout.argtypes = [_vp, ctypes.c_uint64, _vp]


def load() -> ctypes.CDLL:
    """Loads libltvqkv.so (raises ImportError when it has not been built)."""
    global _lib
    if _lib is None:
        with _lib_lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is missing: build it with `python -m nanochat_filter_b200.build` "
                        "(the filtered-QKV ops have no fallback implementation)")
                lib = ctypes.CDLL(LIB_PATH)
                _declare(lib)
                _lib = lib
    return _lib


def is_available() -> bool:
    try:
        load()
        return True
    except (ImportError, OSError):
        return False


def check(rc: int, what: str) -> None:
    if rc != 0:
        lib = load()
        msg = lib.ltvqkv_status_string(rc).decode()
        cuda = lib.ltvqkv_last_cuda_error().decode()
        raise RuntimeError(f"{what} failed: {msg}" + (f" ({cuda})" if cuda else ""))


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return DTYPE_F32
    if dtype == torch.bfloat16:
        return DTYPE_BF16
    raise TypeError(f"unsupported dtype {dtype}: the filtered-QKV kernels take float32 or bfloat16")


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def strides(seq: Sequence[int]):
    arr = (ctypes.c_int64 * len(seq))(*[int(s) for s in seq])
    return arr


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# ------------------------------------------------------------------------------------------
# Workspaces: one zero-initialised byte buffer per (device, stream), grown on demand. The
# kernels leave a workspace ready for the next call on the same stream (counters reset,
# look-back flags epoch-tagged), so it is allocated and zeroed only when it grows.
# ------------------------------------------------------------------------------------------
_ws_lock = threading.Lock()
_workspaces: dict = {}


def workspace(device: torch.device, nbytes: int, kind: str = "shared") -> torch.Tensor:
    """The zero-initialised workspace of (device, current stream, kind). ltvqkv_gemm_bwd keeps counters
    after the header that must read zero at each launch, so it takes kind="gemm_bwd" (a buffer the
    scan entry points, whose look-back flags stay set between calls, never use)."""
    dev = torch.device(device)
    key = (dev.index if dev.index is not None else torch.cuda.current_device(), stream_handle(dev), kind)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            size = max(int(nbytes), 4096)
            if ws is not None:
                size = max(size, 2 * ws.numel())
            ws = torch.zeros(size, dtype=torch.uint8, device=dev)
            _workspaces[key] = ws
        return ws


def workspace_error(ws: torch.Tensor) -> int:
    """Reads and clears the device-side error word of a workspace (synchronises its stream)."""
    lib = load()
    err = ctypes.c_uint32(0)
    check(lib.ltvqkv_workspace_error(ws.data_ptr(), stream_handle(ws.device), ctypes.byref(err)),
          "ltvqkv_workspace_error")
    return int(err.value)


def noalloc_error(device: torch.device) -> int:
    """Reads and clears the error word of ltvqkv_scan_fwd_noalloc's array on `device` (synchronises
    the device's current stream)."""
    lib = load()
    err = ctypes.c_uint32(0)
    with torch.cuda.device(device):
        check(lib.ltvqkv_scan_noalloc_error(stream_handle(device), ctypes.byref(err)), "ltvqkv_scan_noalloc_error")
    return int(err.value)


def all_workspace_errors() -> int:
    """OR of the error words of every cached workspace (0 when no wait ever timed out)."""
    out = 0
    with _ws_lock:
        items = list(_workspaces.values())
    for ws in items:
        out |= workspace_error(ws)
    return out
