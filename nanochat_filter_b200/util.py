"""Dtype policy, init-state resolution and scan tunables of the filtered-QKV path.

Mirrors nanochat/ltv_fused_concat_register_cast_scan_util.py:1-70 of the reference: the
same names, the same autocast decision and the same environment variables. The six tuning
integers are still read and passed through the operator schema; the B200 kernels choose their
own tiling and ignore them.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Optional

import torch

CUDA_SUPPORTS_NATIVE_BF16 = torch.cuda.is_available() and torch.cuda.is_bf16_supported(including_emulation=False)


@dataclass
class LtvInitValues:
    """Cached filter state per head group (reference nanochat/ltv/ltv_filter.py:35-39)."""

    q: Optional[torch.Tensor] = None
    k: Optional[torch.Tensor] = None
    v: Optional[torch.Tensor] = None


def env_int(name: str, default: int) -> int:
    v = os.environ.get(name)
    return default if v is None or v == "" else int(v)


def should_run_cuda_ltv_in_fp32(tensor: torch.Tensor) -> bool:
    return not CUDA_SUPPORTS_NATIVE_BF16 and tensor.dtype == torch.bfloat16 and tensor.is_cuda


def should_run_ltv_in_fp32(device_type: str) -> bool:
    """True only when autocast asks for fp32, or for bf16 on a device without native bf16."""
    if torch.is_autocast_enabled(device_type):
        autocast_dtype = torch.get_autocast_dtype(device_type)
        if device_type == "cuda":
            if autocast_dtype == torch.float32:
                return True
            if autocast_dtype == torch.bfloat16 and not CUDA_SUPPORTS_NATIVE_BF16:
                return True
        return False
    return False


def resolve_inits_original_dtype(B: int, init_param: torch.Tensor, previous_values: LtvInitValues) -> torch.Tensor:
    """[B, H, D] start state: cached q/k/v states concatenated over heads, else init_param."""
    if previous_values.q is not None:
        return torch.cat([previous_values.q, previous_values.k, previous_values.v], dim=1)
    return init_param.unsqueeze(0).expand(B, -1, -1)


_SCAN_THREADS_FORWARD = env_int("LTV_CUDA_FUSED_CONCAT_HEAD_MAJOR_REGISTER_CAST_SCAN_THREADS_FORWARD", 8)
_R_THREADS_FORWARD = env_int("LTV_CUDA_FUSED_CONCAT_HEAD_MAJOR_REGISTER_CAST_R_THREADS_FORWARD", 8)
_R_ITEMS_FORWARD = env_int("LTV_CUDA_FUSED_CONCAT_HEAD_MAJOR_REGISTER_CAST_R_ITEMS_FORWARD", 4)
_SCAN_THREADS_BACKWARD = env_int("LTV_CUDA_FUSED_CONCAT_HEAD_MAJOR_REGISTER_CAST_SCAN_THREADS_BACKWARD", 32)
_R_THREADS_BACKWARD = env_int("LTV_CUDA_FUSED_CONCAT_HEAD_MAJOR_REGISTER_CAST_R_THREADS_BACKWARD", 2)
_R_ITEMS_BACKWARD = env_int("LTV_CUDA_FUSED_CONCAT_HEAD_MAJOR_REGISTER_CAST_R_ITEMS_BACKWARD", 8)
