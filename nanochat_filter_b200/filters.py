"""Filter modules of the filtered-QKV layer (drop-in for the reference's classes).

LtvCombinedQkvFilterBase          nanochat/ltv_combined_qkv_filter_base.py:11-71
LtvCombinedHeadMajorQkvFilter     nanochat/ltv_combined_head_major_qkv_filter.py:11-66
LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter
                                  nanochat/ltv_cuda_fused_concat_head_major_register_cast_blelloch_scan_qkv_filter.py:21-73

Parameters keep the reference's names, shapes and layout — `c.weight` [H*(D+Da), C] with
head-major interleaved rows (Q heads, K heads, V heads; per head D value rows then Da logit
rows), `logit_bias` [H, Da] and `init_param` [H, D] — so state dicts and checkpoints load
unchanged. forward(x, previous_values) returns q, k, v as [B, T, heads, D] views of
head-major [B, heads, T, D] storage.
"""

from __future__ import annotations

from abc import abstractmethod

import torch
import torch.nn as nn

from . import ops as _ops
from .util import (
    CUDA_SUPPORTS_NATIVE_BF16,
    LtvInitValues,
    _R_ITEMS_BACKWARD,
    _R_ITEMS_FORWARD,
    _R_THREADS_BACKWARD,
    _R_THREADS_FORWARD,
    _SCAN_THREADS_BACKWARD,
    _SCAN_THREADS_FORWARD,
    resolve_inits_original_dtype,
)


def init_weights_of_init(init_param: torch.Tensor, n_head: int, n_kv_head: int, init_s: float) -> None:
    """Uniform(-init_s, init_s) initial state per head (reference nanochat/ltv/ltv_fused_scan_filter.py:17-39)."""
    assert init_param.shape[0] == n_head + 2 * n_kv_head, "init_param size mismatch"
    assert init_param.requires_grad
    with torch.no_grad():
        init_param.uniform_(-init_s, init_s)


class LtvCombinedQkvFilterBase(nn.Module):
    """One projection `c` producing values and decay logits for all Q, K, V heads."""

    def __init__(self, n_head: int, n_kv_head: int, head_dim: int, r: int):
        super().__init__()
        assert head_dim % r == 0, "Head dimension must be divisible by r"
        num_alpha_groups = head_dim // r
        total_active_heads = n_head + 2 * n_kv_head
        self.c = nn.Linear(n_head * head_dim, total_active_heads * (head_dim + num_alpha_groups), bias=False)
        self.init_param = nn.Parameter(torch.empty(total_active_heads, head_dim))
        self.head_dim = head_dim
        self.n_head = n_head
        self.n_kv_head = n_kv_head
        self.num_alpha_groups = num_alpha_groups
        self.total_active_heads = total_active_heads
        self.r = r
        self.q_size = n_head * head_dim
        self.kv_size = n_kv_head * head_dim
        self.logit_size = total_active_heads * self.num_alpha_groups
        self.split_sections = [self.q_size, self.kv_size, self.kv_size, self.logit_size]

    @abstractmethod
    def forward(self, x, previous_values: LtvInitValues) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        pass

    @abstractmethod
    def init_weights(self, alpha_mlp_bias_init: float, weight_s: float, bias_s: float, init_s: float):
        pass

    def get_matrix_linear_params(self):
        return [self.c.weight], [self.logit_bias, self.init_param]

    def get_init_parameters(self):
        return [self.init_param]

    def estimate_flops(self, sequence_len: int) -> int:
        alpha_proj_params = self.total_active_heads * self.num_alpha_groups * self.c.in_features
        return 6 * alpha_proj_params + 7 * self.total_active_heads * self.head_dim

    def ltv_parameter_count(self) -> int:
        qkv_proj_params = self.total_active_heads * self.head_dim * self.c.in_features
        return sum(p.numel() for p in self.parameters()) - qkv_proj_params


class LtvCombinedHeadMajorQkvFilter(LtvCombinedQkvFilterBase):
    """Head-major layout: [head 0 values | head 0 logits | head 1 values | head 1 logits | ...]."""

    def __init__(self, n_head: int, n_kv_head: int, head_dim: int, r: int):
        super().__init__(n_head, n_kv_head, head_dim, r)
        self.logit_bias = nn.Parameter(torch.empty(self.total_active_heads, self.num_alpha_groups))

    def init_weights(self, alpha_mlp_bias_init: float, weight_s: float, bias_s: float, init_s: float):
        H, D, Da, C = self.total_active_heads, self.head_dim, self.num_alpha_groups, self.c.in_features
        w = self.c.weight
        vals = w.new_empty(H * D, C).uniform_(-weight_s, weight_s)      # Q, K, V value rows
        logits = w.new_empty(H * Da, C).uniform_(-weight_s, weight_s)   # decay-logit rows
        interleaved = torch.cat([vals.view(H, D, C), logits.view(H, Da, C)], dim=1).view(-1, C)
        assert w.requires_grad
        with torch.no_grad():
            w.copy_(interleaved)
        torch.nn.init.uniform_(self.logit_bias, alpha_mlp_bias_init - bias_s, alpha_mlp_bias_init + bias_s)
        init_weights_of_init(self.init_param, self.n_head, self.n_kv_head, init_s)


class LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter(LtvCombinedHeadMajorQkvFilter):
    """CUDA filter: tcgen05 projection into [B, F, T], then the scan.

    Decode steps (T == 1 with cached state, no autograd) take the one-launch `ltv_decode_step`
    path; bf16/fp16 sequences take `ltv_proj_scan` (projection and scan forward in one call);
    fp32 runs follow the reference's two-op composition.
    """

    use_decode_kernel: bool = True

    def forward(self, x, previous_values: LtvInitValues):
        B, T, _ = x.size()
        autocast_dtype = torch.get_autocast_dtype("cuda")
        run_ltv_in_fp32 = autocast_dtype == torch.float32 if CUDA_SUPPORTS_NATIVE_BF16 else True

        if (self.use_decode_kernel and T == 1 and not run_ltv_in_fp32 and x.is_cuda
                and not (torch.is_grad_enabled() and (x.requires_grad or self.c.weight.requires_grad))):
            return self._decode(x, previous_values)

        if not run_ltv_in_fp32:
            # projection + scan in one call (tensor-core accumulator straight into the recurrence);
            # outputs and gradients equal the two-op composition below bit for bit
            if previous_values.q is None:
                # training: one initial state [H, D] for every sequence (its gradient is summed over
                # the batch inside the scan backward instead of by an expand's backward)
                inits = self.init_param
            else:
                inits = resolve_inits_original_dtype(B, self.init_param, previous_values).to(dtype=x.dtype).contiguous()
            _, hq, hk, hv = _ops.ltv_proj_scan(x.contiguous(), self.c.weight, inits, self.logit_bias.contiguous(),
                                               self.n_head, self.n_kv_head, self.num_alpha_groups, self.r, True)
            return hq.transpose(1, 2), hk.transpose(1, 2), hv.transpose(1, 2)

        out_buf = _ops.fused_linear_transpose(x.float() if run_ltv_in_fp32 else x,
                                              self.c.weight.float() if run_ltv_in_fp32 else self.c.weight)
        kernel_combined = out_buf.transpose(1, 2)  # (B, T, F) view with strides (F*T, 1, T)
        inits = resolve_inits_original_dtype(B, self.init_param, previous_values).to(
            dtype=kernel_combined.dtype).contiguous()
        kernel_inits = inits.float() if run_ltv_in_fp32 else inits
        hq, hk, hv = _ops.ltv_cuda_fused_concat_head_major_register_cast_blelloch_scan(
            kernel_combined, kernel_inits, self.logit_bias.contiguous(), self.n_head, self.n_kv_head,
            self.num_alpha_groups, self.r, _SCAN_THREADS_FORWARD, _R_THREADS_FORWARD, _R_ITEMS_FORWARD,
            _SCAN_THREADS_BACKWARD, _R_THREADS_BACKWARD, _R_ITEMS_BACKWARD, True)
        if run_ltv_in_fp32:
            hq, hk, hv = hq.to(kernel_combined.dtype), hk.to(kernel_combined.dtype), hv.to(kernel_combined.dtype)
        return hq.transpose(1, 2), hk.transpose(1, 2), hv.transpose(1, 2)

    def forward_rotary_norm(self, x, previous_values: LtvInitValues, cos_sin):
        """forward() followed by the reference attention's prologue on q and k (nanochat/gpt.py:224-230:
        apply_rotary_emb, then norm): returns (q, k, v) [B, T, heads, D], q and k rotated and
        RMS-normalised, v the raw filter output. bf16 sequences on the one-kernel shapes run the
        prologue inside the filter's own kernels (the scan's epilogue forward, the checkpoint replay
        backward), so the extra pass over q and k disappears; results equal forward() followed by the
        fused rotary + norm operator bit for bit, which is what every other case runs."""
        cos, sin = cos_sin
        B, T, _ = x.size()
        autocast_dtype = torch.get_autocast_dtype("cuda")
        run_ltv_in_fp32 = autocast_dtype == torch.float32 if CUDA_SUPPORTS_NATIVE_BF16 else True
        decode = (self.use_decode_kernel and T == 1 and not run_ltv_in_fp32 and x.is_cuda
                  and not (torch.is_grad_enabled() and (x.requires_grad or self.c.weight.requires_grad)))
        if not run_ltv_in_fp32 and not decode:
            if previous_values.q is None:
                inits = self.init_param
            else:
                inits = resolve_inits_original_dtype(B, self.init_param, previous_values).to(dtype=x.dtype).contiguous()
            hq, hk, hv = _ops.ltv_proj_scan_rope_norm(x.contiguous(), self.c.weight, inits,
                                                      self.logit_bias.contiguous(), cos, sin, self.n_head,
                                                      self.n_kv_head, self.num_alpha_groups, self.r, True)
            return hq.transpose(1, 2), hk.transpose(1, 2), hv.transpose(1, 2)
        q, k, v = self.forward(x, previous_values)
        q, k = _ops.rotary_qk_norm(q, k, cos, sin)
        return q, k, v

    def _decode(self, x, previous_values: LtvInitValues):
        B = x.shape[0]
        pq = pk = pv = None
        if previous_values.q is not None:
            pq, pk, pv = (t.to(x.dtype) for t in (previous_values.q, previous_values.k, previous_values.v))
        q, k, v = _ops.ltv_decode_step(x, self.c.weight, self.logit_bias, pq, pk, pv, self.init_param, self.n_head,
                                       self.n_kv_head, self.num_alpha_groups, self.r, True)
        return q.view(B, 1, self.n_head, self.head_dim), k.view(B, 1, self.n_kv_head, self.head_dim), v.view(
            B, 1, self.n_kv_head, self.head_dim)
