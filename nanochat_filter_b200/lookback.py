"""Look-back (chunk-restarting) filtered-QKV: chunk spec, filter classes, computer module.

ChunksAndHistory / UNBOUNDED_P                        nanochat/gpt_config.py:9-45
LtvLookBackHeadMajorQkvFilter                         nanochat/ltv_look_back_head_major_qkv_filter_base.py:12-87
LtvLookBackFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter
                                                      nanochat/ltv_look_back_fused_concat_head_major_register_cast_blelloch_scan_qkv_filter.py:45-99
LtvLookBackFusedConcatHeadMajorRegisterCastSequentialScanQkvFilter
                                                      nanochat/ltv_look_back_fused_concat_head_major_register_cast_sequential_scan_qkv_filter.py:40-90
advance_kv_cache / LtvLookBackQkvComputerModule       nanochat/ltv_look_back_qkv_computer_module.py:15-209

A layer's outputs at token t come from the recurrence restarted from the initial state K - 1
tokens before t's chunk (chunks [0, P), then every Q tokens). In decode, the cache keeps for
each layer the current chunk's state (`special`), a countdown to the next chunk boundary, and a
deque of the warm-up states of the chunks that start within the next K - 1 tokens; advance_kv_cache
feeds new tokens through those recurrences (full, unchunked recurrences over the new tokens) so
that token-by-token decoding equals the chunked batch forward. The filters' default operators are
this package's CUDA operators; any callables with the reference's signatures can be passed.
"""

from __future__ import annotations

import collections
from abc import ABC, abstractmethod
from typing import Callable, Optional

import torch
import torch.nn as nn

from . import ops as _ops
from .filters import LtvCombinedHeadMajorQkvFilter
from .util import (
    _R_ITEMS_BACKWARD,
    _R_ITEMS_FORWARD,
    _R_THREADS_BACKWARD,
    _R_THREADS_FORWARD,
    _SCAN_THREADS_BACKWARD,
    _SCAN_THREADS_FORWARD,
    should_run_ltv_in_fp32,
)

UNBOUNDED_P = 2_147_483_647


class ChunksAndHistory:
    """Chunking of one layer: first chunk p tokens, then chunks of q; k - 1 tokens of warm-up."""

    def __init__(self, p: int, q: int, k: int):
        assert p >= 0
        assert q >= 1
        assert k >= 1
        self.p, self.q, self.k = p, q, k

    def deque_size(self) -> int:
        """Number of chunk starts whose warm-up windows can be open at once."""
        return 0 if self.is_unbounded() else (self.k - 1 + self.q - 1) // self.q

    def is_unbounded(self) -> bool:
        return self.p == UNBOUNDED_P

    def to_dict(self):
        return {"p": self.p, "q": self.q, "k": self.k}

    def to_comma_separated_str(self) -> str:
        return f"{self.p},{self.q},{self.k}"

    def __str__(self):
        return self.to_comma_separated_str()

    def __repr__(self):
        return f"ChunksAndHistory(p={self.p}, q={self.q}, k={self.k})"

    @classmethod
    def from_dict(cls, d):
        return cls(**d)


UNBOUNDED_LAYER_SPEC = ChunksAndHistory(p=UNBOUNDED_P, q=1, k=1)


class LtvLookBackHeadMajorQkvFilter(LtvCombinedHeadMajorQkvFilter, ABC):
    """Combined head-major projection followed by the look-back scan of `layer_spec`."""

    def __init__(self, n_head: int, n_kv_head: int, head_dim: int, r: int, layer_spec: ChunksAndHistory):
        super().__init__(n_head, n_kv_head, head_dim, r)
        self.layer_spec = layer_spec

    @abstractmethod
    def _project(self, x: torch.Tensor) -> torch.Tensor:
        """x [B, T, C] -> combined [B, T, F] (any strides the scan accepts)."""

    @abstractmethod
    def _look_back_op(self, combined, inits, logit_bias, full_recurrence: bool):
        """-> q, k, v as [B, T, heads, D]."""

    def forward(self, x: torch.Tensor, resolved_inits: torch.Tensor, full_recurrence: bool):
        run_ltv_in_fp32 = should_run_ltv_in_fp32(x.device.type)
        combined = self._project(x.float() if run_ltv_in_fp32 else x)
        logit_bias = self.logit_bias.contiguous()
        inits = resolved_inits.to(dtype=combined.dtype).contiguous()
        hq, hk, hv = self._look_back_op(combined, inits.float() if run_ltv_in_fp32 else inits,
                                        logit_bias.float() if run_ltv_in_fp32 else logit_bias, full_recurrence)
        if run_ltv_in_fp32:
            hq, hk, hv = hq.to(combined.dtype), hk.to(combined.dtype), hv.to(combined.dtype)
        return hq, hk, hv

    def _pqk(self, full_recurrence: bool):
        if full_recurrence:
            return UNBOUNDED_P, 1, 1
        return self.layer_spec.p, self.layer_spec.q, self.layer_spec.k


def _default_transpose_op(x, weight):
    return _ops.fused_linear_transpose(x, weight)


def _default_blelloch_look_back_op(*args):
    return torch.ops.nanochat_cuda.ltv_look_back_fused_concat_head_major_register_cast_blelloch_scan_cuda_op(*args)


def _default_sequential_look_back_op(*args):
    return torch.ops.nanochat_cuda.ltv_look_back_fused_concat_head_major_register_cast_sequential_scan_cuda_op(*args)


class LtvLookBackFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter(LtvLookBackHeadMajorQkvFilter):
    """Projection into [B, F, T] (tcgen05 GEMM), scanned through its [B, T, F] transposed view."""

    def __init__(self, n_head: int, n_kv_head: int, head_dim: int, r: int, layer_spec: ChunksAndHistory,
                 transpose_op: Optional[Callable] = None, look_back_op: Optional[Callable] = None):
        super().__init__(n_head, n_kv_head, head_dim, r, layer_spec)
        self.transpose_op = transpose_op or _default_transpose_op
        self.look_back_op = look_back_op or _default_blelloch_look_back_op

    def _project(self, x):
        f32 = x.dtype == torch.float32
        # decode slices x[:, t:t+1] of a batch are strided; the projection operator takes contiguous x
        x = x.contiguous()
        out_buf = self.transpose_op(x.float() if f32 else x, self.c.weight.float() if f32 else self.c.weight)
        return out_buf.transpose(1, 2)

    def _look_back_op(self, combined, inits, logit_bias, full_recurrence):
        P, Q, K = self._pqk(full_recurrence)
        hq, hk, hv = self.look_back_op(combined, inits, logit_bias, self.n_head, self.n_kv_head, self.num_alpha_groups,
                                       self.r, P, Q, K, _SCAN_THREADS_FORWARD, _R_THREADS_FORWARD, _R_ITEMS_FORWARD,
                                       _SCAN_THREADS_BACKWARD, _R_THREADS_BACKWARD, _R_ITEMS_BACKWARD, True)
        return hq.transpose(1, 2), hk.transpose(1, 2), hv.transpose(1, 2)


class LtvLookBackFusedConcatHeadMajorRegisterCastSequentialScanQkvFilter(LtvLookBackHeadMajorQkvFilter):
    """Plain nn.Linear projection ([B, T, F] contiguous) and the look-back scan."""

    def __init__(self, n_head: int, n_kv_head: int, head_dim: int, r: int, layer_spec: ChunksAndHistory,
                 sequential_look_back_op: Optional[Callable] = None):
        super().__init__(n_head, n_kv_head, head_dim, r, layer_spec)
        self.sequential_look_back_op = sequential_look_back_op or _default_sequential_look_back_op

    def _project(self, x):
        return self.c(x).contiguous()

    def _look_back_op(self, combined, inits, logit_bias, full_recurrence):
        P, Q, K = self._pqk(full_recurrence)
        hq, hk, hv = self.sequential_look_back_op(combined, inits, logit_bias, self.n_head, self.n_kv_head,
                                                  self.num_alpha_groups, self.r, P, Q, K, _R_THREADS_FORWARD,
                                                  _R_ITEMS_FORWARD, _R_THREADS_BACKWARD, _R_ITEMS_BACKWARD, True)
        return hq.transpose(1, 2), hk.transpose(1, 2), hv.transpose(1, 2)


def advance_kv_cache(x: torch.Tensor, layer_idx: int, ltv_filter: LtvLookBackHeadMajorQkvFilter,
                     resolved_inits: torch.Tensor, kv_cache):
    """Feeds x [B, n, C] through layer `layer_idx`'s look-back state in the cache; returns q, k, v
    [B, n, heads, D] equal to the chunked forward over the whole sequence so far (reference
    nanochat/ltv_look_back_qkv_computer_module.py:15-164)."""
    from .kv_cache import TypeDevice, make_empty_last_qkv_like_specials

    lq = kv_cache.last_qkv
    if lq is None:
        assert not layer_idx
        td = TypeDevice(x.dtype, x.device)
        lq = kv_cache.last_qkv = make_empty_last_qkv_like_specials(
            kv_cache.last_q_shape, kv_cache.last_k_v_shape, td, td, td,
            mls=[spec.deque_size() for spec in kv_cache.layer_specs])
    else:
        assert lq.q and lq.k and lq.v
    spec = kv_cache.layer_specs[layer_idx]
    # initial state per projection: resolved_inits [B, H, D] split along the head dimension
    q0, k0, v0 = torch.split(resolved_inits, [ltv_filter.n_head, ltv_filter.n_kv_head, ltv_filter.n_kv_head], dim=1)
    for proj, x0 in ((lq.q, q0), (lq.k, k0), (lq.v, v0)):
        layer = proj.layers[layer_idx]
        if not layer.is_initialized():
            proj.special[layer_idx, :, :, :] = x0
            layer.countdown = spec.p or spec.q
            ml = spec.deque_size()
            layer.d = collections.deque(maxlen=0) if spec.is_unbounded() else collections.deque([x0] * ml, maxlen=ml)
    ql, kl, vl = (p.layers[layer_idx] for p in (lq.q, lq.k, lq.v))
    n = x.shape[1]
    start = 0
    result = []
    while start < n:
        al = min(ql.countdown, n - start)  # tokens until the next chunk boundary (q, k, v move together)
        inits_cat = torch.cat([lq.q.special[layer_idx], lq.k.special[layer_idx], lq.v.special[layer_idx]], dim=1)
        a_q, a_k, a_v = ltv_filter.forward(x=x[:, start:start + al, :], resolved_inits=inits_cat,
                                           full_recurrence=True)
        result.append((a_q, a_k, a_v))
        (countdown,) = {ql.countdown, kl.countdown, vl.countdown}
        for i, (dq, dk, dv) in enumerate(zip(ql.d, kl.d, vl.d, strict=True)):
            # deque entry i is the warm-up state of the chunk starting i boundaries after the next
            offset_i = ql.countdown + i * spec.q - spec.k + 1
            kt = x[:, start + max(offset_i, 0):start + al, :]
            if kt.shape[1]:
                q, k, v = ltv_filter.forward(x=kt, resolved_inits=torch.cat([dq, dk, dv], dim=1), full_recurrence=True)
                ql.d[i], kl.d[i], vl.d[i] = q[:, -1], k[:, -1], v[:, -1]
        if al == ql.countdown:
            # a chunk boundary: the oldest warm-up state becomes the new chunk's state
            new_q = ql.d[0] if ql.d else q0
            new_k = kl.d[0] if kl.d else k0
            new_v = vl.d[0] if vl.d else v0
            ql.d.append(q0)
            kl.d.append(k0)
            vl.d.append(v0)
            lq.q.special[layer_idx, :, :, :] = new_q
            lq.k.special[layer_idx, :, :, :] = new_k
            lq.v.special[layer_idx, :, :, :] = new_v
            ql.countdown = kl.countdown = vl.countdown = spec.q
        else:
            ql.countdown = kl.countdown = vl.countdown = countdown - al
            lq.q.special[layer_idx, :, :, :] = a_q[:, -1]
            lq.k.special[layer_idx, :, :, :] = a_k[:, -1]
            lq.v.special[layer_idx, :, :, :] = a_v[:, -1]
        start += al
    assert lq.m == layer_idx or lq.m == kv_cache.num_ltv_layers()
    if lq.m != kv_cache.num_ltv_layers():
        lq.m += 1
    B, D = x.shape[0], ltv_filter.head_dim
    kw = dict(dtype=x.dtype, device=x.device)
    parts = ([torch.empty(B, 0, ltv_filter.n_head, D, **kw)], [torch.empty(B, 0, ltv_filter.n_kv_head, D, **kw)],
             [torch.empty(B, 0, ltv_filter.n_kv_head, D, **kw)])
    for q, k, v in result:
        parts[0].append(q)
        parts[1].append(k)
        parts[2].append(v)
    return torch.cat(parts[0], dim=1), torch.cat(parts[1], dim=1), torch.cat(parts[2], dim=1)


class LtvLookBackQkvComputerModule(nn.Module):
    """Chunked forward without a cache; cache advance (advance_kv_cache) with one."""

    def __init__(self, layer_idx: int, ltv_filter: LtvLookBackHeadMajorQkvFilter):
        super().__init__()
        self.ltv_filter = ltv_filter
        self.advance_last_qkv = lambda kv_cache, resolved_inits, x: advance_kv_cache(
            x, layer_idx, self.ltv_filter, resolved_inits, kv_cache)

    def forward(self, x, kv_cache=None):
        B = x.size(0)
        resolved_inits = self.ltv_filter.init_param.unsqueeze(0).expand(B, -1, -1)
        if kv_cache is not None:
            return self.advance_last_qkv(kv_cache, resolved_inits, x)
        return self.ltv_filter(x, resolved_inits, full_recurrence=False)

    def init_weights(self, alpha_mlp_bias_init: float, weight_s: float, bias_s: float, init_s: float):
        self.ltv_filter.init_weights(alpha_mlp_bias_init=alpha_mlp_bias_init, weight_s=weight_s, bias_s=bias_s,
                                     init_s=init_s)

    def get_matrix_linear_params(self):
        return self.ltv_filter.get_matrix_linear_params()

    def estimate_flops(self, sequence_len: int) -> int:
        return self.ltv_filter.estimate_flops(sequence_len)

    def ltv_parameter_count(self) -> int:
        return self.ltv_filter.ltv_parameter_count()
