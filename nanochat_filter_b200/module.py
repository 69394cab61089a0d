"""LtvCombinedQkvComputerModule: the attention layer's QKV computer (drop-in).

Mirrors nanochat/ltv_combined_qkv_computer_module.py:12-60: picks the start state (the
cached last q/k/v of this layer during decode, else the filter's learnable init_param), runs
the filter and stores the last time step back into the cache.
"""

from __future__ import annotations

from typing import Optional

import torch.nn as nn

from . import ops as _ops
from .filters import LtvCombinedQkvFilterBase
from .kv_cache import KVCache
from .util import LtvInitValues


class LtvCombinedQkvComputerModule(nn.Module):
    def __init__(self, layer_idx: int, ltv_filter: LtvCombinedQkvFilterBase):
        super().__init__()
        self.ltv_filter = ltv_filter
        self.layer_idx = layer_idx

    def forward(self, x, kv_cache: Optional[KVCache]):
        if kv_cache and kv_cache.has_last_qkv(self.layer_idx):
            lq = kv_cache.last_qkv
            previous_values = LtvInitValues(q=lq.q.special[self.layer_idx], k=lq.k.special[self.layer_idx],
                                            v=lq.v.special[self.layer_idx])
        else:
            previous_values = LtvInitValues(None, None, None)
        q, k, v = self.ltv_filter(x, previous_values)
        if kv_cache:
            kv_cache.update_last_qkv(self.layer_idx, q[:, -1, :, :], k[:, -1, :, :], v[:, -1, :, :])
        return q, k, v

    def forward_rotary_norm(self, x, kv_cache: Optional[KVCache], cos_sin):
        """forward() followed by the attention's prologue on q and k (nanochat/gpt.py:224-230:
        apply_rotary_emb with `cos_sin`, then norm); v as forward() returns it. Without a KV cache
        (training) filters that have `forward_rotary_norm` fold the prologue into their kernels; with a
        cache the raw last states go into it as forward() stores them, and the prologue runs as the
        fused rotary + norm operator."""
        fused = getattr(self.ltv_filter, "forward_rotary_norm", None)
        if not kv_cache and fused is not None:
            return fused(x, LtvInitValues(None, None, None), cos_sin)
        q, k, v = self.forward(x, kv_cache)
        q, k = _ops.rotary_qk_norm(q, k, cos_sin[0], cos_sin[1])
        return q, k, v

    def init_weights(self, alpha_mlp_bias_init: float, weight_s: float, bias_s: float, init_s: float):
        self.ltv_filter.init_weights(alpha_mlp_bias_init=alpha_mlp_bias_init, weight_s=weight_s, bias_s=bias_s,
                                     init_s=init_s)

    def get_matrix_linear_params(self):
        return self.ltv_filter.get_matrix_linear_params()

    def estimate_flops(self, sequence_len: int) -> int:
        return self.ltv_filter.estimate_flops(sequence_len)

    def ltv_parameter_count(self) -> int:
        return self.ltv_filter.ltv_parameter_count()
