"""Filter-state part of the decode KV cache (drop-in for the reference's last_qkv handling).

Mirrors nanochat/kv_cache.py:87-178 and the last_qkv methods of KVCache (:180-294): the
per-layer filter state lives in `last_qkv.{q,k,v}.special[layer]` ([L, B, heads, D]),
`update_last_qkv` stores the newest step, `has_last_qkv` says whether a layer has state,
`prefill` copies (and broadcasts over batch) another cache's state. The attention K/V tensors
and the look-back deques of the reference's cache are outside the filtered-QKV path.
"""

from __future__ import annotations

from typing import Optional

import torch


class LookBack:
    """`special` holds the state of every filtered layer: [L, B, heads, D]."""

    def __init__(self, special: torch.Tensor):
        self.special = special

    def merge_from(self, other: "LookBack") -> None:
        self.special[:, :, :, :] = other.special


class LastQkv:
    def __init__(self, q: Optional[LookBack], k: Optional[LookBack], v: Optional[LookBack], m: int):
        self.q, self.k, self.v, self.m = q, k, v, m


class KVCache:
    def __init__(self, batch_size: int, num_q_heads: int, num_kv_heads: int, seq_len: int, head_dim: int,
                 num_layers: int, num_ltv_layers: Optional[int] = None):
        assert num_q_heads % num_kv_heads == 0
        n_ltv = num_layers if num_ltv_layers is None else num_ltv_layers
        self.pos = 0
        self.last_qkv: Optional[LastQkv] = None
        self.last_q_shape = (n_ltv, batch_size, num_q_heads, head_dim)
        self.last_k_v_shape = (n_ltv, batch_size, num_kv_heads, head_dim)
        self._num_ltv_layers = n_ltv

    def num_ltv_layers(self) -> int:
        return self._num_ltv_layers

    def get_pos(self) -> int:
        return self.pos

    def update_last_qkv(self, layer_idx: int, q: Optional[torch.Tensor], k: Optional[torch.Tensor],
                        v: Optional[torch.Tensor]) -> None:
        lq = self.last_qkv
        if lq is None:
            assert layer_idx == 0

            def mk(t, shape):
                return None if t is None else LookBack(torch.empty(shape, dtype=t.dtype, device=t.device))

            lq = self.last_qkv = LastQkv(mk(q, self.last_q_shape), mk(k, self.last_k_v_shape),
                                         mk(v, self.last_k_v_shape), 0)
        assert lq.m == layer_idx or lq.m == self.num_ltv_layers()
        for t, lb, shape in ((q, lq.q, self.last_q_shape), (k, lq.k, self.last_k_v_shape),
                             (v, lq.v, self.last_k_v_shape)):
            assert (t is None) == (lb is None)
            if t is not None:
                assert tuple(t.shape) == tuple(shape[1:])
                lb.special[layer_idx, :, :, :] = t
        if lq.m != self.num_ltv_layers():
            lq.m += 1

    def has_last_qkv(self, layer_idx: int) -> bool:
        lq = self.last_qkv
        return bool(lq) and layer_idx < lq.m

    def prefill(self, other: "KVCache") -> None:
        """Copies another cache's filter state, broadcasting a batch-1 state over this batch."""
        if other.last_qkv is None:
            self.last_qkv = None
        else:
            o = other.last_qkv

            def cp(lb, shape):
                if lb is None:
                    return None
                out = torch.empty(shape, dtype=lb.special.dtype, device=lb.special.device)
                out[:, :, :, :] = lb.special
                return LookBack(out)

            self.last_qkv = LastQkv(cp(o.q, self.last_q_shape), cp(o.k, self.last_k_v_shape),
                                    cp(o.v, self.last_k_v_shape), o.m)
        self.pos = other.pos
