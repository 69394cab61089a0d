"""Filter-state part of the decode KV cache (drop-in for the reference's last_qkv handling).

Mirrors nanochat/kv_cache.py:10-178 and the last_qkv methods of KVCache (:180-294): the
per-layer filter state lives in `last_qkv.{q,k,v}.special[layer]` ([L, B, heads, D]);
`update_last_qkv` stores the newest step, `has_last_qkv` says whether a layer has state,
`prefill` copies (and broadcasts over batch) another cache's state. For look-back layers
(`layer_specs` with a bounded chunking) each projection also keeps per layer a countdown to the
next chunk boundary and a deque of the warm-up states of upcoming chunks (`Layer`), maintained by
`lookback.advance_kv_cache`. The attention K/V tensors are outside the filtered-QKV path.
"""

from __future__ import annotations

import collections
from typing import List, Optional

import torch

_INVALID_COUNTDOWN = -1


class Layer:
    """Look-back bookkeeping of one layer: tokens to the next chunk boundary and warm-up states."""

    def __init__(self, countdown: int, d: collections.deque):
        self.countdown = countdown
        self.d = d

    def merge_from(self, other: "Layer") -> None:
        self.countdown = other.countdown
        for mine, theirs in zip(self.d, other.d, strict=True):
            mine[:, :, :] = theirs

    def is_initialized(self) -> bool:
        return self.countdown != _INVALID_COUNTDOWN


class LookBack:
    """`special` holds the state of every filtered layer: [L, B, heads, D]; `layers` their bookkeeping."""

    def __init__(self, special: torch.Tensor, layers: Optional[List[Layer]] = None):
        self.special = special
        self.layers = layers if layers is not None else [
            Layer(_INVALID_COUNTDOWN, collections.deque(maxlen=0)) for _ in range(len(special))]
        assert len(self.layers) == len(special)

    def merge_from(self, other: "LookBack") -> None:
        self.special[:, :, :, :] = other.special
        for mine, theirs in zip(self.layers, other.layers):
            mine.merge_from(theirs)


def _empty_lookback(shape, dtype, device, mls: List[int]) -> LookBack:
    """Uninitialised state for len(mls) layers; layer i's deque holds mls[i] states."""
    assert shape[0] == len(mls)
    special = torch.empty(shape, dtype=dtype, device=device)
    layers = [Layer(_INVALID_COUNTDOWN, collections.deque(
        [torch.empty(shape[1:], dtype=dtype, device=device) for _ in range(ml)], maxlen=ml)) for ml in mls]
    return LookBack(special, layers)


class LastQkv:
    def __init__(self, q: Optional[LookBack], k: Optional[LookBack], v: Optional[LookBack], m: int):
        self.q, self.k, self.v, self.m = q, k, v, m

    def merge_from(self, other: "LastQkv") -> None:
        for mine, theirs in ((self.q, other.q), (self.k, other.k), (self.v, other.v)):
            if theirs is None:
                assert mine is None
            else:
                mine.merge_from(theirs)
                assert other.m == len(theirs.special)
        self.m = other.m


class TypeDevice:
    def __init__(self, dtype, device):
        self.dtype = dtype
        self.device = device


def make_empty_last_qkv_like_specials(last_q_shape, last_k_v_shape, q: Optional[TypeDevice],
                                      k: Optional[TypeDevice], v: Optional[TypeDevice], mls: List[int]) -> LastQkv:
    def mk(td, shape):
        return None if td is None else _empty_lookback(shape, td.dtype, td.device, mls)

    return LastQkv(mk(q, last_q_shape), mk(k, last_k_v_shape), mk(v, last_k_v_shape), 0)


class KVCache:
    def __init__(self, batch_size: int, num_q_heads: int, num_kv_heads: int, seq_len: int, head_dim: int,
                 num_layers: int, layer_specs=None):
        """`layer_specs`: one ChunksAndHistory per filtered layer (reference signature); None means
        `num_layers` unbounded (plain-scan) layers."""
        from .lookback import UNBOUNDED_LAYER_SPEC

        assert num_q_heads % num_kv_heads == 0
        if layer_specs is None:
            layer_specs = [UNBOUNDED_LAYER_SPEC] * num_layers
        self.pos = 0
        self.last_qkv: Optional[LastQkv] = None
        self.last_q_shape = (len(layer_specs), batch_size, num_q_heads, head_dim)
        self.last_k_v_shape = (len(layer_specs), batch_size, num_kv_heads, head_dim)
        self.layer_specs = list(layer_specs)

    def num_ltv_layers(self) -> int:
        return len(self.layer_specs)

    def get_pos(self) -> int:
        return self.pos

    def update_last_qkv(self, layer_idx: int, q: Optional[torch.Tensor], k: Optional[torch.Tensor],
                        v: Optional[torch.Tensor]) -> None:
        lq = self.last_qkv
        if lq is None:
            assert layer_idx == 0

            def td(t):
                return None if t is None else TypeDevice(t.dtype, t.device)

            lq = self.last_qkv = make_empty_last_qkv_like_specials(
                self.last_q_shape, self.last_k_v_shape, td(q), td(k), td(v), [0] * self.num_ltv_layers())
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
        o = other.last_qkv
        if o is None:
            self.last_qkv = None
        else:
            def like(lb, shape):
                if lb is None:
                    return None
                return _empty_lookback(shape, lb.special.dtype, lb.special.device, [len(l.d) for l in lb.layers])

            self.last_qkv = LastQkv(like(o.q, self.last_q_shape), like(o.k, self.last_k_v_shape),
                                    like(o.v, self.last_k_v_shape), 0)
            self.last_qkv.merge_from(o)
        self.pos = other.pos
