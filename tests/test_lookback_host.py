"""Host logic of the look-back path (no GPU): the decode cache advance and the filter classes.

Ports the reference's exhaustive cache test (tests/test_look_back_advance_kv_cache_exhaustive.py:
all token-count sequences of N steps with 0..A-1 tokens each, several (p, q, k), both filter
variants): feeding the tokens all at once, step by step, and step by step through a prefilled copy
of the cache give the same q, k, v. Beyond the reference test, all three also equal the chunked
forward over the whole sequence. The filters get CPU stand-ins for the projection and the scan
(the operators' CUDA implementations are covered by the GPU tests): a matmul and a direct loop
over the chunking rule of nanochat/ops/ltv_reference_ops.py:37-124.
"""

from __future__ import annotations

import itertools

import pytest
import torch

import nanochat_filter_b200 as nf


def cpu_transpose(x, w):
    return torch.matmul(x, w.T).transpose(1, 2).contiguous()


def cpu_look_back(combined, inits, logit_bias, NH, NKVH, Da, r, P, Q, K, *tuning_and_flag):
    use_sigmoid = tuning_and_flag[-1]
    B, T, _ = combined.shape
    H, D = NH + 2 * NKVH, Da * r
    outs = [torch.empty(B, n, T, D, dtype=combined.dtype) for n in (NH, NKVH, NKVH)]
    chunks = [(0, min(P, T))] if T > P else [(0, T)]
    if T > P:
        s = P
        while s < T:
            chunks.append((s, min(s + Q, T)))
            s += Q
    for b in range(B):
        for h in range(H):
            which, hl = (0, h) if h < NH else ((1, h - NH) if h < NH + NKVH else (2, h - NH - NKVH))
            col = h * (D + Da)
            for t0, t1 in chunks:
                st = inits[b, h].float().clone()
                for t in range(max(0, t0 - (K - 1)), t1):
                    raw = combined[b, t, col + D:col + D + Da].float() + logit_bias[h]
                    a = (torch.sigmoid(raw) if use_sigmoid else raw).repeat_interleave(r)
                    st = (1 - a) * st + a * combined[b, t, col:col + D].float()
                    if t >= t0:
                        outs[which][b, hl, t] = st.to(combined.dtype)
    return tuple(outs)


def make_blelloch(nh, nkvh, hd, r, spec):
    return nf.LtvLookBackFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter(
        nh, nkvh, hd, r, spec, transpose_op=cpu_transpose, look_back_op=cpu_look_back)


def make_sequential(nh, nkvh, hd, r, spec):
    return nf.LtvLookBackFusedConcatHeadMajorRegisterCastSequentialScanQkvFilter(
        nh, nkvh, hd, r, spec, sequential_look_back_op=cpu_look_back)


def new_cache(spec, total):
    return nf.KVCache(batch_size=1, num_q_heads=1, num_kv_heads=1, seq_len=max(1, total) + 10, head_dim=2,
                      num_layers=1, layer_specs=[spec])


@pytest.mark.parametrize("make", [make_blelloch, make_sequential], ids=["blelloch", "sequential"])
@pytest.mark.parametrize("p,q,k", [(3, 2, 2), (5, 3, 2), (4, 2, 3), (1, 1, 1), (10, 2, 5)])
@pytest.mark.parametrize("N,A", [(1, 3), (2, 3), (3, 2), (3, 3)])
def test_advance_kv_cache_exhaustive(make, p, q, k, N, A):
    spec = nf.ChunksAndHistory(p=p, q=q, k=k)
    filt = make(1, 1, 2, 1, spec)
    with torch.no_grad():
        filt.c.weight.copy_(torch.linspace(-1, 1, filt.c.weight.numel()).view_as(filt.c.weight))
        filt.logit_bias.fill_(0.0)
        filt.init_param.fill_(0.0)
    for counts in itertools.product(range(A), repeat=N):
        total = sum(counts)
        torch.manual_seed(42)
        x = torch.randn(1, total, 2)
        inits = filt.init_param.unsqueeze(0).expand(1, -1, -1)
        with torch.no_grad():
            all_at_once = nf.advance_kv_cache(x, 0, filt, inits, new_cache(spec, total))
            step_cache, prev = new_cache(spec, total), new_cache(spec, total)
            stepped, prefilled = [], []
            start = 0
            for n in counts:
                xs = x[:, start:start + n]
                start += n
                stepped.append(nf.advance_kv_cache(xs, 0, filt, inits, step_cache))
                prefilled.append(nf.advance_kv_cache(xs, 0, filt, inits, prev))
                fresh = new_cache(spec, total)
                fresh.prefill(prev)
                prev = fresh
            batch = filt(x, inits, full_recurrence=False)
        for i in range(3):
            torch.testing.assert_close(torch.cat([s[i] for s in stepped], dim=1), all_at_once[i])
            torch.testing.assert_close(torch.cat([s[i] for s in prefilled], dim=1), all_at_once[i])
            torch.testing.assert_close(batch[i], all_at_once[i])


def test_computer_module_and_chunk_spec():
    spec = nf.ChunksAndHistory(p=4, q=3, k=2)
    assert spec.deque_size() == 1 and not spec.is_unbounded() and str(spec) == "4,3,2"
    assert nf.ChunksAndHistory.from_dict(spec.to_dict()).to_dict() == {"p": 4, "q": 3, "k": 2}
    assert nf.UNBOUNDED_LAYER_SPEC.is_unbounded() and nf.UNBOUNDED_LAYER_SPEC.deque_size() == 0
    filt = make_blelloch(2, 1, 4, 2, spec)
    filt.init_weights(2.0, 0.1, 0.5, 0.5)
    mod = nf.LtvLookBackQkvComputerModule(0, filt)
    x = torch.randn(2, 9, 8)
    with torch.no_grad():
        q, k, v = mod(x)
        cache = nf.KVCache(2, 2, 1, 16, 4, num_layers=1, layer_specs=[spec])
        qs = [mod(x[:, t:t + 1], cache)[0] for t in range(9)]
    assert q.shape == (2, 9, 2, 4) and k.shape == (2, 9, 1, 4)
    torch.testing.assert_close(torch.cat(qs, dim=1), q)
    assert mod.get_matrix_linear_params()[0][0] is filt.c.weight
