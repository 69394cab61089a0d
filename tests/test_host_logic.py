"""Host-side behaviour that needs no GPU: operator schemas and fake kernels (torch.compile
tracing), module API and parameter layout, dtype policy, KV-cache state handling, and the
absence of any CPU fallback."""

from __future__ import annotations

import pytest
import torch

import nanochat_filter_b200 as nf
from nanochat_filter_b200 import filters, util

OPS = torch.ops.nanochat_cuda


def test_operator_schemas_match_reference_names():
    names = {
        "ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_op",
        "ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_forward_kernel",
        "ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_backward_kernel",
        "fused_linear_transpose",
        "fused_linear_transpose_cuda_op",
        "fused_linear_transpose_backward_kernel",
        "ltv_decode_step",
    }
    for n in names:
        assert hasattr(OPS, n), n
    schema = str(OPS.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_op.default._schema)
    assert "int scan_threads_forward" in schema and "bool use_sigmoid" in schema
    schema = str(OPS.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_backward_kernel.default._schema)
    assert "Tensor(a!) grad_combined" in schema and "Tensor(c!) grad_logit_bias" in schema


def test_fake_kernels_give_reference_shapes():
    B, T, C, NH, NKVH, D, r = 3, 17, 256, 2, 1, 128, 64
    Da = D // r
    H = NH + 2 * NKVH
    F = H * (D + Da)
    x = torch.empty(B, T, C, device="meta")
    w = torch.empty(F, C, device="meta")
    out = OPS.fused_linear_transpose_cuda_op(x, w)
    assert out.shape == (B, F, T)
    comb = out.transpose(1, 2)
    q, k, v = OPS.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_op(
        comb, torch.empty(B, H, D, device="meta"), torch.empty(H, Da, device="meta"), NH, NKVH, Da, r, 8, 8, 4,
        32, 2, 8, True)
    assert q.shape == (B, NH, T, D) and k.shape == (B, NKVH, T, D) and v.shape == (B, NKVH, T, D)
    sq, sk, sv = OPS.ltv_decode_step(torch.empty(B, C, device="meta"), w, torch.empty(H, Da, device="meta"), None,
                                     None, None, torch.empty(H, D, device="meta"), NH, NKVH, Da, r, True)
    assert sq.shape == (B, NH, D) and sk.shape == (B, NKVH, D)


LB_OPS = [f"ltv_look_back_fused_concat_head_major_register_cast_{kind}_scan_cuda_{part}"
          for kind in ("blelloch", "sequential") for part in ("op", "forward_kernel", "backward_kernel")]


def test_lookback_operator_schemas_match_reference():
    """The six look-back operators with the reference's argument lists (ltv_cuda_ops.py:172-240)."""
    for n in LB_OPS:
        assert hasattr(OPS, n), n
    s = str(getattr(OPS, LB_OPS[0]).default._schema)
    assert "int P, int Q, int K, int scan_threads_forward" in s and s.endswith("-> (Tensor, Tensor, Tensor)")
    s = str(getattr(OPS, LB_OPS[1]).default._schema)
    assert "Tensor(a!) out_q" in s and "int B, int T, int NH" in s
    s = str(getattr(OPS, LB_OPS[3]).default._schema)
    assert "int P, int Q, int K, int r_threads_forward, int r_items_forward, int r_threads_backward" in s
    s = str(getattr(OPS, LB_OPS[5]).default._schema)
    assert "Tensor(c!) grad_logit_bias" in s and "int r_threads_backward, int r_items_backward, bool use_sigmoid" in s


def test_lookback_and_proj_scan_fake_shapes():
    B, T, NH, NKVH, D = 2, 9, 1, 1, 32
    comb = torch.empty(B, T, 3 * (D + 1), device="meta")
    inits, bias = torch.empty(B, 3, D, device="meta"), torch.empty(3, 1, device="meta")
    for kind, tune in (("blelloch", (8, 8, 4, 32, 2, 8)), ("sequential", (2, 4, 2, 8))):
        out = getattr(OPS, f"ltv_look_back_fused_concat_head_major_register_cast_{kind}_scan_cuda_op")(
            comb, inits, bias, NH, NKVH, 1, D, 4, 3, 2, *tune, True)
        assert [tuple(t.shape) for t in out] == [(B, NH, T, D), (B, NKVH, T, D), (B, NKVH, T, D)]
    x, w = torch.empty(B, T, 64, device="meta"), torch.empty(3 * (D + 1), 64, device="meta")
    comb2, q, k, v, ckpt = OPS.ltv_proj_scan_cuda_op(x, w, inits, bias, NH, NKVH, 1, D, True)
    assert tuple(comb2.shape) == (B, 3 * (D + 1), T) and tuple(q.shape) == (B, NH, T, D)
    assert tuple(ckpt.shape) == (0,) and ckpt.dtype == torch.float32  # fp32 and D = 32: no checkpoints
    xb = torch.empty(300, 64, 64, device="meta", dtype=torch.bfloat16)
    wb = torch.empty(129, 64, device="meta", dtype=torch.bfloat16)
    ib, bb = torch.empty(300, 1, 128, device="meta", dtype=torch.bfloat16), torch.empty(1, 1, device="meta")
    ckpt = OPS.ltv_proj_scan_cuda_op(xb, wb, ib, bb, 1, 0, 1, 128, True)[4]
    assert tuple(ckpt.shape) == (300, 1, 2, 128)  # 300 rows of 64 tokens: states at the 32-token chunk starts


def test_lookback_no_cpu_fallback():
    comb = torch.randn(1, 8, 3 * 3)
    with pytest.raises(NotImplementedError):
        OPS.ltv_look_back_fused_concat_head_major_register_cast_sequential_scan_cuda_op(
            comb, torch.randn(1, 3, 2), torch.randn(3, 1), 1, 1, 1, 2, 4, 3, 2, 2, 4, 2, 8, True)


def test_rotary_qk_norm_op_schema_and_fake():
    s = str(OPS.ltv_rotary_qk_norm.default._schema)
    assert s.startswith("nanochat_cuda::ltv_rotary_qk_norm(Tensor q, Tensor k, Tensor cos, Tensor sin)")
    q = torch.empty(2, 5, 3, 8, device="meta")
    k = torch.empty(2, 5, 1, 8, device="meta")
    oq, ok = OPS.ltv_rotary_qk_norm(q, k, torch.empty(1, 5, 1, 4, device="meta"), torch.empty(1, 5, 1, 4, device="meta"))
    assert tuple(oq.shape) == (2, 5, 3, 8) and oq.transpose(1, 2).is_contiguous()
    with pytest.raises(NotImplementedError):
        OPS.ltv_rotary_qk_norm(torch.randn(1, 2, 1, 4), torch.randn(1, 2, 1, 4), torch.randn(2, 2), torch.randn(2, 2))


def test_filter_on_meta_device_traces_shapes():
    f = nf.LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter(6, 6, 128, 128).to("meta")
    x = torch.empty(2, 64, 768, device="meta")
    q, k, v = f(x, nf.LtvInitValues())
    assert q.shape == (2, 64, 6, 128) and k.shape == (2, 64, 6, 128) and v.shape == (2, 64, 6, 128)


@pytest.mark.parametrize("B,T,C", [(32, 64, 128), (2, 96, 256)])
def test_filter_compiles_fullgraph_on_meta(B, T, C):
    """Dynamo traces the filter's forward with fullgraph=True (a graph break raises) through the fake
    kernels, and AOTAutograd traces the backward formula (operators only, no library calls), on the
    one-kernel shape (B * heads >= 2 * SMs: checkpoints, shared initial state) and on the two-op one."""
    NH, NKVH, D, r = 6, 6, 128, 128
    torch._dynamo.reset()
    with torch.device("meta"):
        f = nf.LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter(NH, NKVH, D, r)
        f.c = torch.nn.Linear(C, f.c.out_features, bias=False)
        x = torch.empty(B, T, C, dtype=torch.bfloat16).requires_grad_(True)
        grads = [torch.empty(B, T, n, D, dtype=torch.bfloat16) for n in (NH, NKVH, NKVH)]
    cf = torch.compile(f, fullgraph=True, backend="aot_eager")
    q, k, v = cf(x, nf.LtvInitValues())
    assert q.shape == (B, T, NH, D) and k.shape == (B, T, NKVH, D) and v.shape == (B, T, NKVH, D)
    torch.autograd.backward([q, k, v], grads)
    assert x.grad.shape == x.shape and f.c.weight.grad.shape == f.c.weight.shape
    assert f.init_param.grad.shape == (NH + 2 * NKVH, D) and f.logit_bias.grad.shape == (NH + 2 * NKVH, 1)


@pytest.mark.parametrize("B,T,C", [(32, 64, 128), (2, 96, 256)])
def test_forward_rotary_norm_compiles_fullgraph_on_meta(B, T, C):
    """The filter's forward with the attention's q / k prologue folded in (ltv_proj_scan_rope_norm_cuda_op:
    one-kernel shape with checkpoints, and the two-operator shape) traces with fullgraph=True, forward
    and backward, and gives the reference prologue's shapes ([B, T, heads, D])."""
    NH, NKVH, D, r = 6, 6, 128, 128
    torch._dynamo.reset()
    with torch.device("meta"):
        f = nf.LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter(NH, NKVH, D, r)
        f.c = torch.nn.Linear(C, f.c.out_features, bias=False)
        x = torch.empty(B, T, C, dtype=torch.bfloat16).requires_grad_(True)
        cos = torch.empty(1, T, 1, D // 2, dtype=torch.bfloat16)
        sin = torch.empty(1, T, 1, D // 2, dtype=torch.bfloat16)
        grads = [torch.empty(B, T, n, D, dtype=torch.bfloat16) for n in (NH, NKVH, NKVH)]

    def fwd(x):
        return f.forward_rotary_norm(x, nf.LtvInitValues(), (cos, sin))

    q, k, v = torch.compile(fwd, fullgraph=True, backend="aot_eager")(x)
    assert q.shape == (B, T, NH, D) and k.shape == (B, T, NKVH, D) and v.shape == (B, T, NKVH, D)
    torch.autograd.backward([q, k, v], grads)
    assert x.grad.shape == x.shape and f.c.weight.grad.shape == f.c.weight.shape
    assert f.init_param.grad.shape == (NH + 2 * NKVH, D) and f.logit_bias.grad.shape == (NH + 2 * NKVH, 1)
    s = str(OPS.ltv_proj_scan_rope_norm_cuda_op.default._schema)
    assert s.startswith("nanochat_cuda::ltv_proj_scan_rope_norm_cuda_op(Tensor x, Tensor weight, Tensor inits, "
                        "Tensor logit_bias, Tensor cos, Tensor sin, int NH, int NKVH, int da, int r, bool use_sigmoid)")


def test_ckpt_fake_shape_mirrors_the_kernel_condition():
    """The fake kernel promises checkpoints only where the one-kernel forward runs: C % 8 != 0, a
    head dim other than 128, fp32 or T % 32 != 0 give the empty checkpoint."""
    from nanochat_filter_b200 import ops

    def shape(B, T, C, dtype=torch.bfloat16, NH=6, NKVH=6, da=1, r=128):
        return ops._ckpt_shape(torch.empty(B, T, C, device="meta", dtype=dtype), NH, NKVH, da, r)

    assert shape(32, 64, 128) == (32, 18, 2, 128)
    assert shape(32, 64, 124) == (0,)                       # C % 8 != 0
    assert shape(32, 64, 128, dtype=torch.float32) == (0,)
    assert shape(32, 48, 128) == (0,)                       # T % 32 != 0
    assert shape(32, 64, 128, da=2, r=64) == (0,)           # two decay groups per head
    assert shape(2, 64, 128) == (0,)                        # fewer than two rows per SM


def test_no_cpu_fallback():
    x = torch.randn(1, 8, 16)
    w = torch.randn(24, 16)
    with pytest.raises(NotImplementedError):
        OPS.fused_linear_transpose_cuda_op(x, w)
    comb = torch.randn(1, 8, 3 * 3)
    with pytest.raises(NotImplementedError):
        OPS.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_op(
            comb, torch.randn(1, 3, 2), torch.randn(3, 1), 1, 1, 1, 2, 8, 8, 4, 32, 2, 8, True)


def test_parameters_and_head_major_init_layout():
    NH, NKVH, D, r = 2, 1, 8, 4
    f = nf.LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter(NH, NKVH, D, r)
    H, Da, C = NH + 2 * NKVH, D // r, NH * D
    assert f.c.weight.shape == (H * (D + Da), C)
    assert f.logit_bias.shape == (H, Da) and f.init_param.shape == (H, D)
    torch.manual_seed(0)
    f.init_weights(alpha_mlp_bias_init=2.0, weight_s=0.1, bias_s=0.25, init_s=0.3)
    assert f.logit_bias.min() >= 1.75 and f.logit_bias.max() <= 2.25
    assert f.init_param.abs().max() <= 0.3
    # rows: [head h values (D) | head h logits (Da)] for h = 0..H-1
    torch.manual_seed(0)
    vals = torch.empty(H * D, C).uniform_(-0.1, 0.1)
    logits = torch.empty(H * Da, C).uniform_(-0.1, 0.1)
    w = f.c.weight.detach().view(H, D + Da, C)
    torch.testing.assert_close(w[:, :D].reshape(H * D, C), vals)
    torch.testing.assert_close(w[:, D:].reshape(H * Da, C), logits)
    mats, lins = f.get_matrix_linear_params()
    assert mats == [f.c.weight] and lins == [f.logit_bias, f.init_param]
    assert f.ltv_parameter_count() == H * Da * C + H * Da + H * D
    assert f.estimate_flops(1024) == 6 * H * Da * C + 7 * H * D


def test_dtype_policy_and_inits_resolution():
    assert util.should_run_ltv_in_fp32("cpu") is False
    with torch.autocast("cpu", dtype=torch.bfloat16):
        assert util.should_run_ltv_in_fp32("cpu") is False
    p = torch.randn(3, 4)
    e = util.resolve_inits_original_dtype(2, p, util.LtvInitValues())
    assert e.shape == (2, 3, 4) and torch.equal(e[1], p)
    q, k, v = torch.randn(2, 1, 4), torch.randn(2, 1, 4), torch.randn(2, 1, 4)
    e = util.resolve_inits_original_dtype(2, p, util.LtvInitValues(q, k, v))
    assert torch.equal(e, torch.cat([q, k, v], 1))
    assert util.env_int("LTVQKV_SURELY_UNSET_VARIABLE", 5) == 5


def test_kv_cache_last_qkv_semantics():
    cache = nf.KVCache(batch_size=2, num_q_heads=2, num_kv_heads=1, seq_len=16, head_dim=4, num_layers=2)
    assert not cache.has_last_qkv(0)
    q, k, v = torch.randn(2, 2, 4), torch.randn(2, 1, 4), torch.randn(2, 1, 4)
    cache.update_last_qkv(0, q, k, v)
    assert cache.has_last_qkv(0) and not cache.has_last_qkv(1)
    cache.update_last_qkv(1, q + 1, k + 1, v + 1)
    assert cache.has_last_qkv(1)
    assert torch.equal(cache.last_qkv.q.special[1], q + 1)
    # a later step overwrites layer 0 again
    cache.update_last_qkv(0, q * 2, k * 2, v * 2)
    assert torch.equal(cache.last_qkv.k.special[0], k * 2)
    # prefill broadcasts a batch-1 state over the batch
    one = nf.KVCache(batch_size=1, num_q_heads=2, num_kv_heads=1, seq_len=16, head_dim=4, num_layers=2)
    one.update_last_qkv(0, q[:1], k[:1], v[:1])
    one.update_last_qkv(1, q[1:], k[1:], v[1:])
    one.pos = 7
    many = nf.KVCache(batch_size=3, num_q_heads=2, num_kv_heads=1, seq_len=16, head_dim=4, num_layers=2)
    many.prefill(one)
    assert many.pos == 7 and many.has_last_qkv(1)
    assert torch.equal(many.last_qkv.q.special[0], q[:1].expand(3, 2, 4))


class _FakeFilter(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.calls = []

    def forward(self, x, previous_values):
        # previous_values are views of the cache state (as in the reference), so record copies
        self.calls.append(nf.LtvInitValues(*(None if t is None else t.clone() for t in (
            previous_values.q, previous_values.k, previous_values.v))))
        B, T, _ = x.shape
        return (torch.full((B, T, 2, 4), float(T)), torch.full((B, T, 1, 4), 1.0), torch.full((B, T, 1, 4), 2.0))


def test_computer_module_threads_cache_state():
    filt = _FakeFilter()
    mod = nf.LtvCombinedQkvComputerModule(0, filt)
    cache = nf.KVCache(batch_size=2, num_q_heads=2, num_kv_heads=1, seq_len=16, head_dim=4, num_layers=1)
    mod(torch.zeros(2, 5, 8), cache)
    assert filt.calls[-1].q is None
    mod(torch.zeros(2, 1, 8), cache)
    assert filt.calls[-1].q is not None and torch.equal(filt.calls[-1].q, torch.full((2, 2, 4), 5.0))
    assert torch.equal(cache.last_qkv.q.special[0], torch.full((2, 2, 4), 1.0))
    mod(torch.zeros(2, 3, 8), None)
    assert filt.calls[-1].q is None


def test_filter_parameter_discovery():
    from nanochat_filter_b200.dist import filter_parameters

    m = torch.nn.ModuleList([nf.LtvCombinedQkvComputerModule(i, filters.LtvCombinedHeadMajorQkvFilter(2, 1, 8, 4))
                             for i in range(2)])
    ps = filter_parameters([m])
    assert len(ps) == 6
    assert ps[0] is m[0].ltv_filter.c.weight
