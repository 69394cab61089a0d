"""torch.library operators of the filtered-QKV hot path (namespace `nanochat_cuda`).

Same op names, schemas, ownership and error behaviour as the reference's registry
(nanochat/ops/ltv_cuda_ops.py:3, 115-145, 242-250; implementations in
nanochat/ops/ltv_cuda_fused_concat_head_major_register_cast_blelloch_scan.py:31-289 and
nanochat/ops/fused_linear_transpose.py:20-134; fake kernels in nanochat/ops/ltv_cuda_meta.py),
so code written against the reference's `torch.ops.nanochat_cuda.*` runs unchanged:

  ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_op      (autograd)
  ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_forward_kernel
  ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_backward_kernel
  fused_linear_transpose_cuda_op                                       (autograd)
  fused_linear_transpose
  fused_linear_transpose_backward_kernel

the look-back (chunk-restarting) scans of nanochat/ops/ltv_cuda_look_back_fused_concat_head_major_register_cast_
{blelloch,sequential}_scan.py (schemas ltv_cuda_ops.py:172-240; both families share one implementation):

  ltv_look_back_fused_concat_head_major_register_cast_{blelloch,sequential}_scan_cuda_op (autograd)
  ..._forward_kernel, ..._backward_kernel

plus ops the reference does not have: `ltv_decode_step` (one-launch decode update),
`ltv_proj_scan_cuda_op` / `ltv_proj_scan_forward_kernel` (projection and scan forward in one
call, the composition the reference's filter runs as two ops; same outputs bit for bit; its fifth
output holds the scan state at every 32-token chunk start) and `ltv_scan_ckpt_backward_kernel`
(the scan backward replaying the outputs from those states instead of reading them; same
gradients bit for bit), and the rotary + QK-norm consumer ops.

The CUDA implementations call libltvqkv.so through its C ABI; only "CUDA" and "Meta"
dispatch keys are registered, so CPU tensors raise NotImplementedError from the dispatcher —
there is no CPU fallback. The scan's tuning integers are accepted and ignored (the B200
kernels pick their own tiling).
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib

_SCAN_OP = "ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_op"
_SCAN_FWD = "ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_forward_kernel"
_SCAN_BWD = "ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_backward_kernel"

lib = torch.library.Library("nanochat_cuda", "DEF")

lib.define(
    f"{_SCAN_OP}("
    "Tensor combined, Tensor inits, Tensor logit_bias, "
    "int NH, int NKVH, int da, int r, "
    "int scan_threads_forward, int r_threads_forward, int r_items_forward, "
    "int scan_threads_backward, int r_threads_backward, int r_items_backward, "
    "bool use_sigmoid"
    ") -> (Tensor, Tensor, Tensor)"
)
lib.define(
    f"{_SCAN_FWD}("
    "Tensor combined, Tensor inits, Tensor logit_bias, "
    "Tensor(a!) out_q, Tensor(b!) out_k, Tensor(c!) out_v, "
    "int T, int NH, int NKVH, int da, int r, "
    "int scan_threads_forward, int r_threads_forward, int r_items_forward, "
    "bool use_sigmoid"
    ") -> ()"
)
lib.define(
    f"{_SCAN_BWD}("
    "Tensor combined, Tensor inits, Tensor logit_bias, "
    "Tensor hq, Tensor hk, Tensor hv, "
    "Tensor grad_hq, Tensor grad_hk, Tensor grad_hv, "
    "Tensor(a!) grad_combined, Tensor(b!) grad_inits, Tensor(c!) grad_logit_bias, "
    "int NH, int NKVH, int da, int r, "
    "int scan_threads_backward, int r_threads_backward, int r_items_backward, "
    "bool use_sigmoid"
    ") -> ()"
)
lib.define("fused_linear_transpose(Tensor x, Tensor weight, Tensor(a!) out) -> ()")
lib.define("fused_linear_transpose_cuda_op(Tensor x, Tensor weight) -> Tensor")
lib.define(
    "fused_linear_transpose_backward_kernel("
    "Tensor x, Tensor weight, Tensor grad_out, Tensor(a!) grad_x, Tensor(b!) grad_weight"
    ") -> ()"
)
_LB = "ltv_look_back_fused_concat_head_major_register_cast_{}_scan_cuda_{}"
_LB_TUNE_FWD = {"blelloch": "int scan_threads_forward, int r_threads_forward, int r_items_forward, ",
                "sequential": "int r_threads_forward, int r_items_forward, "}
_LB_TUNE_BWD = {"blelloch": "int scan_threads_backward, int r_threads_backward, int r_items_backward, ",
                "sequential": "int r_threads_backward, int r_items_backward, "}
for _kind in ("blelloch", "sequential"):
    lib.define(
        f"{_LB.format(_kind, 'op')}("
        "Tensor combined, Tensor inits, Tensor logit_bias, int NH, int NKVH, int da, int r, int P, int Q, int K, "
        f"{_LB_TUNE_FWD[_kind]}{_LB_TUNE_BWD[_kind]}bool use_sigmoid"
        ") -> (Tensor, Tensor, Tensor)"
    )
    lib.define(
        f"{_LB.format(_kind, 'forward_kernel')}("
        "Tensor combined, Tensor inits, Tensor logit_bias, Tensor(a!) out_q, Tensor(b!) out_k, Tensor(c!) out_v, "
        "int B, int T, int NH, int NKVH, int da, int r, int P, int Q, int K, "
        f"{_LB_TUNE_FWD[_kind]}bool use_sigmoid"
        ") -> ()"
    )
    lib.define(
        f"{_LB.format(_kind, 'backward_kernel')}("
        "Tensor combined, Tensor inits, Tensor logit_bias, Tensor hq, Tensor hk, Tensor hv, "
        "Tensor grad_hq, Tensor grad_hk, Tensor grad_hv, "
        "Tensor(a!) grad_combined, Tensor(b!) grad_inits, Tensor(c!) grad_logit_bias, "
        "int NH, int NKVH, int da, int r, int P, int Q, int K, "
        f"{_LB_TUNE_BWD[_kind]}bool use_sigmoid"
        ") -> ()"
    )
lib.define(
    "ltv_proj_scan_forward_kernel("
    "Tensor x, Tensor weight, Tensor inits, Tensor logit_bias, Tensor(a!) combined, "
    "Tensor(b!) out_q, Tensor(c!) out_k, Tensor(d!) out_v, int NH, int NKVH, int da, int r, bool use_sigmoid"
    ") -> ()"
)
lib.define(
    "ltv_proj_scan_cuda_op("
    "Tensor x, Tensor weight, Tensor inits, Tensor logit_bias, int NH, int NKVH, int da, int r, bool use_sigmoid"
    ") -> (Tensor, Tensor, Tensor, Tensor, Tensor)"
)
lib.define(
    "ltv_scan_ckpt_backward_kernel("
    "Tensor combined, Tensor inits, Tensor logit_bias, Tensor ckpt, Tensor grad_hq, Tensor grad_hk, Tensor grad_hv, "
    "Tensor(a!) grad_combined, Tensor(b!) grad_inits, Tensor(c!) grad_logit_bias, int NH, int NKVH, int da, int r, "
    "bool use_sigmoid"
    ") -> ()"
)
lib.define("ltv_rotary_qk_norm(Tensor q, Tensor k, Tensor cos, Tensor sin) -> (Tensor, Tensor)")
lib.define(
    "ltv_proj_scan_rope_norm_cuda_op("
    "Tensor x, Tensor weight, Tensor inits, Tensor logit_bias, Tensor cos, Tensor sin, int NH, int NKVH, int da, "
    "int r, bool use_sigmoid"
    ") -> (Tensor, Tensor, Tensor, Tensor, Tensor)"
)
lib.define(
    "ltv_rotary_qk_norm_ckpt_backward("
    "Tensor combined, Tensor inits, Tensor logit_bias, Tensor ckpt, Tensor cos, Tensor sin, Tensor grad_q, "
    "Tensor grad_k, int NH, int NKVH, int da, int r, bool use_sigmoid"
    ") -> (Tensor, Tensor)"
)
lib.define(
    "ltv_rotary_qk_norm_backward(Tensor q, Tensor k, Tensor cos, Tensor sin, Tensor grad_q, Tensor grad_k) "
    "-> (Tensor, Tensor)"
)
lib.define(
    "ltv_decode_step_("
    "Tensor x, Tensor weight, Tensor logit_bias, Tensor(a!) state_q, Tensor(b!) state_k, Tensor(c!) state_v, "
    "int NH, int NKVH, int da, int r, bool use_sigmoid"
    ") -> ()"
)
lib.define(
    "ltv_decode_step("
    "Tensor x, Tensor weight, Tensor logit_bias, Tensor? prev_q, Tensor? prev_k, Tensor? prev_v, "
    "Tensor init_param, int NH, int NKVH, int da, int r, bool use_sigmoid"
    ") -> (Tensor, Tensor, Tensor)"
)


# ------------------------------------------------------------------------------------------
# Scan
# ------------------------------------------------------------------------------------------
def _check_scan_inputs(combined, inits, logit_bias, NH, NKVH, da, r):
    if combined.dim() != 3:
        raise RuntimeError(f"combined must be [B, T, F], got {tuple(combined.shape)}")
    H = NH + 2 * NKVH
    D = da * r
    B, T, F = combined.shape
    if F != H * (D + da):
        raise RuntimeError(f"combined has F={F}, expected (NH+2*NKVH)*(D+da) = {H * (D + da)}")
    if tuple(inits.shape) != (B, H, D):
        raise RuntimeError(f"inits must be [B, H, D] = {(B, H, D)}, got {tuple(inits.shape)}")
    if tuple(logit_bias.shape) != (H, da):
        raise RuntimeError(f"logit_bias must be [H, da] = {(H, da)}, got {tuple(logit_bias.shape)}")
    if combined.dtype != inits.dtype:
        raise RuntimeError(f"combined ({combined.dtype}) and inits ({inits.dtype}) must share a dtype")
    if logit_bias.dtype != torch.float32:
        raise RuntimeError(f"logit_bias must be float32, got {logit_bias.dtype}")


def _scan_forward_kernel(combined, inits, logit_bias, out_q, out_k, out_v, T, NH, NKVH, da, r,
                         scan_threads_forward, r_threads_forward, r_items_forward, use_sigmoid):
    _check_scan_inputs(combined, inits, logit_bias, NH, NKVH, da, r)
    L = _lib.load()
    B = combined.shape[0]
    inits = inits.contiguous()
    logit_bias = logit_bias.contiguous()
    for o in (out_q, out_k, out_v):
        if not o.is_contiguous() or o.dtype != combined.dtype:
            raise RuntimeError("out_q/out_k/out_v must be contiguous and share combined's dtype")
    nbytes = L.ltvqkv_scan_workspace_bytes(B, T, NH, NKVH, da, r)
    ws = _lib.workspace(combined.device, nbytes)
    sc = combined.stride()
    rc = L.ltvqkv_scan_fwd(_lib.dtype_code(combined.dtype), combined.data_ptr(), sc[0], sc[1], sc[2],
                           inits.data_ptr(), logit_bias.data_ptr(), out_q.data_ptr(), out_k.data_ptr(),
                           out_v.data_ptr(), B, T, NH, NKVH, da, r, int(bool(use_sigmoid)),
                           ws.data_ptr(), ws.numel(), _lib.stream_handle(combined.device))
    _lib.check(rc, "ltvqkv_scan_fwd")


def _scan_op(combined, inits, logit_bias, NH, NKVH, da, r, scan_threads_forward, r_threads_forward,
             r_items_forward, scan_threads_backward, r_threads_backward, r_items_backward, use_sigmoid):
    B, T, _ = combined.shape
    D = da * r
    kw = dict(device=combined.device, dtype=combined.dtype, memory_format=torch.contiguous_format)
    out_q = torch.empty((B, NH, T, D), **kw)
    out_k = torch.empty((B, NKVH, T, D), **kw)
    out_v = torch.empty((B, NKVH, T, D), **kw)
    _scan_forward_kernel(combined, inits, logit_bias, out_q, out_k, out_v, T, NH, NKVH, da, r,
                         scan_threads_forward, r_threads_forward, r_items_forward, use_sigmoid)
    return out_q, out_k, out_v


def _scan_backward_kernel(combined, inits, logit_bias, hq, hk, hv, grad_hq, grad_hk, grad_hv, grad_combined,
                          grad_inits, grad_logit_bias, NH, NKVH, da, r, scan_threads_backward, r_threads_backward,
                          r_items_backward, use_sigmoid):
    _check_scan_inputs(combined, inits, logit_bias, NH, NKVH, da, r)
    L = _lib.load()
    B, T, _ = combined.shape
    inits = inits.contiguous()
    logit_bias = logit_bias.contiguous()
    if not grad_inits.is_contiguous() or not grad_logit_bias.is_contiguous():
        raise RuntimeError("grad_inits and grad_logit_bias must be contiguous")
    if grad_combined.shape != combined.shape or grad_combined.dtype != combined.dtype:
        raise RuntimeError("grad_combined must match combined's shape and dtype")
    for t in (hq, hk, hv, grad_hq, grad_hk, grad_hv):
        if t.dtype != combined.dtype:
            raise RuntimeError("saved outputs and their gradients must share combined's dtype")
    nbytes = L.ltvqkv_scan_workspace_bytes(B, T, NH, NKVH, da, r)
    ws = _lib.workspace(combined.device, nbytes)
    sc, gc = combined.stride(), grad_combined.stride()
    S = _lib.strides
    rc = L.ltvqkv_scan_bwd(
        _lib.dtype_code(combined.dtype), combined.data_ptr(), sc[0], sc[1], sc[2], inits.data_ptr(),
        logit_bias.data_ptr(),
        hq.data_ptr(), S(hq.stride()), hk.data_ptr(), S(hk.stride()), hv.data_ptr(), S(hv.stride()),
        grad_hq.data_ptr(), S(grad_hq.stride()), grad_hk.data_ptr(), S(grad_hk.stride()),
        grad_hv.data_ptr(), S(grad_hv.stride()),
        grad_combined.data_ptr(), gc[0], gc[1], gc[2], grad_inits.data_ptr(), grad_logit_bias.data_ptr(),
        B, T, NH, NKVH, da, r, int(bool(use_sigmoid)), ws.data_ptr(), ws.numel(),
        _lib.stream_handle(combined.device))
    _lib.check(rc, "ltvqkv_scan_bwd")


def _scan_setup(ctx, inputs, output):
    (combined, inits, logit_bias, NH, NKVH, da, r, _sf, _rf, _if, sb, rb, ib, use_sigmoid) = inputs
    hq, hk, hv = output
    ctx.save_for_backward(combined, inits, logit_bias, hq, hk, hv)
    ctx.NH, ctx.NKVH, ctx.da, ctx.r = NH, NKVH, da, r
    ctx.tuning = (sb, rb, ib)
    ctx.use_sigmoid = use_sigmoid


def _scan_backward(ctx, grad_hq, grad_hk, grad_hv):
    combined, inits, logit_bias, hq, hk, hv = ctx.saved_tensors
    grad_hq = torch.zeros_like(hq) if grad_hq is None else grad_hq
    grad_hk = torch.zeros_like(hk) if grad_hk is None else grad_hk
    grad_hv = torch.zeros_like(hv) if grad_hv is None else grad_hv
    grad_combined = torch.empty_like(combined)
    grad_inits = torch.empty_like(inits, memory_format=torch.contiguous_format)
    grad_logit_bias = torch.zeros_like(logit_bias, memory_format=torch.contiguous_format)
    torch.ops.nanochat_cuda.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_backward_kernel(
        combined, inits, logit_bias, hq, hk, hv, grad_hq, grad_hk, grad_hv, grad_combined, grad_inits,
        grad_logit_bias, ctx.NH, ctx.NKVH, ctx.da, ctx.r, *ctx.tuning, ctx.use_sigmoid)
    return (grad_combined, grad_inits, grad_logit_bias) + (None,) * 11


torch.library.register_autograd(f"nanochat_cuda::{_SCAN_OP}", _scan_backward, setup_context=_scan_setup)


@torch.library.register_fake(f"nanochat_cuda::{_SCAN_OP}")
def _scan_op_fake(combined, inits, logit_bias, NH, NKVH, da, r, *tuning_and_flag):
    B, T, _ = combined.shape
    D = da * r
    return (combined.new_empty((B, NH, T, D)), combined.new_empty((B, NKVH, T, D)),
            combined.new_empty((B, NKVH, T, D)))


@torch.library.register_fake(f"nanochat_cuda::{_SCAN_FWD}")
def _scan_fwd_fake(*args):
    return None


@torch.library.register_fake(f"nanochat_cuda::{_SCAN_BWD}")
def _scan_bwd_fake(*args):
    return None


# ------------------------------------------------------------------------------------------
# Projection ("fused linear transpose")
# ------------------------------------------------------------------------------------------
def _is_transposed_grad_out(g: torch.Tensor) -> bool:
    return g.stride(1) == 1 and g.stride(2) == g.size(1) and g.stride(0) == g.size(1) * g.size(2)


def _fused_linear_transpose(x, weight, out):
    if not x.is_contiguous() or not weight.is_contiguous() or not out.is_contiguous():
        raise RuntimeError("fused_linear_transpose requires contiguous x, weight, and out tensors")
    L = _lib.load()
    B, T, K = x.shape
    F = weight.shape[0]
    if weight.shape[1] != K or tuple(out.shape) != (B, F, T):
        raise RuntimeError(f"shape mismatch: x {tuple(x.shape)}, weight {tuple(weight.shape)}, out {tuple(out.shape)}")
    if out.dtype != x.dtype:
        raise RuntimeError("out must have x's dtype")
    w = weight if weight.dtype == x.dtype else weight.to(x.dtype)
    ws = _lib.workspace(x.device, L.ltvqkv_gemm_workspace_bytes())
    rc = L.ltvqkv_gemm_fwd(_lib.dtype_code(x.dtype), x.data_ptr(), w.data_ptr(), out.data_ptr(), B, T, K, F,
                           ws.data_ptr(), ws.numel(), _lib.stream_handle(x.device))
    _lib.check(rc, "ltvqkv_gemm_fwd")


def _fused_linear_transpose_op(x, weight):
    B, T, _ = x.shape
    F = weight.size(0)
    # Every element is written by the kernel, so no zero fill is needed.
    out = torch.empty((B, F, T), dtype=x.dtype, device=x.device)
    _fused_linear_transpose(x, weight, out)
    return out


def _fused_linear_transpose_backward_kernel(x, weight, grad_out, grad_x, grad_weight):
    if not x.is_contiguous() or not weight.is_contiguous() or not (
            grad_out.is_contiguous() or _is_transposed_grad_out(grad_out)):
        raise RuntimeError(
            "fused_linear_transpose_backward_kernel requires contiguous x and weight, and either contiguous or "
            f"transposed grad_out. Found strides: x={x.stride()}, weight={weight.stride()}, "
            f"grad_out={grad_out.stride()}")
    L = _lib.load()
    B, T, K = x.shape
    F = weight.shape[0]
    w = weight if weight.dtype == grad_out.dtype else weight.to(grad_out.dtype)
    xx = x if x.dtype == grad_out.dtype else x.to(grad_out.dtype)
    gx = grad_x if (grad_x.is_contiguous() and grad_x.dtype == grad_out.dtype) else torch.empty(
        (B, T, K), dtype=grad_out.dtype, device=x.device)
    if not grad_weight.is_contiguous():
        raise RuntimeError("grad_weight must be contiguous")
    ws = _lib.workspace(x.device, L.ltvqkv_gemm_workspace_bytes(), kind="gemm_bwd")
    gs = grad_out.stride()
    rc = L.ltvqkv_gemm_bwd(_lib.dtype_code(grad_out.dtype), xx.data_ptr(), w.data_ptr(), grad_out.data_ptr(),
                           gs[0], gs[1], gs[2], gx.data_ptr(), grad_weight.data_ptr(),
                           _lib.dtype_code(grad_weight.dtype), B, T, K, F, ws.data_ptr(), ws.numel(),
                           _lib.stream_handle(x.device))
    _lib.check(rc, "ltvqkv_gemm_bwd")
    if gx is not grad_x:
        grad_x.copy_(gx)


def _flt_setup(ctx, inputs, output):
    x, weight = inputs
    ctx.save_for_backward(x, weight)


def _flt_backward(ctx, grad_out):
    x, weight = ctx.saved_tensors
    if not x.is_contiguous() or not weight.is_contiguous() or not (
            grad_out.is_contiguous() or _is_transposed_grad_out(grad_out)):
        raise RuntimeError(
            "fused_linear_transpose backward requires contiguous x and weight, and either contiguous or transposed "
            f"grad_out. Found strides: x={x.stride()}, weight={weight.stride()}, grad_out={grad_out.stride()}")
    # Every element of both gradients is written by the kernel.
    grad_x = torch.empty_like(x, memory_format=torch.contiguous_format)
    grad_weight = torch.empty_like(weight, memory_format=torch.contiguous_format)
    torch.ops.nanochat_cuda.fused_linear_transpose_backward_kernel(x, weight, grad_out, grad_x, grad_weight)
    return grad_x, grad_weight


torch.library.register_autograd("nanochat_cuda::fused_linear_transpose_cuda_op", _flt_backward,
                                setup_context=_flt_setup)


@torch.library.register_fake("nanochat_cuda::fused_linear_transpose_cuda_op")
def _flt_fake(x, weight):
    B, T, _ = x.shape
    return x.new_empty((B, weight.shape[0], T))


@torch.library.register_fake("nanochat_cuda::fused_linear_transpose")
def _flt_kernel_fake(x, weight, out):
    return None


@torch.library.register_fake("nanochat_cuda::fused_linear_transpose_backward_kernel")
def _flt_bwd_fake(x, weight, grad_out, grad_x, grad_weight):
    return None


# ------------------------------------------------------------------------------------------
# Look-back scans (reference nanochat/ops/ltv_cuda_look_back_fused_concat_head_major_register_cast_
# {blelloch,sequential}_scan.py: op, forward_kernel, backward_kernel, autograd _setup/backward)
# ------------------------------------------------------------------------------------------
def _check_pqk(P, Q, K):
    if P < 1 or Q < 1 or K < 1:
        raise RuntimeError(f"look-back chunking needs P, Q, K >= 1, got P={P}, Q={Q}, K={K}")


def _lb_forward_kernel(combined, inits, logit_bias, out_q, out_k, out_v, B, T, NH, NKVH, da, r, P, Q, K,
                       *tuning_and_flag):
    use_sigmoid = tuning_and_flag[-1]
    _check_scan_inputs(combined, inits, logit_bias, NH, NKVH, da, r)
    _check_pqk(P, Q, K)
    if combined.shape[0] != B or combined.shape[1] != T:
        raise RuntimeError(f"B={B}, T={T} do not match combined {tuple(combined.shape)}")
    for o in (out_q, out_k, out_v):
        if not o.is_contiguous() or o.dtype != combined.dtype:
            raise RuntimeError("out_q/out_k/out_v must be contiguous and share combined's dtype")
    L = _lib.load()
    inits = inits.contiguous()
    logit_bias = logit_bias.contiguous()
    sc = combined.stride()
    rc = L.ltvqkv_lookback_scan_fwd(_lib.dtype_code(combined.dtype), combined.data_ptr(), sc[0], sc[1], sc[2],
                                    inits.data_ptr(), logit_bias.data_ptr(), out_q.data_ptr(), out_k.data_ptr(),
                                    out_v.data_ptr(), B, T, NH, NKVH, da, r, P, Q, K, int(bool(use_sigmoid)),
                                    _lib.stream_handle(combined.device))
    _lib.check(rc, "ltvqkv_lookback_scan_fwd")


def _lb_op(combined, inits, logit_bias, NH, NKVH, da, r, P, Q, K, *tuning_and_flag):
    B, T, _ = combined.shape
    D = da * r
    kw = dict(device=combined.device, dtype=combined.dtype, memory_format=torch.contiguous_format)
    out_q = torch.empty((B, NH, T, D), **kw)
    out_k = torch.empty((B, NKVH, T, D), **kw)
    out_v = torch.empty((B, NKVH, T, D), **kw)
    _lb_forward_kernel(combined, inits, logit_bias, out_q, out_k, out_v, B, T, NH, NKVH, da, r, P, Q, K,
                       tuning_and_flag[-1])
    return out_q, out_k, out_v


def _lb_backward_kernel(combined, inits, logit_bias, hq, hk, hv, grad_hq, grad_hk, grad_hv, grad_combined,
                        grad_inits, grad_logit_bias, NH, NKVH, da, r, P, Q, K, *tuning_and_flag):
    use_sigmoid = tuning_and_flag[-1]
    _check_scan_inputs(combined, inits, logit_bias, NH, NKVH, da, r)
    _check_pqk(P, Q, K)
    if not grad_inits.is_contiguous() or not grad_logit_bias.is_contiguous():
        raise RuntimeError("grad_inits and grad_logit_bias must be contiguous")
    if grad_combined.shape != combined.shape or grad_combined.dtype != combined.dtype:
        raise RuntimeError("grad_combined must match combined's shape and dtype")
    for t in (hq, hk, hv, grad_hq, grad_hk, grad_hv):
        if t.dtype != combined.dtype:
            raise RuntimeError("saved outputs and their gradients must share combined's dtype")
    L = _lib.load()
    B, T, _ = combined.shape
    inits = inits.contiguous()
    logit_bias = logit_bias.contiguous()
    ws = _lib.workspace(combined.device, L.ltvqkv_lookback_bwd_workspace_bytes(B, T, NH, NKVH, da, r, P, Q, K),
                        kind="lookback_bwd")
    sc, gc = combined.stride(), grad_combined.stride()
    S = _lib.strides
    rc = L.ltvqkv_lookback_scan_bwd(
        _lib.dtype_code(combined.dtype), combined.data_ptr(), sc[0], sc[1], sc[2], inits.data_ptr(),
        logit_bias.data_ptr(),
        hq.data_ptr(), S(hq.stride()), hk.data_ptr(), S(hk.stride()), hv.data_ptr(), S(hv.stride()),
        grad_hq.data_ptr(), S(grad_hq.stride()), grad_hk.data_ptr(), S(grad_hk.stride()),
        grad_hv.data_ptr(), S(grad_hv.stride()),
        grad_combined.data_ptr(), gc[0], gc[1], gc[2], grad_inits.data_ptr(), grad_logit_bias.data_ptr(),
        B, T, NH, NKVH, da, r, P, Q, K, int(bool(use_sigmoid)), ws.data_ptr(), ws.numel(),
        _lib.stream_handle(combined.device))
    _lib.check(rc, "ltvqkv_lookback_scan_bwd")


def _lb_setup(ctx, inputs, output):
    combined, inits, logit_bias, NH, NKVH, da, r, P, Q, K = inputs[:10]
    ctx.save_for_backward(combined, inits, logit_bias, *output)
    ctx.args = (NH, NKVH, da, r, P, Q, K)
    ctx.tuning_bwd = tuple(inputs[10:-1])[len(inputs[10:-1]) // 2:]
    ctx.use_sigmoid = inputs[-1]


def _make_lb_backward(kind):
    def _lb_backward(ctx, grad_hq, grad_hk, grad_hv):
        combined, inits, logit_bias, hq, hk, hv = ctx.saved_tensors
        grad_hq = torch.zeros_like(hq) if grad_hq is None else grad_hq
        grad_hk = torch.zeros_like(hk) if grad_hk is None else grad_hk
        grad_hv = torch.zeros_like(hv) if grad_hv is None else grad_hv
        grad_combined = torch.empty_like(combined)
        grad_inits = torch.empty_like(inits, memory_format=torch.contiguous_format)
        grad_logit_bias = torch.zeros_like(logit_bias, memory_format=torch.contiguous_format)
        getattr(torch.ops.nanochat_cuda, _LB.format(kind, "backward_kernel"))(
            combined, inits, logit_bias, hq, hk, hv, grad_hq, grad_hk, grad_hv, grad_combined, grad_inits,
            grad_logit_bias, *ctx.args, *ctx.tuning_bwd, ctx.use_sigmoid)
        return (grad_combined, grad_inits, grad_logit_bias) + (None,) * (len(ctx.tuning_bwd) * 2 + 8)
    return _lb_backward


def _lb_op_fake(combined, inits, logit_bias, NH, NKVH, da, r, *rest):
    B, T, _ = combined.shape
    D = da * r
    return (combined.new_empty((B, NH, T, D)), combined.new_empty((B, NKVH, T, D)),
            combined.new_empty((B, NKVH, T, D)))


for _kind in ("blelloch", "sequential"):
    torch.library.register_autograd(f"nanochat_cuda::{_LB.format(_kind, 'op')}", _make_lb_backward(_kind),
                                    setup_context=_lb_setup)
    torch.library.register_fake(f"nanochat_cuda::{_LB.format(_kind, 'op')}", _lb_op_fake)
    torch.library.register_fake(f"nanochat_cuda::{_LB.format(_kind, 'forward_kernel')}", lambda *args: None)
    torch.library.register_fake(f"nanochat_cuda::{_LB.format(_kind, 'backward_kernel')}", lambda *args: None)


# ------------------------------------------------------------------------------------------
# Projection + scan forward in one call
# ------------------------------------------------------------------------------------------
def _proj_scan_forward_kernel(x, weight, inits, logit_bias, combined, out_q, out_k, out_v, NH, NKVH, da, r,
                              use_sigmoid, ckpt=None):
    """fused_linear_transpose(x, weight) -> combined [B, F, T], then the scan over combined^T.

    Equals `fused_linear_transpose` followed by the scan forward kernel on `combined.transpose(1, 2)`
    (the reference filter's composition,
    nanochat/ltv_cuda_fused_concat_head_major_register_cast_blelloch_scan_qkv_filter.py:24-73).
    With `ckpt` ([B, H, T / 32, D] fp32) the scan states at the 32-token chunk starts are written
    too, and `inits` may be one state [H, D] for every sequence instead of [B, H, D]; returns False
    (and writes nothing) where the one-kernel form that does both does not apply.
    """
    if not x.is_contiguous() or x.dim() != 3:
        raise RuntimeError("ltv_proj_scan requires a contiguous [B, T, C] x")
    L = _lib.load()
    B, T, C = x.shape
    H = NH + 2 * NKVH
    D = da * r
    F = H * (D + da)
    w = (weight if weight.dtype == x.dtype else weight.to(x.dtype)).contiguous()
    if tuple(w.shape) != (F, C):
        raise RuntimeError(f"weight must be [{F}, {C}], got {tuple(w.shape)}")
    if tuple(combined.shape) != (B, F, T) or not combined.is_contiguous() or combined.dtype != x.dtype:
        raise RuntimeError("combined must be a contiguous [B, F, T] tensor of x's dtype")
    shared = inits.dim() == 2
    if shared and ckpt is None:
        raise RuntimeError("a shared [H, D] initial state is taken with the checkpoint output only")
    _check_scan_inputs(combined.transpose(1, 2), inits.unsqueeze(0).expand(B, -1, -1) if shared else inits,
                       logit_bias, NH, NKVH, da, r)
    inits = inits.contiguous()
    logit_bias = logit_bias.contiguous()
    for o, n in ((out_q, NH), (out_k, NKVH), (out_v, NKVH)):
        if not o.is_contiguous() or o.dtype != x.dtype or tuple(o.shape) != (B, n, T, D):
            raise RuntimeError("out_q/out_k/out_v must be contiguous [B, heads, T, D] of x's dtype")
    nbytes = max(L.ltvqkv_scan_workspace_bytes(B, T, NH, NKVH, da, r), L.ltvqkv_gemm_workspace_bytes())
    ws = _lib.workspace(x.device, nbytes)
    head = (_lib.dtype_code(x.dtype), x.data_ptr(), w.data_ptr(), inits.data_ptr())
    outs = (logit_bias.data_ptr(), combined.data_ptr(), out_q.data_ptr(), out_k.data_ptr(), out_v.data_ptr())
    rest = (B, T, C, NH, NKVH, da, r, int(bool(use_sigmoid)), ws.data_ptr(), ws.numel(), _lib.stream_handle(x.device))
    if ckpt is not None:
        if tuple(ckpt.shape) != (B, H, T // 32, D) or ckpt.dtype != torch.float32 or not ckpt.is_contiguous():
            raise RuntimeError("ckpt must be a contiguous [B, H, T / 32, D] float32 tensor")
        rc = L.ltvqkv_proj_scan_fwd_ckpt(*head, 0 if shared else H * D, *outs, ckpt.data_ptr(), *rest)
        if rc == _lib.ERR_UNSUPPORTED:
            return False
        _lib.check(rc, "ltvqkv_proj_scan_fwd_ckpt")
        return True
    rc = L.ltvqkv_proj_scan_fwd(*head, *outs, *rest)
    _lib.check(rc, "ltvqkv_proj_scan_fwd")
    return False


def _ckpt_shape(x, NH, NKVH, da, r):
    """Shape of the state checkpoints the one-kernel forward writes for these sizes, or (0,) where it
    does not apply. Mirrors the library's condition for that kernel (ltvqkv_proj_scan_fwd_ckpt): bf16,
    head dim 128 in one decay group, T % 32 == 0, C % 8 == 0, at most 128 heads and at least two
    (batch, head) rows per SM; its 16-byte alignment condition holds because _proj_scan_op hands
    the kernel aligned x and weight (copies where the caller's are not)."""
    B, T, C = x.shape
    H, D = NH + 2 * NKVH, da * r
    if (x.dtype != torch.bfloat16 or D != 128 or da != 1 or T % 32 != 0 or T == 0 or C % 8 != 0 or C == 0
            or not 1 <= H <= 128):
        return (0,)
    dev = x.device if x.device.type == "cuda" else None
    sms = (torch.cuda.get_device_properties(dev if dev is not None else torch.cuda.current_device())
           .multi_processor_count if torch.cuda.is_available() else 148)
    return (B, H, T // 32, D) if B * H >= 2 * sms else (0,)


def _proj_scan_op(x, weight, inits, logit_bias, NH, NKVH, da, r, use_sigmoid):
    B, T, _ = x.shape
    D = da * r
    F = (NH + 2 * NKVH) * (D + da)
    kw = dict(device=x.device, dtype=x.dtype)
    combined = torch.empty((B, F, T), **kw)
    out_q = torch.empty((B, NH, T, D), **kw)
    out_k = torch.empty((B, NKVH, T, D), **kw)
    out_v = torch.empty((B, NKVH, T, D), **kw)
    shared = inits.dim() == 2
    inits_k = inits.to(x.dtype) if shared else inits  # the state starts from its value in x's dtype
    ckpt = torch.empty(_ckpt_shape(x, NH, NKVH, da, r), device=x.device, dtype=torch.float32)
    if ckpt.numel():
        # the one-kernel form reads x and W with TMA (16-byte aligned bases): realign offset views so
        # that the checkpoint output the fake kernel promises is always written
        if x.data_ptr() % 16:
            x = x.clone()
        if weight.dtype == x.dtype and weight.is_contiguous() and weight.data_ptr() % 16:
            weight = weight.clone()
    if ckpt.numel() and _proj_scan_forward_kernel(x, weight, inits_k, logit_bias, combined, out_q, out_k, out_v, NH,
                                                  NKVH, da, r, use_sigmoid, ckpt):
        return combined, out_q, out_k, out_v, ckpt
    if shared:
        inits_k = inits_k.unsqueeze(0).expand(B, -1, -1).contiguous()
    _proj_scan_forward_kernel(x, weight, inits_k, logit_bias, combined, out_q, out_k, out_v, NH, NKVH, da, r,
                              use_sigmoid)
    return combined, out_q, out_k, out_v, ckpt.new_empty((0,))


def _rows_ok(t):
    """The row-streaming backward's layout for an upstream gradient: unit channel stride, 16-byte
    aligned rows."""
    st = t.stride()
    return st[3] == 1 and all(s_ % 8 == 0 for s_ in st[:3]) and t.data_ptr() % 16 == 0


def _scan_ckpt_backward(combined, inits, logit_bias, ckpt, grad_hq, grad_hk, grad_hv, grad_combined, grad_inits,
                        grad_logit_bias, NH, NKVH, da, r, use_sigmoid):
    """ltvqkv_scan_bwd_ckpt; returns its status (ERR_UNSUPPORTED: nothing was launched)."""
    L = _lib.load()
    B, T, _ = combined.shape
    H, D = NH + 2 * NKVH, da * r
    shared = inits.dim() == 2
    _check_scan_inputs(combined, inits.unsqueeze(0).expand(B, -1, -1) if shared else inits, logit_bias, NH, NKVH,
                       da, r)
    inits = inits.contiguous()
    if inits.data_ptr() % 16:  # the kernel loads initial states with 16-byte bulk copies
        inits = inits.clone()
    logit_bias = logit_bias.contiguous()
    # the row-streaming kernel's layout for the upstream gradients (unit channel stride, 16-byte rows)
    grad_hq, grad_hk, grad_hv = (g if _rows_ok(g) else g.contiguous() for g in (grad_hq, grad_hk, grad_hv))
    if not grad_inits.is_contiguous() or not grad_logit_bias.is_contiguous():
        raise RuntimeError("grad_inits and grad_logit_bias must be contiguous")
    if shared and (tuple(grad_inits.shape) != (H, D) or grad_inits.dtype != torch.float32):
        raise RuntimeError("with one initial state [H, D] for every sequence, grad_inits is its float32 [H, D] "
                           "gradient (summed over the batch)")
    if grad_combined.shape != combined.shape or grad_combined.dtype != combined.dtype:
        raise RuntimeError("grad_combined must match combined's shape and dtype")
    if ckpt.dtype != torch.float32 or not ckpt.is_contiguous():
        raise RuntimeError("ckpt must be a contiguous float32 tensor")
    for t in (grad_hq, grad_hk, grad_hv):
        if t.dtype != combined.dtype:
            raise RuntimeError("output gradients must share combined's dtype")
    nbytes = L.ltvqkv_scan_workspace_bytes(B, T, NH, NKVH, da, r)
    ws = _lib.workspace(combined.device, nbytes)
    sc, gc = combined.stride(), grad_combined.stride()
    S = _lib.strides
    return L.ltvqkv_scan_bwd_ckpt(
        _lib.dtype_code(combined.dtype), combined.data_ptr(), sc[0], sc[1], sc[2], inits.data_ptr(),
        0 if shared else H * D, logit_bias.data_ptr(), ckpt.data_ptr(),
        grad_hq.data_ptr(), S(grad_hq.stride()), grad_hk.data_ptr(), S(grad_hk.stride()),
        grad_hv.data_ptr(), S(grad_hv.stride()),
        grad_combined.data_ptr(), gc[0], gc[1], gc[2], grad_inits.data_ptr(), grad_logit_bias.data_ptr(),
        B, T, NH, NKVH, da, r, int(bool(use_sigmoid)), ws.data_ptr(), ws.numel(),
        _lib.stream_handle(combined.device))


def _scan_ckpt_backward_kernel(combined, inits, logit_bias, ckpt, grad_hq, grad_hk, grad_hv, grad_combined,
                               grad_inits, grad_logit_bias, NH, NKVH, da, r, use_sigmoid):
    """The scan backward kernel from the forward's state checkpoints (ltv_proj_scan_cuda_op's fifth
    output) instead of its outputs; results equal the backward kernel's bit for bit, except that
    grad_logit_bias is overwritten (not added to), and that with one initial state [H, D] for every
    sequence grad_inits is its float32 [H, D] gradient (each sequence's term rounded to combined's
    dtype, summed in batch order)."""
    rc = _scan_ckpt_backward(combined, inits, logit_bias, ckpt, grad_hq, grad_hk, grad_hv, grad_combined, grad_inits,
                             grad_logit_bias, NH, NKVH, da, r, use_sigmoid)
    _lib.check(rc, "ltvqkv_scan_bwd_ckpt")


def _ps_setup(ctx, inputs, output):
    x, weight, inits, logit_bias, NH, NKVH, da, r, use_sigmoid = inputs
    combined, hq, hk, hv, ckpt = output
    # `combined` is usually not used downstream: keep its gradient None instead of a zero tensor
    ctx.set_materialize_grads(False)
    ctx.mark_non_differentiable(ckpt)
    ctx.save_for_backward(x, weight, combined, inits, logit_bias, hq, hk, hv, ckpt)
    ctx.args = (NH, NKVH, da, r)
    ctx.use_sigmoid = use_sigmoid


def _ps_backward(ctx, grad_comb, grad_hq, grad_hk, grad_hv, _grad_ckpt):
    # the two reference backward kernels in sequence: scan backward into grad_combined (whose
    # [B, F, T] memory is the projection's grad_out), then the projection backward. Where the
    # forward wrote state checkpoints the scan backward replays its outputs from them (equal results,
    # less memory traffic) instead of reading them.
    # Only operators here (no library calls, no pointer checks): under torch.compile AOTAutograd
    # traces this function with fake tensors. The checkpoints are non-empty exactly where the
    # one-kernel forward ran, and that kernel's shapes are ones the checkpoint backward takes.
    x, weight, comb, inits, logit_bias, hq, hk, hv, ckpt = ctx.saved_tensors
    NH, NKVH, da, r = ctx.args
    B = x.shape[0]
    shared = inits.dim() == 2
    inits_k = inits.to(x.dtype) if shared else inits
    combined = comb.transpose(1, 2)
    grad_hq = torch.zeros_like(hq) if grad_hq is None else grad_hq
    grad_hk = torch.zeros_like(hk) if grad_hk is None else grad_hk
    grad_hv = torch.zeros_like(hv) if grad_hv is None else grad_hv
    grad_combined = torch.empty_like(combined)
    if ckpt.numel():
        grad_inits = (torch.empty(inits_k.shape, device=x.device, dtype=torch.float32) if shared
                      else torch.empty_like(inits_k, memory_format=torch.contiguous_format))
        grad_logit_bias = torch.empty_like(logit_bias, memory_format=torch.contiguous_format)
        torch.ops.nanochat_cuda.ltv_scan_ckpt_backward_kernel(combined, inits_k, logit_bias, ckpt, grad_hq, grad_hk,
                                                              grad_hv, grad_combined, grad_inits, grad_logit_bias, NH,
                                                              NKVH, da, r, ctx.use_sigmoid)
    else:
        ib = inits_k.unsqueeze(0).expand(B, -1, -1).contiguous() if shared else inits_k
        grad_inits = torch.empty_like(ib, memory_format=torch.contiguous_format)
        grad_logit_bias = torch.zeros_like(logit_bias, memory_format=torch.contiguous_format)
        torch.ops.nanochat_cuda.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_backward_kernel(
            combined, ib, logit_bias, hq, hk, hv, grad_hq, grad_hk, grad_hv, grad_combined, grad_inits,
            grad_logit_bias, NH, NKVH, da, r, 32, 2, 8, ctx.use_sigmoid)
        if shared:
            grad_inits = grad_inits.float().sum(0)
    if shared:
        grad_inits = grad_inits.to(inits.dtype)
    grad_out = grad_combined.transpose(1, 2)
    if grad_comb is not None:
        grad_out = grad_out + grad_comb
    grad_x = torch.empty_like(x, memory_format=torch.contiguous_format)
    grad_weight = torch.empty_like(weight, memory_format=torch.contiguous_format)
    torch.ops.nanochat_cuda.fused_linear_transpose_backward_kernel(x, weight, grad_out, grad_x, grad_weight)
    return (grad_x, grad_weight, grad_inits, grad_logit_bias) + (None,) * 5


torch.library.register_autograd("nanochat_cuda::ltv_proj_scan_cuda_op", _ps_backward, setup_context=_ps_setup)


@torch.library.register_fake("nanochat_cuda::ltv_proj_scan_cuda_op")
def _proj_scan_fake(x, weight, inits, logit_bias, NH, NKVH, da, r, use_sigmoid):
    B, T, _ = x.shape
    D = da * r
    F = (NH + 2 * NKVH) * (D + da)
    return (x.new_empty((B, F, T)), x.new_empty((B, NH, T, D)), x.new_empty((B, NKVH, T, D)),
            x.new_empty((B, NKVH, T, D)), x.new_empty(_ckpt_shape(x, NH, NKVH, da, r), dtype=torch.float32))


@torch.library.register_fake("nanochat_cuda::ltv_scan_ckpt_backward_kernel")
def _scan_ckpt_backward_fake(*args):
    return None


@torch.library.register_fake("nanochat_cuda::ltv_proj_scan_forward_kernel")
def _proj_scan_kernel_fake(*args):
    return None


# ------------------------------------------------------------------------------------------
# Rotary embedding + QK RMS-norm of the filtered q and k (the reference attention's prologue,
# nanochat/gpt.py:96-111, 224-230), fused
# ------------------------------------------------------------------------------------------
# F.rms_norm's default eps for bf16 and fp32 inputs: the epsilon of its fp32 compute type
_RMS_EPS = float(torch.finfo(torch.float32).eps)


def _rot_cs(cos, sin, q):
    if cos.dim() == 4:  # the model's [1, T, 1, D/2] rotary cache
        cos, sin = cos[0, :, 0, :], sin[0, :, 0, :]
    if cos.dtype != q.dtype:
        cos, sin = cos.to(q.dtype), sin.to(q.dtype)
    if cos.stride() != sin.stride():
        cos, sin = cos.contiguous(), sin.contiguous()
    return cos, sin


def _rot_check(q, k, cos):
    if q.dim() != 4 or k.dim() != 4 or q.shape[0] != k.shape[0] or q.shape[1] != k.shape[1] or \
            q.shape[3] != k.shape[3] or q.dtype != k.dtype:
        raise RuntimeError(f"q and k must be [B, T, heads, D] of one dtype, got {tuple(q.shape)}, {tuple(k.shape)}")
    T, D = q.shape[1], q.shape[3]
    if D % 2 == 0 and tuple(cos.shape) != (T, D // 2):
        raise RuntimeError(f"cos/sin must hold [T, D/2] = {(T, D // 2)} values, got {tuple(cos.shape)}")


def _head_major_like(x):
    B, T, H, D = x.shape
    return torch.empty((B, H, T, D), dtype=x.dtype, device=x.device).transpose(1, 2)


def _rotary_qk_norm(q, k, cos, sin):
    cos, sin = _rot_cs(cos, sin, q)
    _rot_check(q, k, cos)
    L = _lib.load()
    oq, ok = _head_major_like(q), _head_major_like(k)
    S = _lib.strides
    B, T, NH, D = q.shape
    rc = L.ltvqkv_rotary_qk_norm_fwd(_lib.dtype_code(q.dtype), q.data_ptr(), S(q.stride()), k.data_ptr(),
                                     S(k.stride()), cos.data_ptr(), sin.data_ptr(), S(cos.stride()), oq.data_ptr(),
                                     S(oq.stride()), ok.data_ptr(), S(ok.stride()), B, T, NH, k.shape[2], D,
                                     _RMS_EPS, _lib.stream_handle(q.device))
    _lib.check(rc, "ltvqkv_rotary_qk_norm_fwd")
    return oq, ok


def _rotary_qk_norm_backward_kernel(q, k, cos, sin, grad_q, grad_k):
    cos, sin = _rot_cs(cos, sin, q)
    _rot_check(q, k, cos)
    L = _lib.load()
    dq, dk = torch.empty_like(q), torch.empty_like(k)
    grad_q, grad_k = grad_q.to(q.dtype), grad_k.to(k.dtype)
    S = _lib.strides
    B, T, NH, D = q.shape
    rc = L.ltvqkv_rotary_qk_norm_bwd(_lib.dtype_code(q.dtype), q.data_ptr(), S(q.stride()), k.data_ptr(),
                                     S(k.stride()), cos.data_ptr(), sin.data_ptr(), S(cos.stride()),
                                     grad_q.data_ptr(), S(grad_q.stride()), grad_k.data_ptr(), S(grad_k.stride()),
                                     dq.data_ptr(), S(dq.stride()), dk.data_ptr(), S(dk.stride()), B, T, NH,
                                     k.shape[2], D, _RMS_EPS, _lib.stream_handle(q.device))
    _lib.check(rc, "ltvqkv_rotary_qk_norm_bwd")
    return dq, dk


def _rot_setup(ctx, inputs, output):
    q, k, cos, sin = inputs
    ctx.save_for_backward(q, k, cos, sin)


def _rot_backward(ctx, grad_oq, grad_ok):
    q, k, cos, sin = ctx.saved_tensors
    grad_oq = torch.zeros_like(q) if grad_oq is None else grad_oq
    grad_ok = torch.zeros_like(k) if grad_ok is None else grad_ok
    dq, dk = torch.ops.nanochat_cuda.ltv_rotary_qk_norm_backward(q, k, cos, sin, grad_oq, grad_ok)
    return dq, dk, None, None


torch.library.register_autograd("nanochat_cuda::ltv_rotary_qk_norm", _rot_backward, setup_context=_rot_setup)


@torch.library.register_fake("nanochat_cuda::ltv_rotary_qk_norm")
def _rot_fake(q, k, cos, sin):
    return _head_major_like(q), _head_major_like(k)


@torch.library.register_fake("nanochat_cuda::ltv_rotary_qk_norm_backward")
def _rot_bwd_fake(q, k, cos, sin, grad_q, grad_k):
    return torch.empty_like(q), torch.empty_like(k)


# ------------------------------------------------------------------------------------------
# Projection + scan forward with the attention's q / k prologue (rotary + RMS norm) in the scan's
# epilogue, and the matching checkpoint backward
# ------------------------------------------------------------------------------------------
def _rope_tables(cos, sin, x, D):
    """The rotary tables as [T, D/2] rows of x's dtype that the kernels read as bf16 pairs (unit
    element stride, even row stride, 4-byte aligned); the model's [1, T, 1, D/2] buffers and their
    position slices pass as views."""
    cos, sin = _rot_cs(cos, sin, x)
    T = x.shape[1]
    if tuple(cos.shape) != (T, D // 2) or tuple(sin.shape) != (T, D // 2):
        raise RuntimeError(f"cos/sin must hold [T, D/2] = {(T, D // 2)} values, got {tuple(cos.shape)}")

    def ok(t):
        return t.stride(1) == 1 and t.stride(0) % 2 == 0 and t.data_ptr() % 4 == 0

    if not (ok(cos) and ok(sin) and cos.stride() == sin.stride()):
        cos, sin = cos.contiguous(), sin.contiguous()
    return cos, sin


def _proj_scan_rope_op(x, weight, inits, logit_bias, cos, sin, NH, NKVH, da, r, use_sigmoid):
    """ltv_proj_scan_cuda_op whose q and k outputs are rotated and RMS-normalised (nanochat/gpt.py:
    224-230, `apply_rotary_emb` then `norm`): outputs equal ltv_proj_scan_cuda_op followed by
    ltv_rotary_qk_norm bit for bit. On the one-kernel shapes (ltv_proj_scan_cuda_op's checkpoint
    condition) the prologue runs inside the scan's epilogue and the raw q / k are never stored;
    elsewhere the two operators run in sequence (the fifth output is then empty)."""
    if not x.is_contiguous() or x.dim() != 3:
        raise RuntimeError("ltv_proj_scan_rope_norm_cuda_op requires a contiguous [B, T, C] x")
    shape = _ckpt_shape(x, NH, NKVH, da, r)
    if len(shape) != 4:
        combined, q, k, v, ckpt = _proj_scan_op(x, weight, inits, logit_bias, NH, NKVH, da, r, use_sigmoid)
        qn, kn = _rotary_qk_norm(q.transpose(1, 2), k.transpose(1, 2), cos, sin)
        return combined, qn.transpose(1, 2), kn.transpose(1, 2), v, ckpt
    L = _lib.load()
    B, T, C = x.shape
    H = NH + 2 * NKVH
    D = da * r
    F = H * (D + da)
    cos, sin = _rope_tables(cos, sin, x, D)
    if x.data_ptr() % 16:
        x = x.clone()
    w = (weight if weight.dtype == x.dtype else weight.to(x.dtype)).contiguous()
    if w.data_ptr() % 16:
        w = w.clone()
    if tuple(w.shape) != (F, C):
        raise RuntimeError(f"weight must be [{F}, {C}], got {tuple(w.shape)}")
    shared = inits.dim() == 2
    inits_k = (inits.to(x.dtype) if shared else inits).contiguous()
    kw = dict(device=x.device, dtype=x.dtype)
    combined = torch.empty((B, F, T), **kw)
    _check_scan_inputs(combined.transpose(1, 2), inits_k.unsqueeze(0).expand(B, -1, -1) if shared else inits_k,
                       logit_bias, NH, NKVH, da, r)
    logit_bias = logit_bias.contiguous()
    out_q = torch.empty((B, NH, T, D), **kw)
    out_k = torch.empty((B, NKVH, T, D), **kw)
    out_v = torch.empty((B, NKVH, T, D), **kw)
    ckpt = torch.empty(shape, device=x.device, dtype=torch.float32)
    nbytes = max(L.ltvqkv_scan_workspace_bytes(B, T, NH, NKVH, da, r), L.ltvqkv_gemm_workspace_bytes())
    ws = _lib.workspace(x.device, nbytes)
    rc = L.ltvqkv_proj_scan_fwd_ckpt_rope(
        _lib.dtype_code(x.dtype), x.data_ptr(), w.data_ptr(), inits_k.data_ptr(), 0 if shared else H * D,
        logit_bias.data_ptr(), combined.data_ptr(), out_q.data_ptr(), out_k.data_ptr(), out_v.data_ptr(),
        ckpt.data_ptr(), cos.data_ptr(), sin.data_ptr(), cos.stride(0), _RMS_EPS, B, T, C, NH, NKVH, da, r,
        int(bool(use_sigmoid)), ws.data_ptr(), ws.numel(), _lib.stream_handle(x.device))
    _lib.check(rc, "ltvqkv_proj_scan_fwd_ckpt_rope")
    return combined, out_q, out_k, out_v, ckpt


def _rotary_qk_norm_ckpt_backward(combined, inits, logit_bias, ckpt, cos, sin, grad_q, grad_k, NH, NKVH, da, r,
                                  use_sigmoid):
    """Gradients of the raw q / k ([B, heads, T, D], head-major) from those of the rotated, normalised
    q / k that ltv_proj_scan_rope_norm_cuda_op returned, the raw values replayed from its state
    checkpoints: ltv_rotary_qk_norm_backward's results on the raw outputs, bit for bit."""
    L = _lib.load()
    B, T, _ = combined.shape
    H, D = NH + 2 * NKVH, da * r
    shared = inits.dim() == 2
    _check_scan_inputs(combined, inits.unsqueeze(0).expand(B, -1, -1) if shared else inits, logit_bias, NH, NKVH,
                       da, r)
    comb = combined.transpose(1, 2)  # the [B, F, T] projection buffer
    if not comb.is_contiguous():
        raise RuntimeError("combined must be the transposed view of a contiguous [B, F, T] buffer")
    cos, sin = _rope_tables(cos, sin, combined.new_empty((B, T, 0)), D)
    inits = inits.contiguous()
    logit_bias = logit_bias.contiguous()
    if ckpt.dtype != torch.float32 or not ckpt.is_contiguous() or tuple(ckpt.shape) != (B, H, T // 32, D):
        raise RuntimeError("ckpt must be the forward's contiguous [B, H, T / 32, D] float32 checkpoints")

    def pairs(g):
        st = g.stride()
        ok = st[3] == 1 and all(x % 2 == 0 for x in st[:3]) and g.data_ptr() % 4 == 0
        return g if ok and g.dtype == combined.dtype else g.to(combined.dtype).contiguous()

    grad_q, grad_k = pairs(grad_q), pairs(grad_k)
    dq = torch.empty((B, NH, T, D), device=combined.device, dtype=combined.dtype)
    dk = torch.empty((B, NKVH, T, D), device=combined.device, dtype=combined.dtype)
    S = _lib.strides
    rc = L.ltvqkv_rotary_qk_norm_bwd_ckpt(
        _lib.dtype_code(combined.dtype), comb.data_ptr(), inits.data_ptr(), 0 if shared else H * D,
        logit_bias.data_ptr(), ckpt.data_ptr(), cos.data_ptr(), sin.data_ptr(), cos.stride(0), _RMS_EPS,
        grad_q.data_ptr(), S(grad_q.stride()), grad_k.data_ptr(), S(grad_k.stride()), dq.data_ptr(), S(dq.stride()),
        dk.data_ptr(), S(dk.stride()), B, T, NH, NKVH, da, r, int(bool(use_sigmoid)), _lib.stream_handle(combined.device))
    _lib.check(rc, "ltvqkv_rotary_qk_norm_bwd_ckpt")
    return dq, dk


def _psr_setup(ctx, inputs, output):
    x, weight, inits, logit_bias, cos, sin, NH, NKVH, da, r, use_sigmoid = inputs
    combined, oq, ok, ov, ckpt = output
    ctx.set_materialize_grads(False)
    ctx.mark_non_differentiable(ckpt)
    ctx.save_for_backward(x, weight, combined, inits, logit_bias, cos, sin, ckpt)
    ctx.args = (NH, NKVH, da, r)
    ctx.out_shapes = (oq.shape, ok.shape, ov.shape)
    ctx.use_sigmoid = use_sigmoid


def _psr_backward(ctx, grad_comb, grad_q, grad_k, grad_v, _grad_ckpt):
    # the checkpoint backward with the rotary + norm backward of q / k folded in, then the
    # projection backward (operators only: AOTAutograd traces this with fake tensors)
    x, weight, comb, inits, logit_bias, cos, sin, ckpt = ctx.saved_tensors
    NH, NKVH, da, r = ctx.args
    B, T = x.shape[0], x.shape[1]
    shared = inits.dim() == 2
    inits_k = inits.to(x.dtype) if shared else inits
    combined = comb.transpose(1, 2)
    zs = [x.new_zeros(sh) for sh in ctx.out_shapes]
    grad_q = zs[0] if grad_q is None else grad_q
    grad_k = zs[1] if grad_k is None else grad_k
    grad_v = zs[2] if grad_v is None else grad_v
    grad_combined = torch.empty_like(combined)
    if ckpt.numel():
        # the raw q / k gradients (raw outputs replayed from the checkpoints), then the checkpoint
        # scan backward as for ltv_proj_scan_cuda_op
        dq, dk = torch.ops.nanochat_cuda.ltv_rotary_qk_norm_ckpt_backward(combined, inits_k, logit_bias, ckpt, cos,
                                                                          sin, grad_q, grad_k, NH, NKVH, da, r,
                                                                          ctx.use_sigmoid)
        grad_inits = (torch.empty(inits_k.shape, device=x.device, dtype=torch.float32) if shared
                      else torch.empty_like(inits_k, memory_format=torch.contiguous_format))
        grad_logit_bias = torch.empty_like(logit_bias, memory_format=torch.contiguous_format)
        torch.ops.nanochat_cuda.ltv_scan_ckpt_backward_kernel(combined, inits_k, logit_bias, ckpt, dq, dk, grad_v,
                                                              grad_combined, grad_inits, grad_logit_bias, NH, NKVH,
                                                              da, r, ctx.use_sigmoid)
    else:
        # the two-operator forward's raw outputs, recomputed (the same kernel, so the same values),
        # then the rotary backward and the scan backward as their own operators
        ib = inits_k.unsqueeze(0).expand(B, -1, -1).contiguous() if shared else inits_k
        hq, hk, hv = (x.new_empty(sh) for sh in ctx.out_shapes)
        torch.ops.nanochat_cuda.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_forward_kernel(
            combined, ib, logit_bias, hq, hk, hv, T, NH, NKVH, da, r, 8, 8, 4, ctx.use_sigmoid)
        dq, dk = torch.ops.nanochat_cuda.ltv_rotary_qk_norm_backward(hq.transpose(1, 2), hk.transpose(1, 2), cos, sin,
                                                                     grad_q.transpose(1, 2), grad_k.transpose(1, 2))
        grad_inits = torch.empty_like(ib, memory_format=torch.contiguous_format)
        grad_logit_bias = torch.zeros_like(logit_bias, memory_format=torch.contiguous_format)
        torch.ops.nanochat_cuda.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_backward_kernel(
            combined, ib, logit_bias, hq, hk, hv, dq.transpose(1, 2), dk.transpose(1, 2), grad_v, grad_combined,
            grad_inits, grad_logit_bias, NH, NKVH, da, r, 32, 2, 8, ctx.use_sigmoid)
        if shared:
            grad_inits = grad_inits.float().sum(0)
    if shared:
        grad_inits = grad_inits.to(inits.dtype)
    grad_out = grad_combined.transpose(1, 2)
    if grad_comb is not None:
        grad_out = grad_out + grad_comb
    grad_x = torch.empty_like(x, memory_format=torch.contiguous_format)
    grad_weight = torch.empty_like(weight, memory_format=torch.contiguous_format)
    torch.ops.nanochat_cuda.fused_linear_transpose_backward_kernel(x, weight, grad_out, grad_x, grad_weight)
    return (grad_x, grad_weight, grad_inits, grad_logit_bias, None, None) + (None,) * 5


torch.library.register_autograd("nanochat_cuda::ltv_proj_scan_rope_norm_cuda_op", _psr_backward,
                                setup_context=_psr_setup)


@torch.library.register_fake("nanochat_cuda::ltv_proj_scan_rope_norm_cuda_op")
def _proj_scan_rope_fake(x, weight, inits, logit_bias, cos, sin, NH, NKVH, da, r, use_sigmoid):
    B, T, _ = x.shape
    D = da * r
    F = (NH + 2 * NKVH) * (D + da)
    return (x.new_empty((B, F, T)), x.new_empty((B, NH, T, D)), x.new_empty((B, NKVH, T, D)),
            x.new_empty((B, NKVH, T, D)), x.new_empty(_ckpt_shape(x, NH, NKVH, da, r), dtype=torch.float32))


@torch.library.register_fake("nanochat_cuda::ltv_rotary_qk_norm_ckpt_backward")
def _rotary_qk_norm_ckpt_backward_fake(combined, inits, logit_bias, ckpt, cos, sin, grad_q, grad_k, NH, NKVH, da, r,
                                       use_sigmoid):
    B, T, _ = combined.shape
    D = da * r
    return combined.new_empty((B, NH, T, D)), combined.new_empty((B, NKVH, T, D))


# ------------------------------------------------------------------------------------------
# Decode step
# ------------------------------------------------------------------------------------------
def _decode_step(x, weight, logit_bias, prev_q, prev_k, prev_v, init_param, NH, NKVH, da, r, use_sigmoid):
    L = _lib.load()
    if x.dim() == 3:
        if x.shape[1] != 1:
            raise RuntimeError("ltv_decode_step takes one token per sequence")
        x = x.reshape(x.shape[0], x.shape[2])
    x = x.contiguous()
    B, C = x.shape
    D = da * r
    H = NH + 2 * NKVH
    w = (weight if weight.dtype == x.dtype else weight.to(x.dtype)).contiguous()
    if tuple(w.shape) != (H * (D + da), C):
        raise RuntimeError(f"weight must be [{H * (D + da)}, {C}], got {tuple(w.shape)}")
    logit_bias = logit_bias.contiguous()
    init = (init_param if init_param.dtype == x.dtype else init_param.to(x.dtype)).contiguous()
    kw = dict(device=x.device, dtype=x.dtype)
    oq, ok, ov = torch.empty((B, NH, D), **kw), torch.empty((B, NKVH, D), **kw), torch.empty((B, NKVH, D), **kw)
    S = _lib.strides
    if prev_q is not None:
        for p, n in ((prev_q, NH), (prev_k, NKVH), (prev_v, NKVH)):
            if p is None or tuple(p.shape) != (B, n, D) or p.dtype != x.dtype:
                raise RuntimeError("previous states must be [B, heads, D] in x's dtype")
        pargs = [prev_q.data_ptr(), S(prev_q.stride()), prev_k.data_ptr(), S(prev_k.stride()),
                 prev_v.data_ptr(), S(prev_v.stride())]
    else:
        pargs = [None, None, None, None, None, None]
    rc = L.ltvqkv_decode_step(_lib.dtype_code(x.dtype), x.data_ptr(), w.data_ptr(), logit_bias.data_ptr(), *pargs,
                              init.data_ptr(), oq.data_ptr(), S(oq.stride()), ok.data_ptr(), S(ok.stride()),
                              ov.data_ptr(), S(ov.stride()), B, C, NH, NKVH, da, r, int(bool(use_sigmoid)),
                              _lib.stream_handle(x.device))
    _lib.check(rc, "ltvqkv_decode_step")
    return oq, ok, ov


def _decode_step_inplace(x, weight, logit_bias, state_q, state_k, state_v, NH, NKVH, da, r, use_sigmoid):
    """ltv_decode_step writing the new states over the previous ones (a cache's states updated in
    place: one launch per layer-step, no copies)."""
    L = _lib.load()
    if x.dim() == 3:
        if x.shape[1] != 1:
            raise RuntimeError("ltv_decode_step_ takes one token per sequence")
        x = x.reshape(x.shape[0], x.shape[2])
    x = x.contiguous()
    B, C = x.shape
    D = da * r
    H = NH + 2 * NKVH
    w = (weight if weight.dtype == x.dtype else weight.to(x.dtype)).contiguous()
    if tuple(w.shape) != (H * (D + da), C):
        raise RuntimeError(f"weight must be [{H * (D + da)}, {C}], got {tuple(w.shape)}")
    for p, n in ((state_q, NH), (state_k, NKVH), (state_v, NKVH)):
        if tuple(p.shape) != (B, n, D) or p.dtype != x.dtype:
            raise RuntimeError("states must be [B, heads, D] in x's dtype")
    logit_bias = logit_bias.contiguous()
    S = _lib.strides
    sq, sk, sv = S(state_q.stride()), S(state_k.stride()), S(state_v.stride())
    rc = L.ltvqkv_decode_step(_lib.dtype_code(x.dtype), x.data_ptr(), w.data_ptr(), logit_bias.data_ptr(),
                              state_q.data_ptr(), sq, state_k.data_ptr(), sk, state_v.data_ptr(), sv, None,
                              state_q.data_ptr(), sq, state_k.data_ptr(), sk, state_v.data_ptr(), sv,
                              B, C, NH, NKVH, da, r, int(bool(use_sigmoid)), _lib.stream_handle(x.device))
    _lib.check(rc, "ltvqkv_decode_step")


@torch.library.register_fake("nanochat_cuda::ltv_decode_step_")
def _decode_step_inplace_fake(*args):
    return None


@torch.library.register_fake("nanochat_cuda::ltv_decode_step")
def _decode_step_fake(x, weight, logit_bias, prev_q, prev_k, prev_v, init_param, NH, NKVH, da, r, use_sigmoid):
    B = x.shape[0]
    D = da * r
    return x.new_empty((B, NH, D)), x.new_empty((B, NKVH, D)), x.new_empty((B, NKVH, D))


# ------------------------------------------------------------------------------------------
# Registration (explicit calls: the decorator form does not hand the function back)
# ------------------------------------------------------------------------------------------
torch.library.impl(f"nanochat_cuda::{_SCAN_FWD}", "CUDA", _scan_forward_kernel)
torch.library.impl(f"nanochat_cuda::{_SCAN_OP}", "CUDA", _scan_op)
torch.library.impl(f"nanochat_cuda::{_SCAN_BWD}", "CUDA", _scan_backward_kernel)
torch.library.impl("nanochat_cuda::fused_linear_transpose", "CUDA", _fused_linear_transpose)
torch.library.impl("nanochat_cuda::fused_linear_transpose_cuda_op", "CUDA", _fused_linear_transpose_op)
torch.library.impl("nanochat_cuda::fused_linear_transpose_backward_kernel", "CUDA", _fused_linear_transpose_backward_kernel)
torch.library.impl("nanochat_cuda::ltv_decode_step", "CUDA", _decode_step)
torch.library.impl("nanochat_cuda::ltv_decode_step_", "CUDA", _decode_step_inplace)
torch.library.impl("nanochat_cuda::ltv_rotary_qk_norm", "CUDA", _rotary_qk_norm)
torch.library.impl("nanochat_cuda::ltv_rotary_qk_norm_backward", "CUDA", _rotary_qk_norm_backward_kernel)
for _kind in ("blelloch", "sequential"):
    torch.library.impl(f"nanochat_cuda::{_LB.format(_kind, 'op')}", "CUDA", _lb_op)
    torch.library.impl(f"nanochat_cuda::{_LB.format(_kind, 'forward_kernel')}", "CUDA", _lb_forward_kernel)
    torch.library.impl(f"nanochat_cuda::{_LB.format(_kind, 'backward_kernel')}", "CUDA", _lb_backward_kernel)
torch.library.impl("nanochat_cuda::ltv_proj_scan_forward_kernel", "CUDA", _proj_scan_forward_kernel)
torch.library.impl("nanochat_cuda::ltv_proj_scan_cuda_op", "CUDA", _proj_scan_op)
torch.library.impl("nanochat_cuda::ltv_scan_ckpt_backward_kernel", "CUDA", _scan_ckpt_backward_kernel)
torch.library.impl("nanochat_cuda::ltv_proj_scan_rope_norm_cuda_op", "CUDA", _proj_scan_rope_op)
torch.library.impl("nanochat_cuda::ltv_rotary_qk_norm_ckpt_backward", "CUDA", _rotary_qk_norm_ckpt_backward)



# ------------------------------------------------------------------------------------------
# Functional wrappers (reference nanochat/ops/ltv_cuda_ops.py:256-299)
# ------------------------------------------------------------------------------------------
def fused_linear_transpose(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """Returns weight @ x^T per batch, shaped (B, F, T), contiguous."""
    return torch.ops.nanochat_cuda.fused_linear_transpose_cuda_op(x, weight)


def ltv_cuda_fused_concat_head_major_register_cast_blelloch_scan(
        combined: torch.Tensor, inits: torch.Tensor, logit_bias: torch.Tensor, NH: int, NKVH: int, da: int, r: int,
        scan_threads_forward: int, r_threads_forward: int, r_items_forward: int, scan_threads_backward: int,
        r_threads_backward: int, r_items_backward: int, use_sigmoid: bool):
    return torch.ops.nanochat_cuda.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_op(
        combined, inits, logit_bias, NH, NKVH, da, r, scan_threads_forward, r_threads_forward, r_items_forward,
        scan_threads_backward, r_threads_backward, r_items_backward, use_sigmoid)


def ltv_decode_step(x: torch.Tensor, weight: torch.Tensor, logit_bias: torch.Tensor,
                    prev_q: Optional[torch.Tensor], prev_k: Optional[torch.Tensor], prev_v: Optional[torch.Tensor],
                    init_param: torch.Tensor, NH: int, NKVH: int, da: int, r: int, use_sigmoid: bool = True):
    """One incremental filter step for x [B, C] (or [B, 1, C]); returns the new states."""
    return torch.ops.nanochat_cuda.ltv_decode_step(x, weight, logit_bias, prev_q, prev_k, prev_v, init_param, NH,
                                                    NKVH, da, r, use_sigmoid)


def ltv_proj_scan(x: torch.Tensor, weight: torch.Tensor, inits: torch.Tensor, logit_bias: torch.Tensor, NH: int,
                  NKVH: int, da: int, r: int, use_sigmoid: bool = True):
    """Projection and scan forward in one call; returns (combined [B, F, T], q, k, v [B, heads, T, D]).
    `inits`: the initial state of every sequence [B, H, D] (x's dtype), or one state [H, D] shared by
    the batch (any float dtype; its gradient is summed over the batch in the kernel)."""
    return torch.ops.nanochat_cuda.ltv_proj_scan_cuda_op(x, weight, inits, logit_bias, NH, NKVH, da, r,
                                                         use_sigmoid)[:4]


def ltv_proj_scan_rope_norm(x: torch.Tensor, weight: torch.Tensor, inits: torch.Tensor, logit_bias: torch.Tensor,
                            cos: torch.Tensor, sin: torch.Tensor, NH: int, NKVH: int, da: int, r: int,
                            use_sigmoid: bool = True):
    """The filter's projection and scan followed by the attention's q / k prologue
    (nanochat/gpt.py:224-230: apply_rotary_emb, then norm): returns (q, k, v) [B, heads, T, D] with q
    and k rotated and RMS-normalised, v the raw filter output. The one-kernel shapes run it inside the
    scan's epilogue (and the backward's replay), others as ltv_proj_scan then ltv_rotary_qk_norm;
    the results are the same bit for bit. cos / sin: the model's rotary tables for these positions,
    [T, D/2] or [1, T, 1, D/2]."""
    return torch.ops.nanochat_cuda.ltv_proj_scan_rope_norm_cuda_op(x.contiguous(), weight, inits, logit_bias, cos,
                                                                   sin, NH, NKVH, da, r, use_sigmoid)[1:4]


def rotary_qk_norm(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """apply_rotary_emb then norm on q and k (nanochat/gpt.py:224-230) in one pass each way;
    q, k [B, T, heads, D] -> [B, T, heads, D] views of head-major storage (the attention's
    transpose(1, 2) is then contiguous)."""
    return torch.ops.nanochat_cuda.ltv_rotary_qk_norm(q, k, cos, sin)
