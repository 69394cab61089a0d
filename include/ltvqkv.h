/*
 * ltvqkv.h — C ABI of the B200 filtered-QKV hot path (libltvqkv.so).
 *
 * The filtered-QKV layer of nanochat-filter computes, per attention layer,
 *   combined[b, f, t] = sum_c W[f, c] * x[b, t, c]                      (projection)
 *   alpha[b, t, h, g] = sigmoid(combined[b, h*(D+Da)+D+g, t] + logit_bias[h, g])
 *   h[t] = (1 - alpha[t]) * h[t-1] + alpha[t] * u[t]                     (EWMA scan)
 * with u = the D value rows of head h, alpha shared by groups of r channels
 * (Da = D / r logit rows per head, head-major rows: [h0 values | h0 logits | h1 ...],
 * Q heads, then K heads, then V heads), h[-1] = inits[b, h, :].
 *
 * Every entry point:
 *   - takes device pointers, element strides (int64, in elements) and sizes;
 *   - enqueues work on `stream` (a cudaStream_t, NULL = legacy default stream)
 *     and returns without synchronising;
 *   - never allocates device memory: the caller passes outputs and, where a kernel
 *     needs scratch, a workspace of at least the size the matching *_workspace_bytes
 *     query returns. A workspace must be zero-filled once before its first use; each
 *     call leaves it ready for the next call on the same stream. Calls that may run
 *     concurrently on the GPU must use different workspaces.
 *   - returns LTVQKV_OK or an error status (never aborts the process).
 *
 * dtype codes: LTVQKV_DTYPE_F32 (float) or LTVQKV_DTYPE_BF16 (bfloat16 storage,
 * fp32 arithmetic). logit_bias and its gradient are always fp32.
 */
#ifndef LTVQKV_H_
#define LTVQKV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LTVQKV_ABI_VERSION 1

#if defined(__GNUC__)
#define LTVQKV_API __attribute__((visibility("default")))
#else
#define LTVQKV_API
#endif

enum ltvqkv_dtype {
  LTVQKV_DTYPE_F32 = 0,
  LTVQKV_DTYPE_BF16 = 1,
};

enum ltvqkv_status {
  LTVQKV_OK = 0,
  LTVQKV_ERR_INVALID_ARG = 1, /* null pointer where data is required, negative size */
  LTVQKV_ERR_SHAPE = 2,       /* sizes inconsistent or beyond what the kernels support */
  LTVQKV_ERR_STRIDE = 3,      /* a layout the kernel does not accept */
  LTVQKV_ERR_DTYPE = 4,       /* unknown dtype code */
  LTVQKV_ERR_ALIGN = 5,       /* pointer alignment a kernel needs is not met */
  LTVQKV_ERR_LAUNCH = 6,      /* CUDA launch or runtime error */
  LTVQKV_ERR_TIMEOUT = 7,     /* a bounded device-side wait gave up (read by ltvqkv_workspace_error) */
  LTVQKV_ERR_WORKSPACE = 8,   /* workspace missing or smaller than required */
  LTVQKV_ERR_UNSUPPORTED = 9, /* valid request this build does not implement */
  LTVQKV_ERR_TOO_LARGE = 10,  /* problem needs more scratch than ltvqkv_scan_fwd_noalloc's fixed array */
};

/* Library ABI version (LTVQKV_ABI_VERSION). */
LTVQKV_API int ltvqkv_abi_version(void);

/* Static, human-readable text for a status code. */
LTVQKV_API const char* ltvqkv_status_string(int status);

/* Text of the last CUDA error seen by this library on the calling thread ("" if none). */
LTVQKV_API const char* ltvqkv_last_cuda_error(void);

/* ------------------------------------------------------------------------------------------
 * Scan: replaces cpp_ewma_cuda.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_forward
 * (reference cpp_ewma/src/ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_forward.cu:532-552,
 * bound in cpp_ewma/src/bindings.cpp; called from
 * nanochat/ops/ltv_cuda_fused_concat_head_major_register_cast_blelloch_scan.py:35-71).
 *
 * combined: [B, T, F] with element strides (sc_b, sc_t, sc_e), F = H*(D+Da), H = NH+2*NKVH,
 *           D = Da*r. Any strides are accepted; (F*T, 1, T) (the transposed projection output)
 *           and (T*F, F, 1) take vectorised paths.
 * inits:    [B, H, D] contiguous, same dtype as combined.
 * out_q/k/v:[B, NH, T, D] / [B, NKVH, T, D] / [B, NKVH, T, D] contiguous, same dtype.
 * use_sigmoid: 1 -> alpha = sigmoid(logit + bias); 0 -> alpha = logit + bias.
 * ------------------------------------------------------------------------------------------ */
LTVQKV_API size_t ltvqkv_scan_workspace_bytes(int B, int T, int NH, int NKVH, int Da, int r);

LTVQKV_API int ltvqkv_scan_fwd(int dtype,
                    const void* combined, int64_t sc_b, int64_t sc_t, int64_t sc_e,
                    const void* inits, const float* logit_bias,
                    void* out_q, void* out_k, void* out_v,
                    int B, int T, int NH, int NKVH, int Da, int r, int use_sigmoid,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free variant of ltvqkv_scan_fwd (no counterpart in the reference). For callers
 * that cannot allocate device memory or hand out a workspace on the call path — plugin hosts
 * and serving runtimes that own all device memory under a fixed plan, or foreign-language
 * callers without an allocator. Same arguments and results as ltvqkv_scan_fwd minus the
 * workspace: the scan's scratch (chunk aggregates, carries, look-back flags) is a fixed 32 MiB
 * file-scope device array in the library
 * (held on every GPU that loads the library until exit). Shapes whose forward scratch exceeds
 * it return LTVQKV_ERR_TOO_LARGE (D = 128, r = 128: about 1 KiB per (batch, head, 64-token
 * chunk) tile, so up to about 32 k tiles; B=4, T=16384, 8+8+8 heads needs 24 576 and fits). Calls no cudaMalloc/cudaFree.
 * The first call on a device looks up the array's address (may load the library's device code
 * there) and should come before any stream capture. All calls share the array and each clears
 * its counters and flags on `stream`: calls that overlap on the GPU race. A bounded device-side
 * wait that gives up inside a call records LTVQKV_ERR_TIMEOUT in the array's error word, which
 * later calls leave set: read it with ltvqkv_scan_noalloc_error. */
LTVQKV_API int ltvqkv_scan_fwd_noalloc(int dtype,
                    const void* combined, int64_t sc_b, int64_t sc_t, int64_t sc_e,
                    const void* inits, const float* logit_bias,
                    void* out_q, void* out_k, void* out_v,
                    int B, int T, int NH, int NKVH, int Da, int r, int use_sigmoid,
                    void* stream);

/* Reads and clears the error word of ltvqkv_scan_fwd_noalloc's array on the current device
 * (synchronises `stream`): *err_out receives LTVQKV_OK, or LTVQKV_ERR_TIMEOUT when a bounded
 * device-side wait of an earlier allocation-free call gave up (its outputs are then incomplete).
 * No reference counterpart: the allocation-free entry point has none. Allocates nothing. */
LTVQKV_API int ltvqkv_scan_noalloc_error(void* stream, uint32_t* err_out);

/* Scan backward: replaces cpp_ewma_cuda.ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_backward
 * (reference cpp_ewma/src/ltv_fused_concat_head_major_register_cast_blelloch_scan_cuda_backward.cu:882-976;
 * called from nanochat/ops/ltv_cuda_fused_concat_head_major_register_cast_blelloch_scan.py:145-193).
 *
 * h_strides / g_strides: 4 element strides (b, h, t, d) for each of hq, hk, hv (saved forward
 * outputs) and grad_hq, grad_hk, grad_hv (upstream gradients); any strides are accepted.
 * grad_combined: [B, T, F] with strides (gc_b, gc_t, gc_e) — written for every element
 *                (value channels: du = alpha*g_hat; logit channels: sum over the r channels
 *                of the group of d_alpha * alpha*(1-alpha)).
 * grad_inits:    [B, H, D] contiguous, written.
 * grad_logit_bias: [H, Da] fp32, ACCUMULATED into (+=), as the reference's atomicAdd is.
 * Deterministic: no floating-point atomics.
 */
LTVQKV_API int ltvqkv_scan_bwd(int dtype,
                    const void* combined, int64_t sc_b, int64_t sc_t, int64_t sc_e,
                    const void* inits, const float* logit_bias,
                    const void* hq, const int64_t* hq_strides,
                    const void* hk, const int64_t* hk_strides,
                    const void* hv, const int64_t* hv_strides,
                    const void* grad_hq, const int64_t* gq_strides,
                    const void* grad_hk, const int64_t* gk_strides,
                    const void* grad_hv, const int64_t* gv_strides,
                    void* grad_combined, int64_t gc_b, int64_t gc_t, int64_t gc_e,
                    void* grad_inits, float* grad_logit_bias,
                    int B, int T, int NH, int NKVH, int Da, int r, int use_sigmoid,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Scan backward from state checkpoints: ltvqkv_scan_bwd without the forward's outputs hq/hk/hv.
 * ckpt is what ltvqkv_proj_scan_fwd_ckpt wrote for the same combined, inits and logit_bias; the
 * kernel replays each 32-token chunk's outputs from it (the forward's own arithmetic, so results
 * equal ltvqkv_scan_bwd's bit for bit) and reads 8 KB less per chunk of D = 128. Taken by bf16,
 * D = 128, T % 32 == 0, B * H >= 2 * (SM count) and the production layouts ltvqkv_scan_bwd's
 * row-streaming kernel needs; other requests return LTVQKV_ERR_UNSUPPORTED before anything is
 * launched. No reference function corresponds (the reference always reads the outputs).
 * Differences from ltvqkv_scan_bwd: grad_logit_bias is overwritten (not added to); inits_bs is the
 * element distance between the sequences' initial states, H * D (inits [B, H, D]) or 0 (one state
 * [H, D] for every sequence, the training case), and with 0 grad_inits is fp32 [H, D]: the
 * per-sequence gradients, each rounded to dtype, summed in batch order. */
LTVQKV_API int ltvqkv_scan_bwd_ckpt(int dtype,
                    const void* combined, int64_t sc_b, int64_t sc_t, int64_t sc_e,
                    const void* inits, int64_t inits_bs, const float* logit_bias, const float* ckpt,
                    const void* grad_hq, const int64_t* gq_strides,
                    const void* grad_hk, const int64_t* gk_strides,
                    const void* grad_hv, const int64_t* gv_strides,
                    void* grad_combined, int64_t gc_b, int64_t gc_t, int64_t gc_e,
                    void* grad_inits, float* grad_logit_bias,
                    int B, int T, int NH, int NKVH, int Da, int r, int use_sigmoid,
                    void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------
 * Look-back scan: replaces cpp_ewma_cuda.ltv_look_back_fused_concat_head_major_register_cast_
 * {blelloch,sequential}_scan_cuda_{forward,backward} (reference cpp_ewma/src/ltv_look_back_*.cu;
 * semantics nanochat/ops/ltv_reference_ops.py:37-124). Tokens are split into chunks [0, P),
 * [P + (i-1) Q, P + i Q); each chunk's outputs come from the recurrence restarted from the initial
 * state K - 1 tokens before the chunk (those warm-up states are not output). P >= T is the plain
 * scan. Arguments as ltvqkv_scan_fwd / ltvqkv_scan_bwd plus P, Q, K (>= 1); outputs q/k/v are
 * contiguous [B, heads, T, D]; D = Da * r <= 1024. The backward's workspace holds per-(batch,
 * head) bias partials (ltvqkv_lookback_workspace_bytes); grad_logit_bias is accumulated into
 * (zero it first), grad_combined and grad_inits are overwritten. fp32 follows the reference
 * oracle's operation order (separately rounded products and sums, later chunks' contributions
 * first). A warm-up prefix longer than about 13k tokens (D = 128) returns LTVQKV_ERR_TOO_LARGE. */
LTVQKV_API size_t ltvqkv_lookback_workspace_bytes(int B, int NH, int NKVH, int Da);

/* Workspace for ltvqkv_lookback_scan_bwd that also lets bf16 problems whose warm-up prefix is no
 * longer than any chunk (K - 1 <= min(P, Q), K - 1 <= 64, more than one chunk, D + Da <= 256,
 * r % 32 == 0) in the projection buffer's transposed layout (sc_t = gc_t = 1, T, the row and batch
 * strides multiples of 8, both buffers 16-byte aligned) take the chunk-parallel backward: one CTA per (row, chunk) — the chunks restart from the initial state, so
 * their backward passes are independent — and a fix-up pass that adds the two contributions of every
 * token reached by two chunks in the sequential order (later chunk first, each rounded to bf16) and
 * sums the initial-state gradients over the chunks in descending order. Same grad_combined and
 * grad_inits as the sequential form; the logit-bias sum over tokens is associated per chunk. A
 * workspace of ltvqkv_lookback_workspace_bytes() keeps the sequential form. Zero-filled once. */
LTVQKV_API size_t ltvqkv_lookback_bwd_workspace_bytes(int B, int T, int NH, int NKVH, int Da, int r,
                    int64_t P, int64_t Q, int64_t K);
LTVQKV_API int ltvqkv_lookback_scan_fwd(int dtype,
                    const void* combined, int64_t sc_b, int64_t sc_t, int64_t sc_e,
                    const void* inits, const float* logit_bias,
                    void* out_q, void* out_k, void* out_v,
                    int B, int T, int NH, int NKVH, int Da, int r,
                    int64_t P, int64_t Q, int64_t K, int use_sigmoid, void* stream);
LTVQKV_API int ltvqkv_lookback_scan_bwd(int dtype,
                    const void* combined, int64_t sc_b, int64_t sc_t, int64_t sc_e,
                    const void* inits, const float* logit_bias,
                    const void* hq, const int64_t* hq_strides,
                    const void* hk, const int64_t* hk_strides,
                    const void* hv, const int64_t* hv_strides,
                    const void* grad_hq, const int64_t* gq_strides,
                    const void* grad_hk, const int64_t* gk_strides,
                    const void* grad_hv, const int64_t* gv_strides,
                    void* grad_combined, int64_t gc_b, int64_t gc_t, int64_t gc_e,
                    void* grad_inits, float* grad_logit_bias,
                    int B, int T, int NH, int NKVH, int Da, int r,
                    int64_t P, int64_t Q, int64_t K, int use_sigmoid,
                    void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------
 * Consumer prologue of the filtered q and k: rotary embedding then QK RMS-norm, fused. Replaces
 * the reference attention's apply_rotary_emb + norm on q and k (nanochat/gpt.py:96-111, 224-230;
 * no reference C function). q [B, T, NH, D], k [B, T, NKVH, D], outputs and gradients with any
 * element strides (4 per tensor: b, t, head, d); cos/sin [T, D/2] in q's dtype (2 strides: t, j);
 * eps: F.rms_norm's default is the fp32 epsilon for bf16 and fp32 inputs (its compute type).
 * Odd D: no rotation (as the reference). D <= 512.
 * The backward takes the forward's inputs and the output gradients and writes dq, dk. */
LTVQKV_API int ltvqkv_rotary_qk_norm_fwd(int dtype, const void* q, const int64_t* q_strides,
                    const void* k, const int64_t* k_strides, const void* cos, const void* sin,
                    const int64_t* cs_strides, void* out_q, const int64_t* oq_strides,
                    void* out_k, const int64_t* ok_strides,
                    int B, int T, int NH, int NKVH, int D, float eps, void* stream);
LTVQKV_API int ltvqkv_rotary_qk_norm_bwd(int dtype, const void* q, const int64_t* q_strides,
                    const void* k, const int64_t* k_strides, const void* cos, const void* sin,
                    const int64_t* cs_strides, const void* grad_q, const int64_t* gq_strides,
                    const void* grad_k, const int64_t* gk_strides, void* dq, const int64_t* dq_strides,
                    void* dk, const int64_t* dk_strides,
                    int B, int T, int NH, int NKVH, int D, float eps, void* stream);

/* ------------------------------------------------------------------------------------------
 * Projection ("fused linear transpose"): replaces cpp_ewma_cuda.fused_linear_transpose
 * (reference cpp_ewma/src/fused_linear_transpose_forward.cu:23-58; called from
 * nanochat/ops/fused_linear_transpose.py:20-41).
 *   out[b, f, t] = sum_k weight[f, k] * x[b, t, k]
 * x [B, T, K], weight [F, K], out [B, F, T], all contiguous and of `dtype`; fp32 accumulation.
 * bf16 with K % 8 == 0 and T % 8 == 0 runs on tcgen05 tensor cores (TMA-fed, TMEM
 * accumulators); other shapes and fp32 run a CUDA-core kernel with fp32 products.
 * ------------------------------------------------------------------------------------------ */
LTVQKV_API size_t ltvqkv_gemm_workspace_bytes(void);

LTVQKV_API int ltvqkv_gemm_fwd(int dtype, const void* x, const void* weight, void* out,
                    int B, int T, int K, int F,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Projection and scan forward in one call: ltvqkv_gemm_fwd(x, weight -> combined) followed by
 * ltvqkv_scan_fwd(combined viewed [B, T, F] -> q, k, v), as the reference's filter forward calls
 * them (nanochat/ltv_cuda_fused_concat_head_major_register_cast_blelloch_scan_qkv_filter.py:24-73:
 * fused_linear_transpose, then the scan op); no single reference function corresponds. x [B, T, C],
 * weight [F, C], combined [B, F, T] (written, as ltvqkv_gemm_fwd writes it), inits [B, H, D],
 * logit_bias [H, Da] fp32, q/k/v [B, heads, T, D], all contiguous. bf16 with D = 128, Da = 1,
 * T % 32 == 0, C % 8 == 0 and B * H >= 2 * (SM count) runs fused (the head's value rows go from the tensor cores' TMEM
 * accumulator straight into the scan; the decay-logit rows are projected first); other cases run
 * the two entry points in sequence. Results equal the two-call sequence bit for bit. The workspace
 * is the scan's (ltvqkv_scan_workspace_bytes). */
LTVQKV_API int ltvqkv_proj_scan_fwd(int dtype, const void* x, const void* weight, const void* inits,
                    const float* logit_bias, void* combined, void* out_q, void* out_k, void* out_v,
                    int B, int T, int C, int NH, int NKVH, int Da, int r, int use_sigmoid,
                    void* workspace, size_t workspace_bytes, void* stream);

/* As ltvqkv_proj_scan_fwd, and also writes the scan's fp32 state entering every 32-token chunk
 * but the first: ckpt [B, H, T / 32, D] fp32 (16-byte aligned; entry [b, h, j] is the state after
 * token 32 * j + 31, the last one is not written), for ltvqkv_scan_bwd_ckpt. inits_bs: element
 * distance between the sequences' initial states, H * D, or 0 for one state [H, D] shared by every
 * sequence. Only the fused kernel writes checkpoints: where ltvqkv_proj_scan_fwd would run the two
 * entry points in sequence, this returns LTVQKV_ERR_UNSUPPORTED before anything is launched (call
 * ltvqkv_proj_scan_fwd instead). */
LTVQKV_API int ltvqkv_proj_scan_fwd_ckpt(int dtype, const void* x, const void* weight, const void* inits,
                    int64_t inits_bs, const float* logit_bias, void* combined, void* out_q, void* out_k,
                    void* out_v, float* ckpt,
                    int B, int T, int C, int NH, int NKVH, int Da, int r, int use_sigmoid,
                    void* workspace, size_t workspace_bytes, void* stream);

/* As ltvqkv_proj_scan_fwd_ckpt, with the attention's prologue on q and k folded into the scan's
 * epilogue (reference nanochat/gpt.py:96-111, 224-230: apply_rotary_emb then F.rms_norm over the
 * head dim; no reference C function corresponds): out_q / out_k receive the rotated, RMS-normalised
 * rows instead of the raw filter outputs (v unchanged), equal bit for bit to ltvqkv_proj_scan_fwd_ckpt
 * followed by ltvqkv_rotary_qk_norm_fwd. rope_cos / rope_sin: bf16 tables of D / 2 values per token
 * (rows rope_stride elements apart, 4-byte aligned, even stride; the model's cos / sin buffers for
 * the sequence's positions); eps: the norm's epsilon (F.rms_norm's default: FLT_EPSILON). The raw
 * outputs are not stored: ltvqkv_rotary_qk_norm_bwd_ckpt replays them. */
LTVQKV_API int ltvqkv_proj_scan_fwd_ckpt_rope(int dtype, const void* x, const void* weight, const void* inits,
                    int64_t inits_bs, const float* logit_bias, void* combined, void* out_q, void* out_k,
                    void* out_v, float* ckpt, const void* rope_cos, const void* rope_sin,
                    int64_t rope_stride, float eps,
                    int B, int T, int C, int NH, int NKVH, int Da, int r, int use_sigmoid,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Backward of that prologue: dq / dk (the gradients of the raw filter outputs, bf16 [B, heads, T, D]
 * with any pair-aligned strides) from grad_q / grad_k (those of the rotated, normalised rows), with
 * the raw outputs replayed from ckpt — ltvqkv_proj_scan_fwd_ckpt_rope does not store them. Equal bit
 * for bit to ltvqkv_rotary_qk_norm_bwd on the raw outputs ltvqkv_proj_scan_fwd_ckpt would have
 * stored; dq / dk then feed ltvqkv_scan_bwd_ckpt as grad_hq / grad_hk. combined, inits (inits_bs as
 * for the forward), logit_bias and ckpt are the forward's; bf16, D = 128, Da = 1, T % 32 == 0. */
LTVQKV_API int ltvqkv_rotary_qk_norm_bwd_ckpt(int dtype, const void* combined, const void* inits,
                    int64_t inits_bs, const float* logit_bias, const float* ckpt,
                    const void* rope_cos, const void* rope_sin, int64_t rope_stride, float eps,
                    const void* grad_q, const int64_t* gq_strides, const void* grad_k, const int64_t* gk_strides,
                    void* dq, const int64_t* dq_strides, void* dk, const int64_t* dk_strides,
                    int B, int T, int NH, int NKVH, int Da, int r, int use_sigmoid, void* stream);

/* Projection backward: replaces cpp_ewma_cuda.fused_linear_transpose_backward
 * (reference cpp_ewma/src/fused_linear_transpose_backward.cu:22-132; called from
 * nanochat/ops/fused_linear_transpose.py:84-101).
 *   grad_x[b, t, k]   = sum_f grad_out[b, f, t] * weight[f, k]      (overwritten)
 *   grad_weight[f, k] = sum_b sum_t grad_out[b, f, t] * x[b, t, k]  (overwritten)
 * grad_out [B, F, T] with strides (go_b, go_f, go_t): contiguous (F*T, T, 1) or the
 * transposed view (F*T, 1, F). x, weight, grad_x use `dtype`; grad_weight uses
 * grad_weight_dtype (fp32 master weights under autocast). One launch computes both.
 * An fp32 grad_weight over an even number of batches is reduced as two batch halves whose
 * partial sums the kernel combines in place (no zero fill, no floating-point atomics;
 * deterministic) through counters kept in the workspace after its header: use a workspace of
 * ltvqkv_gemm_workspace_bytes() that no scan entry point shares (their look-back flags stay
 * set between calls), zero-filled once.
 */
LTVQKV_API int ltvqkv_gemm_bwd(int dtype, const void* x, const void* weight,
                    const void* grad_out, int64_t go_b, int64_t go_f, int64_t go_t,
                    void* grad_x, void* grad_weight, int grad_weight_dtype,
                    int B, int T, int K, int F,
                    void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------
 * Decode: one incremental filter step per token, replacing the T == 1 pass of
 * LtvCudaFusedConcatHeadMajorRegisterCastBlellochScanQkvFilter.forward with cached state
 * (reference nanochat/ltv_cuda_fused_concat_head_major_register_cast_blelloch_scan_qkv_filter.py:24-73
 * with previous_values from nanochat/kv_cache.py:212-257): projection of x[b, :],
 * rounding of the projected values to `dtype` (as the reference's [B,F,1] buffer does), gate,
 * and one recurrence step, in one launch.
 *   x:       [B, C] contiguous.    weight: [F, C] contiguous.
 *   prev_q/k/v: [B, NH|NKVH, D] with element strides (b, h, d) each given as 3 int64; NULL
 *            prev_q means "no cached state": init_param [H, D] (contiguous) is used for every b.
 *   out_q/k/v: [B, NH|NKVH, D] with element strides (3 int64 each); may alias prev_* exactly
 *            (in-place state update) but must not partially overlap them.
 * ------------------------------------------------------------------------------------------ */
LTVQKV_API int ltvqkv_decode_step(int dtype, const void* x, const void* weight, const float* logit_bias,
                       const void* prev_q, const int64_t* pq_strides,
                       const void* prev_k, const int64_t* pk_strides,
                       const void* prev_v, const int64_t* pv_strides,
                       const void* init_param,
                       void* out_q, const int64_t* oq_strides,
                       void* out_k, const int64_t* ok_strides,
                       void* out_v, const int64_t* ov_strides,
                       int B, int C, int NH, int NKVH, int Da, int r, int use_sigmoid,
                       void* stream);

/* Reads and clears the device-side error word of a workspace (synchronises `stream`).
 * *err_out receives LTVQKV_OK or LTVQKV_ERR_TIMEOUT. */
LTVQKV_API int ltvqkv_workspace_error(void* workspace, void* stream, uint32_t* err_out);

/* Failure-path check (no reference counterpart): launches one thread that waits on a
 * workspace word nothing sets, gives up after limit_ns (at most 5 s), records
 * LTVQKV_ERR_TIMEOUT in the workspace and returns; read it with ltvqkv_workspace_error.
 * This is the bounded-wait path of every inter-CTA wait in the library. With workspace NULL the
 * wait records into ltvqkv_scan_fwd_noalloc's array on the current device instead (read it with
 * ltvqkv_scan_noalloc_error). */
LTVQKV_API int ltvqkv_debug_wait_timeout(void* workspace, uint64_t limit_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LTVQKV_H_ */
