// Look-back (chunk-restarting) scan, forward and backward.
//
// The reference's look-back scans (nanochat/ops/ltv_cuda_look_back_fused_concat_head_major_register_cast_
// {blelloch,sequential}_scan.py; semantics in nanochat/ops/ltv_reference_ops.py:37-124) split the
// T tokens into chunks — [0, P), then [P + (i-1) Q, P + i Q) — and compute every chunk's outputs
// with the same recurrence h_t = (1 - a_t) h_{t-1} + a_t u_t, restarted from the initial state
// K - 1 tokens before the chunk (a warm-up prefix whose states are not output). P >= T is the
// plain scan; K = 1 restarts exactly at each chunk.
//
// B200 layout: one CTA per (batch, head) row, thread c = channel c, tokens walked in order with
// the state in a register; the decay of channel c's group is evaluated by the thread itself. The
// backward walks the chunks in reverse, and inside a chunk first the chunk's own tokens (h_{t-1}
// read from the saved outputs, which are that chunk's states rounded to the storage dtype) and
// then the warm-up prefix, whose states are replayed in 32-token blocks from checkpoints kept in
// shared memory. Contributions of overlapping prefixes to one element of grad_combined are added
// in the reference autograd graph's order — later chunks first, each rounded to the storage dtype
// and summed in it — and in fp32 the per-token group sums of dalpha are sequential in the channel
// index, so fp32 results follow the reference oracle's operation order (separately rounded
// multiplies and adds, no FMA contraction); bf16 sums each warp's 32 channels by a shuffle tree.
// Every grad_combined element is written by exactly one thread. The bf16 forward of the
// production layout (T contiguous per channel row) reads 16-byte pieces of its row instead of one
// element per token (lookback_fwd_rows_kernel, same arithmetic).
#include "ltvqkv_common.cuh"

namespace ltvqkv {
namespace {

constexpr int kLbBlock = 32;  // prefix replay block (tokens)

struct LbArgs {
  const void* combined;
  long long sc_b, sc_t, sc_e;
  const void* inits;
  const float* logit_bias;
  void* out[3];
  const void* h[3];
  long long hs[3][4];
  const void* gh[3];
  long long gs[3][4];
  void* grad_combined;
  long long gc_b, gc_t, gc_e;
  void* grad_inits;
  float* bias_part;  // [B][H][Da]
  int B, T, NH, NKVH, Da, r, D, H, use_sigmoid;
  long long P, Q, K;
  int nchunks, ncp;  // chunks per row; prefix checkpoints
};

template <typename S>
LTVQKV_DEVICE float ld(const void* p, long long i) {
  if constexpr (sizeof(S) == 4) return reinterpret_cast<const float*>(p)[i];
  else return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}
template <typename S>
LTVQKV_DEVICE void st(void* p, long long i, float v) {
  if constexpr (sizeof(S) == 4) reinterpret_cast<float*>(p)[i] = v;
  else reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}
// Rounding to the storage dtype (identity for fp32).
template <typename S>
LTVQKV_DEVICE float qz(float v) {
  if constexpr (sizeof(S) == 4) return v;
  else return __bfloat162float(__float2bfloat16_rn(v));
}

LTVQKV_DEVICE void chunk_bounds(const LbArgs& a, int ci, int& t_start, int& t_end, int& t_pref) {
  long long s = ci == 0 ? 0 : a.P + (long long)(ci - 1) * a.Q;
  long long e = ci == 0 ? a.P : a.P + (long long)ci * a.Q;
  if (e > a.T) e = a.T;
  long long p = s - (a.K - 1);
  t_start = (int)s;
  t_end = (int)e;
  t_pref = p < 0 ? 0 : (int)p;
}

template <typename S>
LTVQKV_DEVICE float lb_alpha(const LbArgs& a, long long cb, int t, int col, int h, int g) {
  const float raw = __fadd_rn(ld<S>(a.combined, cb + (long long)t * a.sc_t + (long long)(col + a.D + g) * a.sc_e),
                              a.logit_bias[h * a.Da + g]);
  if (!a.use_sigmoid) return raw;
  if constexpr (sizeof(S) == 4) return sigmoid_f32_exact(raw);
  else return sigmoid_f32(raw);
}

// lb_alpha in two steps, so that the load can be issued tokens ahead of the arithmetic
template <typename S>
LTVQKV_DEVICE float lb_logit_ld(const LbArgs& a, long long cb, int t, int col, int g) {
  return ld<S>(a.combined, cb + (long long)t * a.sc_t + (long long)(col + a.D + g) * a.sc_e);
}
template <typename S>
LTVQKV_DEVICE float lb_gate(const LbArgs& a, float logit, int h, int g) {
  const float raw = __fadd_rn(logit, a.logit_bias[h * a.Da + g]);
  if (!a.use_sigmoid) return raw;
  if constexpr (sizeof(S) == 4) return sigmoid_f32_exact(raw);
  else return sigmoid_f32(raw);
}

// s' = (1 - a) s + a u, each product and the sum rounded once
LTVQKV_DEVICE float lb_step(float s, float al, float u) {
  return __fadd_rn(__fmul_rn(__fsub_rn(1.0f, al), s), __fmul_rn(al, u));
}

template <typename S>
__global__ void __launch_bounds__(1024) lookback_fwd_kernel(LbArgs a) {
  const int b = blockIdx.x / a.H, h = blockIdx.x % a.H;
  const int c = threadIdx.x;
  if (c >= a.D) return;
  int which, hloc, nheads;
  split_head(h, a.NH, a.NKVH, which, hloc, nheads);
  const long long cb = (long long)b * a.sc_b;
  const int col = h * (a.D + a.Da);
  const int g = c / a.r;
  const float init = ld<S>(a.inits, ((long long)b * a.H + h) * a.D + c);
  const long long ob = ((long long)b * nheads + hloc) * (long long)a.T * a.D + c;
  for (int ci = 0; ci < a.nchunks; ++ci) {
    int t_start, t_end, t_pref;
    chunk_bounds(a, ci, t_start, t_end, t_pref);
    float s = init;
    for (int t = t_pref; t < t_end; ++t) {
      const float al = lb_alpha<S>(a, cb, t, col, h, g);
      s = lb_step(s, al, ld<S>(a.combined, cb + (long long)t * a.sc_t + (long long)(col + c) * a.sc_e));
      if (t >= t_start) st<S>(a.out[which], ob + (long long)t * a.D, s);
    }
  }
}

// Forward for the production layout — the projection buffer's transposed view (T contiguous per
// channel row, element strides sc_t = 1, sc_e = T), bf16: one CTA per (row, chunk) — every chunk
// restarts from the initial state, so the chunks are independent — thread c reads its channel row
// 32 tokens at a time as four 16-byte loads, the next 32 tokens' loads in flight while the current
// ones are walked, and the decays come from a table of the chunk's gates per decay group built once
// in shared memory (one sigmoid per (group, token) instead of one per thread). Same arithmetic as
// lookback_fwd_kernel token for token, so the outputs are identical.
constexpr int kLbGroup = 32;

LTVQKV_DEVICE void lb_load_group(const __nv_bfloat16* urow, int tb, int T, uint4 (&u)[4]) {
#pragma unroll
  for (int k = 0; k < 4; ++k)
    u[k] = tb + 8 * k < T ? __ldg(reinterpret_cast<const uint4*>(urow + tb + 8 * k)) : make_uint4(0, 0, 0, 0);
}

// Gate-table length of one chunk (its warm-up prefix and own tokens; the longest chunk is
// max(P, Q) tokens).
__host__ __device__ inline int lb_chunk_gate_len(int T, long long P, long long Q, long long K) {
  const long long n = (P > Q ? P : Q) + K - 1;
  return (int)(n < T ? n : T);
}

__global__ void __launch_bounds__(1024) lookback_fwd_rows_kernel(LbArgs a) {
  extern __shared__ float lb_gate[];  // [Da][gstride]: gates of tokens t_pref ..
  const int row = blockIdx.x / a.nchunks, ci = blockIdx.x % a.nchunks;
  const int b = row / a.H, h = row % a.H;
  const int c = threadIdx.x;
  const long long cb = (long long)b * a.sc_b;
  const int col = h * (a.D + a.Da);
  const int gstride = lb_chunk_gate_len(a.T, a.P, a.Q, a.K);
  int t_start, t_end, t_pref;
  chunk_bounds(a, ci, t_start, t_end, t_pref);
  const int ntok = t_end - t_pref;
  for (int i = threadIdx.x; i < a.Da * ntok; i += blockDim.x) {
    const int g = i / ntok, j = i - g * ntok;
    lb_gate[g * gstride + j] = lb_alpha<__nv_bfloat16>(a, cb, t_pref + j, col, h, g);
  }
  __syncthreads();
  if (c >= a.D) return;
  int which, hloc, nheads;
  split_head(h, a.NH, a.NKVH, which, hloc, nheads);
  const float* gr = lb_gate + (c / a.r) * gstride - t_pref;  // indexed by token
  const float init = ld<__nv_bfloat16>(a.inits, ((long long)b * a.H + h) * a.D + c);
  const __nv_bfloat16* urow = reinterpret_cast<const __nv_bfloat16*>(a.combined) + cb + (long long)(col + c) * a.T;
  __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(a.out[which]) + ((long long)b * nheads + hloc) * a.T * a.D + c;
  float s = init;
  int tb = t_pref & ~7;
  uint4 cur[4], nxt[4];
  lb_load_group(urow, tb, a.T, cur);
  for (; tb < t_end; tb += kLbGroup) {
    if (tb + kLbGroup < t_end) lb_load_group(urow, tb + kLbGroup, a.T, nxt);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t wv[4] = {cur[k].x, cur[k].y, cur[k].z, cur[k].w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int t = tb + 8 * k + e;
        if (t >= t_pref && t < t_end) {
          s = lb_step(s, gr[t], (e & 1) ? bf16_hi(wv[e / 2]) : bf16_lo(wv[e / 2]));
          if (t >= t_start) orow[(long long)t * a.D] = __float2bfloat16_rn(s);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) cur[k] = nxt[k];
  }
}

// One token of the reverse sweep: du and dlogit contributions of this chunk (rounded to the
// storage dtype and added to what later chunks left, or stored when no later chunk reached the
// token), the group sums of dalpha, and the adjoint carry. All threads of the CTA call it.
template <typename S>
LTVQKV_DEVICE void lb_bwd_token(const LbArgs& a, float* red, long long cb, long long gcb, int col, int h, int g,
                                bool active, int c, int t, float sprev, bool first, float& gacc, float& bias_acc) {
  float al = 0.f;
  if (active) {
    al = lb_alpha<S>(a, cb, t, col, h, g);
    const float u = ld<S>(a.combined, cb + (long long)t * a.sc_t + (long long)(col + c) * a.sc_e);
    const long long gi = gcb + (long long)t * a.gc_t + (long long)(col + c) * a.gc_e;
    const float du = qz<S>(__fmul_rn(gacc, al));
    st<S>(a.grad_combined, gi, first ? du : __fadd_rn(ld<S>(a.grad_combined, gi), du));
    red[c] = __fmul_rn(gacc, __fsub_rn(u, sprev));
  }
  // bf16 with groups of whole warps: each warp's 32 terms summed by a shuffle tree, the warps of a
  // group in order (fp32 keeps the oracle's sequential channel order)
  constexpr bool kTree = sizeof(S) == 2;
  const bool tree = kTree && a.r % 32 == 0;
  if (tree) {
    float v = active ? red[c] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();  // every red[c] has been read
    if ((c & 31) == 0) red[c / 32] = v;
  }
  __syncthreads();
  if (c < a.Da) {
    float ga = 0.f;
    if (tree) {
      for (int k = 0; k < a.r / 32; ++k) ga = __fadd_rn(ga, red[c * (a.r / 32) + k]);
    } else {
      for (int k = 0; k < a.r; ++k) ga = __fadd_rn(ga, red[c * a.r + k]);
    }
    const float ag = lb_alpha<S>(a, cb, t, col, h, c);
    const float graw = a.use_sigmoid ? __fmul_rn(__fmul_rn(ga, __fsub_rn(1.0f, ag)), ag) : ga;
    const long long gi = gcb + (long long)t * a.gc_t + (long long)(col + a.D + c) * a.gc_e;
    const float dl = qz<S>(graw);
    st<S>(a.grad_combined, gi, first ? dl : __fadd_rn(ld<S>(a.grad_combined, gi), dl));
    bias_acc = __fadd_rn(bias_acc, graw);
  }
  __syncthreads();
  if (active) gacc = __fmul_rn(gacc, __fsub_rn(1.0f, al));
}

template <typename S>
__global__ void __launch_bounds__(1024) lookback_bwd_kernel(LbArgs a) {
  extern __shared__ float sm[];
  const int nth = blockDim.x;
  float* red = sm;                       // [nth]
  float* cp = red + nth;                 // [ncp][D]: state before each kLbBlock-th prefix token
  float* blk = cp + (long long)a.ncp * a.D;  // [kLbBlock][D]: replayed states of one prefix block
  const int b = blockIdx.x / a.H, h = blockIdx.x % a.H;
  const int c = threadIdx.x;
  const bool active = c < a.D;
  const int cc = active ? c : 0;
  int which, hloc, nheads;
  split_head(h, a.NH, a.NKVH, which, hloc, nheads);
  const long long cb = (long long)b * a.sc_b, gcb = (long long)b * a.gc_b;
  const int col = h * (a.D + a.Da);
  const int g = cc / a.r;
  const long long* hs = a.hs[which];
  const long long* gs = a.gs[which];
  const long long hb = (long long)b * hs[0] + (long long)hloc * hs[1] + (long long)cc * hs[3];
  const long long gb = (long long)b * gs[0] + (long long)hloc * gs[1] + (long long)cc * gs[3];
  const float init = active ? ld<S>(a.inits, ((long long)b * a.H + h) * a.D + cc) : 0.f;
  float ginit = 0.f;
  float bias_acc = 0.f;  // threads c < Da: their group's bias gradient
  int next_pref = a.T;   // t_pref of the next (later) chunk: tokens at or beyond it were reached already
  for (int ci = a.nchunks - 1; ci >= 0; --ci) {
    int t_start, t_end, t_pref;
    chunk_bounds(a, ci, t_start, t_end, t_pref);
    const int npre = t_start - t_pref;
    // warm-up prefix replay with checkpoints (states before tokens t_pref + kLbBlock * j)
    float s = init;
    for (int i = 0; i < npre; ++i) {
      if (active && i % kLbBlock == 0) cp[(long long)(i / kLbBlock) * a.D + c] = s;
      if (active) s = lb_step(s, lb_alpha<S>(a, cb, t_pref + i, col, h, g),
                              ld<S>(a.combined, cb + (long long)(t_pref + i) * a.sc_t + (long long)(col + c) * a.sc_e));
    }
    const float s_pre = qz<S>(s);  // the chunk's h_{t_start - 1}, rounded like a stored output
    float gacc = 0.f;
    // the chunk's own tokens: h_{t-1} is the saved output
    for (int t = t_end - 1; t >= t_start; --t) {
      float sprev = 0.f;
      if (active) {
        gacc = __fadd_rn(gacc, ld<S>(a.gh[which], gb + (long long)t * gs[2]));
        sprev = t > t_start ? ld<S>(a.h[which], hb + (long long)(t - 1) * hs[2]) : s_pre;
      }
      lb_bwd_token<S>(a, red, cb, gcb, col, h, g, active, c, t, sprev, t < next_pref, gacc, bias_acc);
    }
    // the prefix, one replayed block at a time from the last
    for (int j = (npre - 1) / kLbBlock; npre > 0 && j >= 0; --j) {
      const int i0 = j * kLbBlock, n = min(kLbBlock, npre - i0);
      if (active) {
        float q = cp[(long long)j * a.D + c];
        for (int i = 0; i < n; ++i) {
          blk[(long long)i * a.D + c] = q;
          q = lb_step(q, lb_alpha<S>(a, cb, t_pref + i0 + i, col, h, g),
                      ld<S>(a.combined, cb + (long long)(t_pref + i0 + i) * a.sc_t + (long long)(col + c) * a.sc_e));
        }
      }
      for (int i = n - 1; i >= 0; --i) {
        const int t = t_pref + i0 + i;
        const float sprev = active ? qz<S>(blk[(long long)i * a.D + c]) : 0.f;
        lb_bwd_token<S>(a, red, cb, gcb, col, h, g, active, c, t, sprev, t < next_pref, gacc, bias_acc);
      }
    }
    ginit = __fadd_rn(ginit, gacc);
    next_pref = t_pref;
  }
  if (active) st<S>(a.grad_inits, ((long long)b * a.H + h) * a.D + c, ginit);
  if (c < a.Da) a.bias_part[((long long)b * a.H + h) * a.Da + c] = bias_acc;
}

// ------------------------------------------------------------------------------------------
// Chunk-parallel backward (bf16, warm-up prefix no longer than any chunk: K - 1 <= min(P, Q)).
// Every chunk restarts from the initial state, so the chunks' backward passes are independent:
// one CTA per (row, chunk) runs lookback_bwd_kernel's per-chunk body (prefix states replayed into
// shared memory, own tokens with h_{t-1} from the saved outputs, then the prefix), reading the value
// rows in aligned 8-token pieces (16 bytes) and writing grad_combined the same way where a piece is
// the chunk's alone. Tokens reached by two chunks — a chunk's last K - 1 own
// tokens are the next chunk's warm-up prefix — have both contributions, each rounded to bf16, kept
// in workspace slots; lookback_bwd_fixup_kernel then adds them in the sequential kernel's order
// (later chunk first) and sums the chunks' initial-state gradients in descending chunk order, as
// the sequential kernel does. The per-row logit-bias sum adds per-chunk partials (a different
// association than the sequential walk; bf16 only).
struct LbParWs {  // workspace slots of the chunk-parallel backward
  __nv_bfloat16* own;  // [rows][nchunks][K - 1][lb_slot_row]: a chunk's contributions to its last K - 1 tokens
  __nv_bfloat16* pre;  // [rows][nchunks][K - 1][lb_slot_row]: a chunk's contributions to its warm-up prefix
  float* gi;           // [rows][nchunks][D]: each chunk's initial-state gradient
  float* bp;           // [rows][nchunks][Da]: each chunk's logit-bias partial
};

// A slot's token row: D + Da entries padded to a multiple of 8 (16-byte rows).
__host__ __device__ inline int lb_slot_row(int D, int Da) { return (D + Da + 7) & ~7; }

__host__ __device__ inline size_t lb_par_ws_bytes(int B, int H, int D, int Da, int nchunks, long long K) {
  const size_t rows = (size_t)B * H, slots = rows * (size_t)nchunks;
  const size_t kk = (size_t)(K > 1 ? K - 1 : 0);
  const size_t bf = slots * kk * (size_t)lb_slot_row(D, Da) * 2;
  return 2 * ((bf + 255) / 256 * 256) + slots * (size_t)D * 4 + ((slots * (size_t)Da * 4 + 255) / 256 * 256);
}

// Eight tokens (8-aligned group starting at t0) of a channel / logit row in the production layout.
LTVQKV_DEVICE uint4 lb_row8(const LbArgs& a, long long cb, int rowidx, int t0) {
  return __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.combined) + cb +
                                               (long long)rowidx * a.sc_e + t0));
}
LTVQKV_DEVICE float lb_pick(const uint4& w8, int e) {
  const uint32_t wv = e < 2 ? w8.x : (e < 4 ? w8.y : (e < 6 ? w8.z : w8.w));
  return (e & 1) ? bf16_hi(wv) : bf16_lo(wv);
}

// Sums eight values over the warp's 32 lanes, each by the tree of a 16-8-4-2-1 xor butterfly (the
// same pairs of partial sums, so the same result bit for bit), in 9 shuffles instead of 40: every
// level keeps half of the lane's values and sends the other half. Lane l ends with the sum of
// value (l >> 2) & 7.
LTVQKV_DEVICE float lb_warp_sum8(const float (&v)[8], int lane) {
  const bool h4 = lane & 16, h3 = lane & 8, h2 = lane & 4;
  float r1[4], r2[2];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float keep = h4 ? v[k + 4] : v[k], send = h4 ? v[k] : v[k + 4];
    r1[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const float keep = h3 ? r1[j + 2] : r1[j], send = h3 ? r1[j] : r1[j + 2];
    r2[j] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  float r3 = (h2 ? r2[1] : r2[0]) + __shfl_xor_sync(0xffffffffu, h2 ? r2[0] : r2[1], 4);
  r3 += __shfl_xor_sync(0xffffffffu, r3, 2);
  r3 += __shfl_xor_sync(0xffffffffu, r3, 1);
  return r3;
}

constexpr int kLbStages = 3;  // 8-token groups of copies in flight (the current one and two ahead)
__host__ __device__ inline size_t lb_par_stage_bytes(int D) { return (size_t)48 * D; }

// One CTA per (row, chunk), thread = channel. Shared memory: three stages of 8-token group tiles
// (upstream-gradient rows, saved-output rows one token back, the value rows' 16-byte pieces) copied
// by cp.async two groups ahead of their use, the chunk's gates (every token's gate computed once,
// not by each thread), the warm-up prefix's states, and per group the warps' dalpha sums and the
// group's logit gradients. The group's eight tokens walk the adjoint carry; their dalpha terms are
// summed over each warp by one reduce-scatter tree and over the gate group's warps after one
// barrier per group, by 8 * Da threads (token, gate group) at once.
template <int kD>  // head dim when known at compile time (0: a.D)
__global__ void __launch_bounds__(256, 4) lookback_bwd_par_kernel(LbArgs a, LbParWs w) {
  const int D = kD ? kD : a.D;
  extern __shared__ __align__(16) float sm[];
  const int nwarps = blockDim.x / 32;
  const int gstride = lb_chunk_gate_len(a.T, a.P, a.Q, a.K);
  const size_t stage_bytes = lb_par_stage_bytes(D);
  char* stages = reinterpret_cast<char*>(sm);
  float* wsum = reinterpret_cast<float*>(stages + kLbStages * stage_bytes);  // [2][8][nwarps]: per-warp
                                                                               // dalpha sums, by group parity
  float* grs = wsum + 16 * nwarps;    // [2][Da][8]: the group's logit-bias terms, by group parity
  float* gt = grs + 16 * a.Da;        // [Da][gstride]: gates of tokens t_pref ..
  float* pst = gt + a.Da * gstride;   // [K - 1][D]: the warm-up prefix's states (before each token)
  const int row = blockIdx.x / a.nchunks, ci = blockIdx.x % a.nchunks;
  const int b = row / a.H, h = row % a.H;
  const int c = threadIdx.x, warp = c / 32, lane = c % 32;
  const bool active = c < D;
  const int cc = active ? c : 0;
  using S = __nv_bfloat16;
  int which, hloc, nheads;
  split_head(h, a.NH, a.NKVH, which, hloc, nheads);
  const long long cb = (long long)b * a.sc_b, gcb = (long long)b * a.gc_b;
  const int col = h * (D + a.Da);
  const int g = cc / a.r, rw = a.r / 32;
  const long long* hs = a.hs[which];
  const long long* gs = a.gs[which];
  // channel 0 of this row's saved outputs and upstream gradients (channels contiguous)
  const S* h0 = reinterpret_cast<const S*>(a.h[which]) + (long long)b * hs[0] + (long long)hloc * hs[1];
  const S* gh0 = reinterpret_cast<const S*>(a.gh[which]) + (long long)b * gs[0] + (long long)hloc * gs[1];
  const float init = active ? ld<S>(a.inits, ((long long)b * a.H + h) * D + cc) : 0.f;
  const int kk = (int)(a.K - 1), DW = lb_slot_row(D, a.Da);  // slot row
  const long long slot = (long long)row * a.nchunks + ci;
  __nv_bfloat16* gc = reinterpret_cast<__nv_bfloat16*>(a.grad_combined);
  int t_start, t_end, t_pref;
  chunk_bounds(a, ci, t_start, t_end, t_pref);
  // first token reached by the next chunk's warm-up prefix (T: none)
  int np = a.T;
  if (ci + 1 < a.nchunks) {
    int s2, e2, p2;
    chunk_bounds(a, ci + 1, s2, e2, p2);
    np = p2;
  }
  // Group n (tokens ga_n = ga_0 - 8 n .. + 7) goes to stage n % 3: its upstream-gradient rows
  // ga_n .. ga_n + 7 and saved-output rows ga_n - 1 .. ga_n + 6 as [8][D] tiles (one 16-byte piece
  // each per thread: D / 8 pieces per row), and this thread's value piece (tokens ga_n .. + 7).
  // Every commit is one group (empty past the last), so waiting for all but the newest one leaves
  // the next group landed.
  const int ga0 = (t_end - 1) & ~7;
  const int ngroups = (ga0 - (t_pref & ~7)) / 8 + 1;
  const int pe = cc / (D / 8), p8 = (cc - pe * (D / 8)) * 8;  // this thread's tile piece: row, channel
  auto issue = [&](int n) {
    if (active && n < ngroups) {
      const int ga = ga0 - 8 * n;
      char* base = stages + (size_t)(n % kLbStages) * stage_bytes;
      S* ghs = reinterpret_cast<S*>(base);
      S* hts = ghs + 8 * D;
      const int e = pe, t = ga + e;
      cp_async16(ghs + e * D + p8, gh0 + (long long)t * gs[2] + p8);
      if (t >= 1) cp_async16(hts + e * D + p8, h0 + (long long)(t - 1) * hs[2] + p8);
      cp_async16(reinterpret_cast<uint4*>(hts + 8 * D) + c,
                 reinterpret_cast<const S*>(a.combined) + cb + (long long)(col + c) * a.sc_e + ga);
    }
    cp_async_commit();
  };
  issue(0);
  issue(1);
  // the chunk's gates, tokens t_pref .. t_end - 1 (same arithmetic as the sequential kernels)
  const int ntok = t_end - t_pref;
  for (int i = c; i < a.Da * ntok; i += blockDim.x) {
    const int gg = i / ntok, j = i - gg * ntok;
    gt[gg * gstride + j] = lb_gate<S>(a, lb_logit_ld<S>(a, cb, t_pref + j, col, gg), h, gg);
  }
  __syncthreads();
  const float* gtc = gt + g * gstride - t_pref;  // this thread's gate row, indexed by token
  // warm-up prefix states, one aligned 8-token group of value reads at a time
  float s = init;
  for (int ga = t_pref & ~7; ga < t_start; ga += 8) {
    const uint4 u8 = active ? lb_row8(a, cb, col + c, ga) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int t = ga + e;
      if (active && t >= t_pref && t < t_start) {
        pst[(long long)(t - t_pref) * D + c] = s;
        s = lb_step(s, gtc[t], lb_pick(u8, e));
      }
    }
  }
  const float s_pre = qz<S>(s);
  float gacc = 0.f, bias_acc = 0.f;
  int buf = 0, plo = 0, phi = 0, pga = 0;  // the previous group's tokens (bias terms not yet added)
  cp_async_wait<1>();
  __syncthreads();
  // Aligned 8-token groups from the last: own tokens (upstream gradient added, h_{t-1} from the saved
  // outputs, the first one from the prefix replay), then the warm-up prefix (stored states). Each
  // entry goes to grad_combined, or, for a token that another chunk also reaches, to this chunk's
  // own (t >= np) or prefix (t < t_start) slot.
  for (int n = 0; n < ngroups; ++n) {
    const int ga = ga0 - 8 * n;
    issue(n + 2);
    const int lo = max(ga, t_pref), hi = min(ga + 8, t_end);
    const S* ghs = reinterpret_cast<const S*>(stages + (size_t)(n % kLbStages) * stage_bytes);
    const S* hts = ghs + 8 * D;
    const uint4 u8 = active ? reinterpret_cast<const uint4*>(hts + 8 * D)[c] : make_uint4(0, 0, 0, 0);
    float duv[8], v[8];
    if (active && ga > t_start && ga + 8 <= min(t_end, np)) {
      // interior group: eight own tokens, all entries direct, h_{t-1} all from the saved outputs
#pragma unroll
      for (int e = 7; e >= 0; --e) {
        gacc = __fadd_rn(gacc, __bfloat162float(ghs[e * D + c]));
        const float al = gtc[ga + e];
        duv[e] = __fmul_rn(gacc, al);  // rounded to bf16 once, where it is stored
        v[e] = __fmul_rn(gacc, __fsub_rn(lb_pick(u8, e), __bfloat162float(hts[e * D + c])));
        gacc = __fmul_rn(gacc, __fsub_rn(1.0f, al));
      }
    } else {
      float ghv[8], hv[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int t = ga + e;
        ghv[e] = hv[e] = 0.f;
        if (active && t >= max(lo, t_start) && t < hi) {
          ghv[e] = __bfloat162float(ghs[e * D + c]);
          hv[e] = t > t_start ? __bfloat162float(hts[e * D + c]) : s_pre;
        }
        if (active && t >= lo && t < t_start) hv[e] = qz<S>(pst[(long long)(t - t_pref) * D + c]);
      }
#pragma unroll
      for (int e = 7; e >= 0; --e) {
        const int t = ga + e;
        duv[e] = v[e] = 0.f;
        if (active && t >= lo && t < hi) {
          gacc = __fadd_rn(gacc, ghv[e]);  // zero for prefix tokens
          const float al = gtc[t];
          const float du = __fmul_rn(gacc, al);  // rounded to bf16 once, where it is stored
          if (t < t_start) w.pre[(slot * kk + (t - t_pref)) * DW + c] = __float2bfloat16_rn(du);
          else if (t >= np) w.own[(slot * kk + (t - np)) * DW + c] = __float2bfloat16_rn(du);
          else duv[e] = du;
          v[e] = __fmul_rn(gacc, __fsub_rn(lb_pick(u8, e), hv[e]));
          gacc = __fmul_rn(gacc, __fsub_rn(1.0f, al));
        }
      }
    }
    const float vs = lb_warp_sum8(v, lane);
    if ((lane & 3) == 0) wsum[(buf * 8 + (lane >> 2)) * nwarps + warp] = vs;
    cp_async_wait<1>();  // group n + 1's copies (this thread's) landed; the barrier publishes them
    __syncthreads();
    if (c < a.Da) {  // the previous group's logit-bias terms, tokens in descending order
      for (int t = phi - 1; t >= plo; --t) bias_acc = __fadd_rn(bias_acc, grs[((buf ^ 1) * a.Da + c) * 8 + t - pga]);
    }
    if (c < 8 * a.Da) {  // thread (token ga + (c & 7), gate group c >> 3)
      const int e = c & 7, gg = c >> 3, t = ga + e;
      if (t >= lo && t < hi) {
        float gsum = 0.f;
        for (int q = 0; q < rw; ++q) gsum = __fadd_rn(gsum, wsum[(buf * 8 + e) * nwarps + gg * rw + q]);
        const float ag = gt[gg * gstride + t - t_pref];
        const float graw = a.use_sigmoid ? __fmul_rn(__fmul_rn(gsum, __fsub_rn(1.0f, ag)), ag) : gsum;
        const __nv_bfloat16 dl = __float2bfloat16_rn(graw);
        if (t < t_start) w.pre[(slot * kk + (t - t_pref)) * DW + D + gg] = dl;
        else if (t >= np) w.own[(slot * kk + (t - np)) * DW + D + gg] = dl;
        else gc[gcb + (long long)(col + D + gg) * a.gc_e + t] = dl;
        grs[(buf * a.Da + gg) * 8 + e] = graw;
      }
    }
    plo = lo; phi = hi; pga = ga;
    buf ^= 1;
    // this chunk's direct value entries: tokens max(lo, t_start) .. min(hi, np) - 1
    const int dlo = max(lo, t_start), dhi = min(hi, np);
    if (active && dlo < dhi) {
      __nv_bfloat16* gr = gc + gcb + (long long)(col + c) * a.gc_e;
      if (dlo == ga && dhi == ga + 8) {
        *reinterpret_cast<uint4*>(gr + ga) = make_uint4(pack_bf16x2(duv[0], duv[1]), pack_bf16x2(duv[2], duv[3]),
                                                       pack_bf16x2(duv[4], duv[5]), pack_bf16x2(duv[6], duv[7]));
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (ga + e >= dlo && ga + e < dhi) gr[ga + e] = __float2bfloat16_rn(duv[e]);
      }
    }
  }
  __syncthreads();
  if (c < a.Da) {
    for (int t = phi - 1; t >= plo; --t) bias_acc = __fadd_rn(bias_acc, grs[((buf ^ 1) * a.Da + c) * 8 + t - pga]);
  }
  if (active) w.gi[slot * D + c] = gacc;
  if (c < a.Da) w.bp[slot * a.Da + c] = bias_acc;
}

// One CTA per (row, pair of consecutive chunks ci, ci + 1): every token reached by both (the later
// chunk's warm-up prefix) gets the later chunk's contribution plus the earlier one's, in bf16, staged
// through shared memory so that the slots are read and grad_combined written along their contiguous
// axes. The CTAs of ci = 0 also sum the row's initial-state gradient and logit-bias partials over the
// chunks in descending order.
constexpr int kLbFixTok = 16;
__global__ void __launch_bounds__(256) lookback_bwd_fixup_kernel(LbArgs a, LbParWs w) {
  using S = __nv_bfloat16;
  __shared__ float st_sum[256 * (kLbFixTok + 1)];  // [D + Da][kLbFixTok], rows padded by one
  const int row = blockIdx.x / (a.nchunks - 1), ci = blockIdx.x % (a.nchunks - 1);
  const int b = row / a.H, h = row % a.H;
  const long long gcb = (long long)b * a.gc_b;
  const int col = h * (a.D + a.Da);
  const int kk = (int)(a.K - 1), DW = a.D + a.Da, DWp = lb_slot_row(a.D, a.Da), pr = DWp / 8;
  int s1, e1, p1, s2, e2, p2;
  chunk_bounds(a, ci, s1, e1, p1);
  chunk_bounds(a, ci + 1, s2, e2, p2);
  const long long so = (long long)row * a.nchunks + ci, sp = so + 1;
  const int n = e1 - p2;  // tokens p2 .. e1 - 1
  for (int i0 = 0; i0 < n; i0 += kLbFixTok) {
    const int m = min(kLbFixTok, n - i0);
    for (int idx = threadIdx.x; idx < m * pr; idx += blockDim.x) {  // slot rows as 16-byte pieces
      const int i = idx / pr, e0 = (idx - i * pr) * 8;
      const uint4 lv = *reinterpret_cast<const uint4*>(w.pre + (sp * kk + i0 + i) * DWp + e0);
      const uint4 ev = *reinterpret_cast<const uint4*>(w.own + (so * kk + i0 + i) * DWp + e0);
      const uint32_t lw[4] = {lv.x, lv.y, lv.z, lv.w}, ew[4] = {ev.x, ev.y, ev.z, ev.w};
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (e0 + k < DW) {
          const float later = (k & 1) ? bf16_hi(lw[k / 2]) : bf16_lo(lw[k / 2]);
          const float earlier = (k & 1) ? bf16_hi(ew[k / 2]) : bf16_lo(ew[k / 2]);
          st_sum[(e0 + k) * (kLbFixTok + 1) + i] = __fadd_rn(later, earlier);
        }
      }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < DW * kLbFixTok; idx += blockDim.x) {  // grad_combined rows: tokens
      const int e = idx / kLbFixTok, i = idx % kLbFixTok;                   // contiguous
      if (i < m)
        st<S>(a.grad_combined, gcb + (long long)(p2 + i0 + i) * a.gc_t + (long long)(col + e) * a.gc_e,
              st_sum[e * (kLbFixTok + 1) + i]);
    }
    __syncthreads();
  }
  if (ci != 0) return;
  for (int c = threadIdx.x; c < a.D; c += blockDim.x) {
    float gi = 0.f;
    for (int cj = a.nchunks - 1; cj >= 0; --cj) gi = __fadd_rn(gi, w.gi[((long long)row * a.nchunks + cj) * a.D + c]);
    st<S>(a.grad_inits, (long long)row * a.D + c, gi);
  }
  for (int gg = threadIdx.x; gg < a.Da; gg += blockDim.x) {
    float bs = 0.f;
    for (int cj = a.nchunks - 1; cj >= 0; --cj)
      bs = __fadd_rn(bs, w.bp[((long long)row * a.nchunks + cj) * a.Da + gg]);
    a.bias_part[(long long)row * a.Da + gg] = bs;
  }
}

// grad_logit_bias[h, g] += sum over b (descending, the oracle's order) of per-(b, h) partials.
__global__ void lookback_bias_reduce_kernel(const float* part, float* grad_bias, int B, int H, int Da) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= H * Da) return;
  float sum = 0.f;
  for (int b = B - 1; b >= 0; --b) sum = __fadd_rn(sum, part[(long long)b * H * Da + idx]);
  grad_bias[idx] = __fadd_rn(grad_bias[idx], sum);
}

int lb_chunks(int T, long long P, long long Q) {
  if ((long long)T <= P) return 1;
  return (int)(1 + ((long long)T - P + Q - 1) / Q);
}

int lb_validate(int dtype, int B, int T, int NH, int NKVH, int Da, int r, long long P, long long Q, long long K) {
  if (!ltvqkv_host::valid_dtype(dtype)) return LTVQKV_ERR_DTYPE;
  if (B < 0 || T < 0 || NH < 0 || NKVH < 0 || Da < 1 || r < 1 || P < 1 || Q < 1 || K < 1) return LTVQKV_ERR_SHAPE;
  if ((long long)Da * r > 1024) return LTVQKV_ERR_SHAPE;  // one thread per channel
  return LTVQKV_OK;
}

int lb_threads(int D) { return (D + 31) / 32 * 32; }

size_t lb_bwd_smem(int D, int T, long long K, int& ncp) {
  const long long npre_max = std::min<long long>(K - 1, T);
  ncp = (int)((npre_max + kLbBlock - 1) / kLbBlock);
  return sizeof(float) * ((size_t)lb_threads(D) + (size_t)ncp * D + (size_t)kLbBlock * D);
}

}  // namespace
}  // namespace ltvqkv

using namespace ltvqkv;

extern "C" size_t ltvqkv_lookback_workspace_bytes(int B, int NH, int NKVH, int Da) {
  if (B < 0 || NH < 0 || NKVH < 0 || Da < 1) return 0;
  return 256 + sizeof(float) * (size_t)B * (NH + 2 * NKVH) * Da;
}

// Whether the chunk-parallel backward takes these sizes, and the workspace it needs beyond the
// sequential kernel's.
bool lb_par_ok(int dtype, int T, int D, int Da, int r, long long P, long long Q, long long K) {
  (void)r;
  const int nch = lb_chunks(T, P, Q);
  return dtype == LTVQKV_DTYPE_BF16 && D + Da <= 256 && r % 32 == 0 && nch > 1 && K - 1 <= P && K - 1 <= Q &&
         K - 1 <= 64 && T > 0 && (long long)Da * lb_chunk_gate_len(T, P, Q, K) * 4 <= 32 * 1024;
}

extern "C" size_t ltvqkv_lookback_bwd_workspace_bytes(int B, int T, int NH, int NKVH, int Da, int r, int64_t P,
                                                      int64_t Q, int64_t K) {
  const size_t base = ltvqkv_lookback_workspace_bytes(B, NH, NKVH, Da);
  if (base == 0 || T < 0 || r < 1 || P < 1 || Q < 1 || K < 1) return base;
  const int H = NH + 2 * NKVH, D = Da * r;
  if (!lb_par_ok(LTVQKV_DTYPE_BF16, T, D, Da, r, P, Q, K)) return base;
  return (base + 255) / 256 * 256 + lb_par_ws_bytes(B, H, D, Da, lb_chunks(T, P, Q), K);
}

extern "C" int ltvqkv_lookback_scan_fwd(int dtype, const void* combined, int64_t sc_b, int64_t sc_t, int64_t sc_e,
                                        const void* inits, const float* logit_bias, void* out_q, void* out_k,
                                        void* out_v, int B, int T, int NH, int NKVH, int Da, int r, int64_t P,
                                        int64_t Q, int64_t K, int use_sigmoid, void* stream) {
  int rc = lb_validate(dtype, B, T, NH, NKVH, Da, r, P, Q, K);
  if (rc != LTVQKV_OK) return rc;
  const int H = NH + 2 * NKVH;
  if ((long long)B * H * T == 0) return LTVQKV_OK;
  if (!combined || !inits || !logit_bias || (NH > 0 && !out_q) || (NKVH > 0 && (!out_k || !out_v)))
    return LTVQKV_ERR_INVALID_ARG;
  if (sc_b < 0 || sc_t < 0 || sc_e < 0) return LTVQKV_ERR_STRIDE;
  LbArgs a = {};
  a.combined = combined; a.sc_b = sc_b; a.sc_t = sc_t; a.sc_e = sc_e;
  a.inits = inits; a.logit_bias = logit_bias;
  a.out[0] = out_q; a.out[1] = out_k; a.out[2] = out_v;
  a.B = B; a.T = T; a.NH = NH; a.NKVH = NKVH; a.Da = Da; a.r = r; a.D = Da * r; a.H = H;
  a.use_sigmoid = use_sigmoid; a.P = P; a.Q = Q; a.K = K;
  a.nchunks = lb_chunks(T, P, Q);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int threads = lb_threads(a.D);
  const size_t gate_bytes = sizeof(float) * (size_t)Da * lb_chunk_gate_len(T, P, Q, K);
  const size_t ctas = (size_t)B * H * a.nchunks;
  if (dtype == LTVQKV_DTYPE_BF16 && sc_t == 1 && sc_e == T && T % 8 == 0 && sc_b % 8 == 0 &&
      (reinterpret_cast<uintptr_t>(combined) & 15) == 0 && gate_bytes <= 48 * 1024 && ctas <= 0x7fffffffULL)
    lookback_fwd_rows_kernel<<<(unsigned int)ctas, threads, gate_bytes, s>>>(a);
  else if (dtype == LTVQKV_DTYPE_F32)
    lookback_fwd_kernel<float><<<(unsigned int)(B * H), threads, 0, s>>>(a);
  else
    lookback_fwd_kernel<__nv_bfloat16><<<(unsigned int)(B * H), threads, 0, s>>>(a);
  return ltvqkv_host::check_launch();
}

extern "C" int ltvqkv_lookback_scan_bwd(int dtype, const void* combined, int64_t sc_b, int64_t sc_t, int64_t sc_e,
                                        const void* inits, const float* logit_bias, const void* hq,
                                        const int64_t* hq_strides, const void* hk, const int64_t* hk_strides,
                                        const void* hv, const int64_t* hv_strides, const void* grad_hq,
                                        const int64_t* gq_strides, const void* grad_hk, const int64_t* gk_strides,
                                        const void* grad_hv, const int64_t* gv_strides, void* grad_combined,
                                        int64_t gc_b, int64_t gc_t, int64_t gc_e, void* grad_inits,
                                        float* grad_logit_bias, int B, int T, int NH, int NKVH, int Da, int r,
                                        int64_t P, int64_t Q, int64_t K, int use_sigmoid, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  int rc = lb_validate(dtype, B, T, NH, NKVH, Da, r, P, Q, K);
  if (rc != LTVQKV_OK) return rc;
  const int H = NH + 2 * NKVH, D = Da * r;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if ((long long)B * H == 0) return LTVQKV_OK;
  if (T == 0) {
    // no tokens: d init = 0, d bias unchanged
    if (!grad_inits) return LTVQKV_ERR_INVALID_ARG;
    if (cudaMemsetAsync(grad_inits, 0, (size_t)B * H * D * (dtype == LTVQKV_DTYPE_F32 ? 4 : 2), s) != cudaSuccess)
      return ltvqkv_host::check_launch();
    return LTVQKV_OK;
  }
  const void* hp[3] = {hq, hk, hv};
  const void* gp[3] = {grad_hq, grad_hk, grad_hv};
  const int64_t* hst[3] = {hq_strides, hk_strides, hv_strides};
  const int64_t* gst[3] = {gq_strides, gk_strides, gv_strides};
  if (!combined || !inits || !logit_bias || !grad_combined || !grad_inits || !grad_logit_bias)
    return LTVQKV_ERR_INVALID_ARG;
  for (int w = 0; w < 3; ++w) {
    const int n = w == 0 ? NH : NKVH;
    if (n > 0 && (!hp[w] || !gp[w] || !hst[w] || !gst[w])) return LTVQKV_ERR_INVALID_ARG;
  }
  if (sc_b < 0 || sc_t < 0 || sc_e < 0 || gc_b < 0 || gc_t < 0 || gc_e < 0) return LTVQKV_ERR_STRIDE;
  if (!workspace || workspace_bytes < ltvqkv_lookback_workspace_bytes(B, NH, NKVH, Da)) return LTVQKV_ERR_WORKSPACE;
  LbArgs a = {};
  a.combined = combined; a.sc_b = sc_b; a.sc_t = sc_t; a.sc_e = sc_e;
  a.inits = inits; a.logit_bias = logit_bias;
  for (int w = 0; w < 3; ++w) {
    a.h[w] = hp[w];
    a.gh[w] = gp[w];
    for (int k = 0; k < 4; ++k) {
      a.hs[w][k] = hst[w] ? hst[w][k] : 0;
      a.gs[w][k] = gst[w] ? gst[w][k] : 0;
    }
  }
  a.grad_combined = grad_combined; a.gc_b = gc_b; a.gc_t = gc_t; a.gc_e = gc_e;
  a.grad_inits = grad_inits;
  a.bias_part = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + 256);
  a.B = B; a.T = T; a.NH = NH; a.NKVH = NKVH; a.Da = Da; a.r = r; a.D = D; a.H = H;
  a.use_sigmoid = use_sigmoid; a.P = P; a.Q = Q; a.K = K;
  a.nchunks = lb_chunks(T, P, Q);
  const size_t smem = lb_bwd_smem(D, T, K, a.ncp);
  if (smem > 220 * 1024) return LTVQKV_ERR_TOO_LARGE;  // warm-up prefix too long for the checkpoints
  const int threads = lb_threads(D);
  const size_t base = (ltvqkv_lookback_workspace_bytes(B, NH, NKVH, Da) + 255) / 256 * 256;
  // the chunk-parallel form reads and writes 8-token pieces of the production layout (the projection
  // buffer's transposed view: tokens contiguous per row, 16-byte aligned rows)
  bool prod = T % 8 == 0 && sc_t == 1 && gc_t == 1 && sc_e % 8 == 0 && gc_e % 8 == 0 && sc_b % 8 == 0 &&
              gc_b % 8 == 0 && (reinterpret_cast<uintptr_t>(combined) & 15) == 0 &&
              (reinterpret_cast<uintptr_t>(grad_combined) & 15) == 0;
  // and the saved outputs and their gradients copied as 16-byte pieces of channel-contiguous rows
  for (int w = 0; w < 3; ++w) {
    if ((w == 0 ? NH : NKVH) == 0) continue;
    for (const int64_t* st : {hst[w], gst[w]})
      prod = prod && st && st[3] == 1 && st[0] % 8 == 0 && st[1] % 8 == 0 && st[2] % 8 == 0;
    prod = prod && (reinterpret_cast<uintptr_t>(hp[w]) & 15) == 0 && (reinterpret_cast<uintptr_t>(gp[w]) & 15) == 0;
  }
  if (prod && lb_par_ok(dtype, T, D, Da, r, P, Q, K) &&
      workspace_bytes >= base + lb_par_ws_bytes(B, H, D, Da, a.nchunks, K)) {
    // chunk-parallel form (the caller's workspace holds its slots)
    char* wp = reinterpret_cast<char*>(workspace) + base;
    const size_t rows = (size_t)B * H, slots = rows * (size_t)a.nchunks, kk = (size_t)(K - 1);
    const size_t bf = (slots * kk * (size_t)lb_slot_row(D, Da) * 2 + 255) / 256 * 256;
    LbParWs w;
    w.own = reinterpret_cast<__nv_bfloat16*>(wp);
    w.pre = reinterpret_cast<__nv_bfloat16*>(wp + bf);
    w.gi = reinterpret_cast<float*>(wp + 2 * bf);
    w.bp = reinterpret_cast<float*>(wp + 2 * bf + slots * (size_t)D * 4);
    const size_t psm = kLbStages * lb_par_stage_bytes(D) +
                       sizeof(float) * (16 * (size_t)(threads / 32) + 16 * (size_t)Da +
                                        (size_t)Da * lb_chunk_gate_len(T, P, Q, K) + (size_t)(K - 1) * D);
    if (slots > 0x7fffffffULL) return LTVQKV_ERR_SHAPE;
    auto par = D == 128 ? lookback_bwd_par_kernel<128> : lookback_bwd_par_kernel<0>;
    if (psm > 48 * 1024 &&
        cudaFuncSetAttribute(par, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psm) != cudaSuccess)
      return ltvqkv_host::check_launch();
    par<<<(unsigned int)slots, threads, psm, s>>>(a, w);
    rc = ltvqkv_host::check_launch();
    if (rc != LTVQKV_OK) return rc;
    lookback_bwd_fixup_kernel<<<(unsigned int)(rows * (size_t)(a.nchunks - 1)), 256, 0, s>>>(a, w);
    rc = ltvqkv_host::check_launch();
    if (rc != LTVQKV_OK) return rc;
    lookback_bias_reduce_kernel<<<(H * Da + 127) / 128, 128, 0, s>>>(a.bias_part, grad_logit_bias, B, H, Da);
    return ltvqkv_host::check_launch();
  }
  auto kern = dtype == LTVQKV_DTYPE_F32 ? lookback_bwd_kernel<float> : lookback_bwd_kernel<__nv_bfloat16>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return ltvqkv_host::check_launch();
  kern<<<(unsigned int)(B * H), threads, smem, s>>>(a);
  rc = ltvqkv_host::check_launch();
  if (rc != LTVQKV_OK) return rc;
  lookback_bias_reduce_kernel<<<(H * Da + 127) / 128, 128, 0, s>>>(a.bias_part, grad_logit_bias, B, H, Da);
  return ltvqkv_host::check_launch();
}
