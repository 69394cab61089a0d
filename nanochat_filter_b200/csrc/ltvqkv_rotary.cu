// Consumer prologue of the filtered q and k, fused: rotary embedding then QK RMS-norm.
//
// The reference's attention (nanochat/gpt.py:224-230) applies to the filter's q and k
//   apply_rotary_emb (gpt.py:101-111):  y1 = x1 cos + x2 sin,  y2 = x1 (-sin) + x2 cos,
//                                        x1 / x2 the first / second half of the head dim
//                                        (identity for an odd head dim),
//   norm (gpt.py:96-98):                 F.rms_norm over the head dim (fp32 compute, fp32 eps),
// as a chain of elementwise torch kernels. Here one warp per (batch, token, head) row reads the row
// once, rotates (each lane holds matching elements of both halves), reduces the sum of squares with
// shuffles and writes the normalised row; the backward recomputes the rotated row from the saved
// input and applies the two Jacobians in the same pass. Storage-dtype rounding follows the torch
// chain: every product and sum of the rotation is rounded to the storage dtype as torch's bf16
// elementwise ops round; the norm computes in fp32 and rounds once.
#include "ltvqkv_common.cuh"

#include <algorithm>

namespace ltvqkv {
namespace {

struct RotArgs {
  const void* x[2];      // q, k [B, T, heads, D]
  long long xs[2][4];
  const void* cos;       // [T, D/2] (any strides)
  const void* sin;
  long long cs[2];
  void* out[2];
  long long os[2][4];
  const void* g[2];      // backward: upstream gradients
  long long gs[2][4];
  int B, T, NH, NKVH, D;
  float eps;
  int vec;  // pairs of adjacent elements load and store as one (D % 4 == 0, d stride 1, even strides)
};

template <typename S>
LTVQKV_DEVICE float rld(const void* p, long long i) {
  if constexpr (sizeof(S) == 4) return reinterpret_cast<const float*>(p)[i];
  else return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}
template <typename S>
LTVQKV_DEVICE void rst(void* p, long long i, float v) {
  if constexpr (sizeof(S) == 4) reinterpret_cast<float*>(p)[i] = v;
  else reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}
template <typename S>
LTVQKV_DEVICE float2 rld2(const void* p, long long i) {
  if constexpr (sizeof(S) == 4) return *reinterpret_cast<const float2*>(reinterpret_cast<const float*>(p) + i);
  else return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(reinterpret_cast<const __nv_bfloat16*>(p) + i));
}
template <typename S>
LTVQKV_DEVICE void rst2(void* p, long long i, float x, float y) {
  if constexpr (sizeof(S) == 4) *reinterpret_cast<float2*>(reinterpret_cast<float*>(p) + i) = make_float2(x, y);
  else *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(p) + i) = __floats2bfloat162_rn(x, y);
}

// CTA row y -> (tensor, b, head): q heads first. Each warp then walks tokens (one row per token),
// so consecutive warps stream consecutive rows of the filter's head-major storage.
LTVQKV_DEVICE void rot_head(const RotArgs& a, int y, int& w, int& b, int& hh) {
  const int nq = a.B * a.NH;
  w = y < nq ? 0 : 1;
  const int r = y < nq ? y : y - nq;
  const int nh = w == 0 ? a.NH : a.NKVH;
  hh = r % nh;
  b = r / nh;
}

// The rotated row element pair (j, j + d) in the storage dtype's rounding (ltvqkv_common.cuh).
template <typename S>
LTVQKV_DEVICE void rotate(float x1, float x2, float c, float s, float& y1, float& y2) {
  if constexpr (sizeof(S) == 2) {
    rope_rotate_bf16(x1, x2, c, s, y1, y2);
  } else {
    y1 = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    y2 = __fadd_rn(__fmul_rn(x1, -s), __fmul_rn(x2, c));
  }
}

// The rotated element pairs (j, j + 1) and (j + d, j + d + 1) of a row from adjacent-pair loads at
// element offsets i1 (= j) and i2 (= j + d); bf16 rows rotate as packed pairs (ltvqkv_common.cuh).
template <typename S>
LTVQKV_DEVICE void rotate2(const void* x, long long i1, long long i2, const void* cos, const void* sin, long long ci,
                           float& y10, float& y11, float& y20, float& y21) {
  if constexpr (sizeof(S) == 2) {
    const uint32_t* x32 = reinterpret_cast<const uint32_t*>(x);
    uint32_t r1, r2;
    rope_rotate_bf16x2(x32[i1 / 2], x32[i2 / 2], reinterpret_cast<const uint32_t*>(cos)[ci / 2],
                       reinterpret_cast<const uint32_t*>(sin)[ci / 2], r1, r2);
    y10 = bf16_lo(r1); y11 = bf16_hi(r1); y20 = bf16_lo(r2); y21 = bf16_hi(r2);
  } else {
    const float2 c = rld2<S>(cos, ci), sn = rld2<S>(sin, ci);
    const float2 x1 = rld2<S>(x, i1), x2 = rld2<S>(x, i2);
    rotate<S>(x1.x, x2.x, c.x, sn.x, y10, y20);
    rotate<S>(x1.y, x2.y, c.y, sn.y, y11, y21);
  }
}

constexpr int kRotMaxPer = 8;  // elements per lane and half (D <= 512; odd D <= 256)

template <typename S>
__global__ void __launch_bounds__(256, 4) rotary_norm_fwd_kernel(RotArgs a) {
  const int lane = threadIdx.x % 32;
  int w, b, hh;
  rot_head(a, blockIdx.y, w, b, hh);
  for (int t = blockIdx.x * 8 + threadIdx.x / 32; t < a.T; t += gridDim.x * 8) {
  const long long* xs = a.xs[w];
  const long long xb = b * xs[0] + t * xs[1] + hh * xs[2];
  const long long* os = a.os[w];
  const long long ob = b * os[0] + t * os[1] + hh * os[2];
  const bool rot = (a.D & 1) == 0;
  const int d = a.D / 2;
  if (a.vec) {
    // lane holds element pairs (2p, 2p + 1), p = lane + 32 n, of both halves
    float y[4][kRotMaxPer / 2];
    float ss = 0.f;
#pragma unroll
    for (int n = 0; n < kRotMaxPer / 2; ++n) {
      const int j = 2 * (lane + 32 * n);
      y[0][n] = y[1][n] = y[2][n] = y[3][n] = 0.f;
      if (j < d) {
        rotate2<S>(a.x[w], xb + j, xb + j + d, a.cos, a.sin, t * a.cs[0] + j, y[0][n], y[1][n], y[2][n], y[3][n]);
#pragma unroll
        for (int e = 0; e < 4; ++e) ss = __fmaf_rn(y[e][n], y[e][n], ss);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rope_inv_rms(ss, a.D, a.eps);
#pragma unroll
    for (int n = 0; n < kRotMaxPer / 2; ++n) {
      const int j = 2 * (lane + 32 * n);
      if (j < d) {
        rst2<S>(a.out[w], ob + j, y[0][n] * inv, y[1][n] * inv);
        rst2<S>(a.out[w], ob + j + d, y[2][n] * inv, y[3][n] * inv);
      }
    }
    continue;
  }
  // lane holds elements j = lane + 32 n of both halves (rotation) or of the whole row (odd D)
  const int half = rot ? d : a.D;
  float y1[kRotMaxPer], y2[kRotMaxPer];
  float ss = 0.f;
#pragma unroll
  for (int n = 0; n < kRotMaxPer; ++n) {
    const int j = lane + 32 * n;
    y1[n] = y2[n] = 0.f;
    if (j < half) {
      if (rot) {
        const float c = rld<S>(a.cos, t * a.cs[0] + j * a.cs[1]), s = rld<S>(a.sin, t * a.cs[0] + j * a.cs[1]);
        rotate<S>(rld<S>(a.x[w], xb + j * xs[3]), rld<S>(a.x[w], xb + (j + d) * xs[3]), c, s, y1[n], y2[n]);
      } else {
        y1[n] = rld<S>(a.x[w], xb + j * xs[3]);
      }
      ss = __fmaf_rn(y1[n], y1[n], __fmaf_rn(y2[n], y2[n], ss));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rope_inv_rms(ss, a.D, a.eps);
#pragma unroll
  for (int n = 0; n < kRotMaxPer; ++n) {
    const int j = lane + 32 * n;
    if (j < half) {
      rst<S>(a.out[w], ob + j * os[3], y1[n] * inv);
      if (rot) rst<S>(a.out[w], ob + (j + d) * os[3], y2[n] * inv);
    }
  }
  }
}

// Head dim 128, bf16, paired access (the filter's q and k): the same per-token arithmetic as the
// paired paths above (lane l holds the element pairs (2l, 2l + 1) and (2l + 64, 2l + 65)), four
// tokens per warp iteration with every load of the four issued before any of them is used, so that
// a warp keeps 16 (forward) or 24 (backward) loads in flight instead of 4 or 6.
constexpr int kRot128Tok = 4;

__global__ void __launch_bounds__(256, 4) rotary_norm_fwd128_kernel(RotArgs a) {
  const int lane = threadIdx.x % 32;
  int w, b, hh;
  rot_head(a, blockIdx.y, w, b, hh);
  const long long* xs = a.xs[w];
  const long long* os = a.os[w];
  const int S = gridDim.x * 8;
  for (int t0 = blockIdx.x * 8 + threadIdx.x / 32; t0 < a.T; t0 += kRot128Tok * S) {
    uint32_t x1[kRot128Tok], x2[kRot128Tok], cw[kRot128Tok], sw[kRot128Tok];
#pragma unroll
    for (int u = 0; u < kRot128Tok; ++u) {
      const int t = t0 + u * S;
      x1[u] = x2[u] = cw[u] = sw[u] = 0u;
      if (t < a.T) {
        const __nv_bfloat16* xr = reinterpret_cast<const __nv_bfloat16*>(a.x[w]) + b * xs[0] + t * xs[1] + hh * xs[2];
        x1[u] = __ldg(reinterpret_cast<const uint32_t*>(xr) + lane);
        x2[u] = __ldg(reinterpret_cast<const uint32_t*>(xr + 64) + lane);
        cw[u] = __ldg(reinterpret_cast<const uint32_t*>(reinterpret_cast<const __nv_bfloat16*>(a.cos) + t * a.cs[0]) + lane);
        sw[u] = __ldg(reinterpret_cast<const uint32_t*>(reinterpret_cast<const __nv_bfloat16*>(a.sin) + t * a.cs[0]) + lane);
      }
    }
#pragma unroll
    for (int u = 0; u < kRot128Tok; ++u) {
      const int t = t0 + u * S;
      if (t >= a.T) break;  // warp-uniform
      uint32_t r1, r2;
      rope_rotate_bf16x2(x1[u], x2[u], cw[u], sw[u], r1, r2);
      const float y0 = bf16_lo(r1), y1 = bf16_hi(r1), y2 = bf16_lo(r2), y3 = bf16_hi(r2);
      float ss = __fmaf_rn(y0, y0, 0.f);
      ss = __fmaf_rn(y1, y1, ss);
      ss = __fmaf_rn(y2, y2, ss);
      ss = __fmaf_rn(y3, y3, ss);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float inv = rope_inv_rms(ss, 128, a.eps);
      __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(a.out[w]) + b * os[0] + t * os[1] + hh * os[2];
      reinterpret_cast<uint32_t*>(orow)[lane] = pack_bf16x2(y0 * inv, y1 * inv);
      reinterpret_cast<uint32_t*>(orow + 64)[lane] = pack_bf16x2(y2 * inv, y3 * inv);
    }
  }
}

__global__ void __launch_bounds__(256, 4) rotary_norm_bwd128_kernel(RotArgs a) {
  const int lane = threadIdx.x % 32;
  int w, b, hh;
  rot_head(a, blockIdx.y, w, b, hh);
  const long long* xs = a.xs[w];
  const long long* gs = a.gs[w];
  const long long* os = a.os[w];
  const int S = gridDim.x * 8;
  for (int t0 = blockIdx.x * 8 + threadIdx.x / 32; t0 < a.T; t0 += kRot128Tok * S) {
    uint32_t x1[kRot128Tok], x2[kRot128Tok], cw[kRot128Tok], sw[kRot128Tok], g1[kRot128Tok], g2[kRot128Tok];
#pragma unroll
    for (int u = 0; u < kRot128Tok; ++u) {
      const int t = t0 + u * S;
      x1[u] = x2[u] = cw[u] = sw[u] = g1[u] = g2[u] = 0u;
      if (t < a.T) {
        const __nv_bfloat16* xr = reinterpret_cast<const __nv_bfloat16*>(a.x[w]) + b * xs[0] + t * xs[1] + hh * xs[2];
        const __nv_bfloat16* gr = reinterpret_cast<const __nv_bfloat16*>(a.g[w]) + b * gs[0] + t * gs[1] + hh * gs[2];
        x1[u] = __ldg(reinterpret_cast<const uint32_t*>(xr) + lane);
        x2[u] = __ldg(reinterpret_cast<const uint32_t*>(xr + 64) + lane);
        g1[u] = __ldg(reinterpret_cast<const uint32_t*>(gr) + lane);
        g2[u] = __ldg(reinterpret_cast<const uint32_t*>(gr + 64) + lane);
        cw[u] = __ldg(reinterpret_cast<const uint32_t*>(reinterpret_cast<const __nv_bfloat16*>(a.cos) + t * a.cs[0]) + lane);
        sw[u] = __ldg(reinterpret_cast<const uint32_t*>(reinterpret_cast<const __nv_bfloat16*>(a.sin) + t * a.cs[0]) + lane);
      }
    }
#pragma unroll
    for (int u = 0; u < kRot128Tok; ++u) {
      const int t = t0 + u * S;
      if (t >= a.T) break;  // warp-uniform
      uint32_t r1, r2;
      rope_rotate_bf16x2(x1[u], x2[u], cw[u], sw[u], r1, r2);
      const float y[4] = {bf16_lo(r1), bf16_hi(r1), bf16_lo(r2), bf16_hi(r2)};
      const float g[4] = {bf16_lo(g1[u]), bf16_hi(g1[u]), bf16_lo(g2[u]), bf16_hi(g2[u])};
      float ss = 0.f, gy = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        ss = __fmaf_rn(y[e], y[e], ss);
        gy = __fmaf_rn(g[e], y[e], gy);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        ss += __shfl_xor_sync(0xffffffffu, ss, o);
        gy += __shfl_xor_sync(0xffffffffu, gy, o);
      }
      const float r = rope_inv_rms(ss, 128, a.eps);
      const float k3 = rope_k3(r, gy, 128);
      float dx1[2], dx2[2];
#pragma unroll
      for (int e = 0; e < 2; ++e)
        rope_norm_bwd(r, k3, g[e], g[2 + e], y[e], y[2 + e], bf16_lane(cw[u], e), bf16_lane(sw[u], e), dx1[e], dx2[e]);
      __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(a.out[w]) + b * os[0] + t * os[1] + hh * os[2];
      reinterpret_cast<uint32_t*>(orow)[lane] = pack_bf16x2(dx1[0], dx1[1]);
      reinterpret_cast<uint32_t*>(orow + 64)[lane] = pack_bf16x2(dx2[0], dx2[1]);
    }
  }
}

// Backward: z = y r, r = (mean(y^2) + eps)^(-1/2):  dy = r g - y r^3 (sum g y) / D;
// rotation transposed: dx1 = dy1 cos - dy2 sin,  dx2 = dy1 sin + dy2 cos.
template <typename S>
__global__ void __launch_bounds__(256, 3) rotary_norm_bwd_kernel(RotArgs a) {
  const int lane = threadIdx.x % 32;
  int w, b, hh;
  rot_head(a, blockIdx.y, w, b, hh);
  for (int t = blockIdx.x * 8 + threadIdx.x / 32; t < a.T; t += gridDim.x * 8) {
  const long long* xs = a.xs[w];
  const long long xb = b * xs[0] + t * xs[1] + hh * xs[2];
  const long long* gs = a.gs[w];
  const long long gb = b * gs[0] + t * gs[1] + hh * gs[2];
  const long long* os = a.os[w];
  const long long ob = b * os[0] + t * os[1] + hh * os[2];
  const bool rot = (a.D & 1) == 0;
  const int d = a.D / 2;
  if (a.vec) {
    constexpr int NP = kRotMaxPer / 2;
    float y[4][NP], g[4][NP], c2[2][NP], s2[2][NP];
    float ss = 0.f, gy = 0.f;
#pragma unroll
    for (int n = 0; n < NP; ++n) {
      const int j = 2 * (lane + 32 * n);
#pragma unroll
      for (int e = 0; e < 4; ++e) y[e][n] = g[e][n] = 0.f;
      c2[0][n] = c2[1][n] = s2[0][n] = s2[1][n] = 0.f;
      if (j < d) {
        const float2 c = rld2<S>(a.cos, t * a.cs[0] + j), sn = rld2<S>(a.sin, t * a.cs[0] + j);
        c2[0][n] = c.x; c2[1][n] = c.y; s2[0][n] = sn.x; s2[1][n] = sn.y;
        rotate2<S>(a.x[w], xb + j, xb + j + d, a.cos, a.sin, t * a.cs[0] + j, y[0][n], y[1][n], y[2][n], y[3][n]);
        const float2 ga = rld2<S>(a.g[w], gb + j), gbb = rld2<S>(a.g[w], gb + j + d);
        g[0][n] = ga.x; g[1][n] = ga.y; g[2][n] = gbb.x; g[3][n] = gbb.y;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          ss = __fmaf_rn(y[e][n], y[e][n], ss);
          gy = __fmaf_rn(g[e][n], y[e][n], gy);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ss += __shfl_xor_sync(0xffffffffu, ss, o);
      gy += __shfl_xor_sync(0xffffffffu, gy, o);
    }
    const float r = rope_inv_rms(ss, a.D, a.eps);
    const float k3 = rope_k3(r, gy, a.D);
#pragma unroll
    for (int n = 0; n < NP; ++n) {
      const int j = 2 * (lane + 32 * n);
      if (j < d) {
        float dx1[2], dx2[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          rope_norm_bwd(r, k3, g[e][n], g[2 + e][n], y[e][n], y[2 + e][n], c2[e][n], s2[e][n], dx1[e], dx2[e]);
        }
        rst2<S>(a.out[w], ob + j, dx1[0], dx1[1]);
        rst2<S>(a.out[w], ob + j + d, dx2[0], dx2[1]);
      }
    }
    continue;
  }
  const int half = rot ? d : a.D;
  float y1[kRotMaxPer], y2[kRotMaxPer], g1[kRotMaxPer], g2[kRotMaxPer], cs_[kRotMaxPer], sn_[kRotMaxPer];
  float ss = 0.f, gy = 0.f;
#pragma unroll
  for (int n = 0; n < kRotMaxPer; ++n) {
    const int j = lane + 32 * n;
    y1[n] = y2[n] = g1[n] = g2[n] = cs_[n] = sn_[n] = 0.f;
    if (j < half) {
      if (rot) {
        cs_[n] = rld<S>(a.cos, t * a.cs[0] + j * a.cs[1]);
        sn_[n] = rld<S>(a.sin, t * a.cs[0] + j * a.cs[1]);
        rotate<S>(rld<S>(a.x[w], xb + j * xs[3]), rld<S>(a.x[w], xb + (j + d) * xs[3]), cs_[n], sn_[n], y1[n], y2[n]);
        g2[n] = rld<S>(a.g[w], gb + (j + d) * gs[3]);
      } else {
        y1[n] = rld<S>(a.x[w], xb + j * xs[3]);
      }
      g1[n] = rld<S>(a.g[w], gb + j * gs[3]);
      ss = __fmaf_rn(y1[n], y1[n], __fmaf_rn(y2[n], y2[n], ss));
      gy = __fmaf_rn(g1[n], y1[n], __fmaf_rn(g2[n], y2[n], gy));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
    gy += __shfl_xor_sync(0xffffffffu, gy, o);
  }
  const float r = rope_inv_rms(ss, a.D, a.eps);
  const float k3 = rope_k3(r, gy, a.D);
#pragma unroll
  for (int n = 0; n < kRotMaxPer; ++n) {
    const int j = lane + 32 * n;
    if (j < half) {
      if (rot) {
        float dx1, dx2;
        rope_norm_bwd(r, k3, g1[n], g2[n], y1[n], y2[n], cs_[n], sn_[n], dx1, dx2);
        rst<S>(a.out[w], ob + j * os[3], dx1);
        rst<S>(a.out[w], ob + (j + d) * os[3], dx2);
      } else {
        rst<S>(a.out[w], ob + j * os[3], __fmaf_rn(r, g1[n], -__fmul_rn(y1[n], k3)));
      }
    }
  }
  }
}

// ------------------------------------------------------------------------------------------
// Backward of the prologue folded into the fused forward (ltvqkv_proj_scan_fwd_ckpt_rope): that
// forward never stores the raw q / k, so the rotary backward replays them from the scan's
// checkpoints. One CTA (128 threads) per (32-token chunk, batch, q or k head), consecutive CTAs on
// consecutive chunks of one row (their value-row and gradient reads are adjacent in memory; the
// tables are L2-resident either way). Replay: thread c walks channel c of the chunk from
// the state entering it (the checkpoint, or the initial state for the first chunk) with the
// forward's arithmetic (E = fma(1 - a, E, a u), a = sigmoid(logit + bias), u the stored bf16
// projection value), so the rebuilt h_t are the forward's raw outputs bit for bit; they go to
// shared memory as a [32 token][128 channel] tile. Then each warp takes 8 tokens with the standalone
// backward's lane layout and arithmetic (pairs (2l, 2l + 1) and (2l + 64, 2l + 65)), so dq / dk equal
// ltvqkv_rotary_qk_norm_bwd's on the stored raw outputs bit for bit.
// ------------------------------------------------------------------------------------------
struct RopeCkptArgs {
  const __nv_bfloat16* combined;  // [B][F][T]
  const __nv_bfloat16* inits;     // [B][H][128] (sequences inits_bs elements apart; 0: shared)
  long long inits_bs;
  const float* logit_bias;        // [H]
  const float* ckpt;              // [B][H][T / 32][128]
  const __nv_bfloat16* cos;       // [T][64], rows cs elements apart
  const __nv_bfloat16* sin;
  long long cs;
  const __nv_bfloat16* g[2];      // gradients of the rotated, normalised q / k
  long long gs[2][4];
  __nv_bfloat16* d[2];            // gradients of the raw q / k
  long long ds[2][4];
  int B, T, NH, NKVH, H, F, nchunks, use_sigmoid;
  float eps;
};

constexpr int kRopeTT = 32;

__global__ void __launch_bounds__(128, 6) rope_bwd_ckpt_kernel(RopeCkptArgs a) {
  __shared__ float gate[2][kRopeTT];                 // (1 - a_t, a_t)
  __shared__ __align__(16) uint32_t hs[kRopeTT][64];  // raw h_t, bf16 pairs
  const int j = blockIdx.x % a.nchunks, row = blockIdx.x / a.nchunks;
  const int b = row / (a.NH + a.NKVH), h = row % (a.NH + a.NKVH);  // q heads, then k heads
  const int w = h < a.NH ? 0 : 1, hloc = h < a.NH ? h : h - a.NH;
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
  const int t0 = j * kRopeTT;
  const long long frow = (long long)b * a.F + (long long)h * 129;
  if (tid < kRopeTT) {
    const float l = __bfloat162float(a.combined[(frow + 128) * a.T + t0 + tid]) + a.logit_bias[h];
    const float al = a.use_sigmoid ? sigmoid_f32(l) : l;
    gate[0][tid] = 1.0f - al;
    gate[1][tid] = al;
  }
  float E = j == 0 ? __bfloat162float(a.inits[(long long)b * a.inits_bs + (long long)h * 128 + tid])
                   : a.ckpt[(((long long)b * a.H + h) * a.nchunks + (j - 1)) * 128 + tid];
  const uint4* urow = reinterpret_cast<const uint4*>(a.combined + (frow + tid) * a.T + t0);
  uint4 u4[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) u4[k] = __ldg(urow + k);
  // this warp's 8 tokens: table words and output gradients, loaded with the value rows (one latency)
  const long long* gs = a.gs[w];
  const long long* dsr = a.ds[w];
  uint32_t cw8[8], sw8[8], gA8[8], gB8[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int t = t0 + warp * 8 + e;
    const long long tr = (long long)t * a.cs;
    cw8[e] = __ldg(reinterpret_cast<const uint32_t*>(a.cos + tr) + lane);
    sw8[e] = __ldg(reinterpret_cast<const uint32_t*>(a.sin + tr) + lane);
    const __nv_bfloat16* gr = a.g[w] + b * gs[0] + hloc * gs[1] + t * gs[2];
    gA8[e] = __ldg(reinterpret_cast<const uint32_t*>(gr) + lane);
    gB8[e] = __ldg(reinterpret_cast<const uint32_t*>(gr + 64) + lane);
  }
  __syncthreads();
  __nv_bfloat16* hs16 = reinterpret_cast<__nv_bfloat16*>(&hs[0][0]);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t wv[4] = {u4[k].x, u4[k].y, u4[k].z, u4[k].w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int t = 8 * k + e;
      const float u = (e & 1) ? bf16_hi(wv[e / 2]) : bf16_lo(wv[e / 2]);
      E = __fmaf_rn(gate[0][t], E, __fmul_rn(gate[1][t], u));
      hs16[t * 128 + tid] = __float2bfloat16_rn(E);
    }
  }
  __syncthreads();
  // rotary + norm backward of this warp's 8 tokens, four at a time
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t cw[4], sw[4], gA[4], gB[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      cw[e] = cw8[4 * half + e]; sw[e] = sw8[4 * half + e];
      gA[e] = gA8[4 * half + e]; gB[e] = gB8[4 * half + e];
    }
    float y[4][4], g[4][4], ss[4], gy[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int t = warp * 8 + half * 4 + e;
      uint32_t r1, r2;
      rope_rotate_bf16x2(hs[t][lane], hs[t][32 + lane], cw[e], sw[e], r1, r2);
      y[e][0] = bf16_lo(r1); y[e][1] = bf16_hi(r1); y[e][2] = bf16_lo(r2); y[e][3] = bf16_hi(r2);
      g[e][0] = bf16_lo(gA[e]); g[e][1] = bf16_hi(gA[e]); g[e][2] = bf16_lo(gB[e]); g[e][3] = bf16_hi(gB[e]);
      ss[e] = 0.f;
      gy[e] = 0.f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        ss[e] = __fmaf_rn(y[e][q], y[e][q], ss[e]);
        gy[e] = __fmaf_rn(g[e][q], y[e][q], gy[e]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        ss[e] += __shfl_xor_sync(0xffffffffu, ss[e], o);
        gy[e] += __shfl_xor_sync(0xffffffffu, gy[e], o);
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int t = t0 + warp * 8 + half * 4 + e;
      const float r = rope_inv_rms(ss[e], 128, a.eps);
      const float k3 = rope_k3(r, gy[e], 128);
      float dx1[2], dx2[2];
#pragma unroll
      for (int q = 0; q < 2; ++q)
        rope_norm_bwd(r, k3, g[e][q], g[e][2 + q], y[e][q], y[e][2 + q], bf16_lane(cw[e], q), bf16_lane(sw[e], q),
                      dx1[q], dx2[q]);
      __nv_bfloat16* dr = a.d[w] + b * dsr[0] + hloc * dsr[1] + t * dsr[2];
      reinterpret_cast<uint32_t*>(dr)[lane] = pack_bf16x2(dx1[0], dx1[1]);
      reinterpret_cast<uint32_t*>(dr + 64)[lane] = pack_bf16x2(dx2[0], dx2[1]);
    }
  }
}

int rot_setup(RotArgs& a, int dtype, const void* q, const int64_t* qs, const void* k, const int64_t* ks,
              const void* cos, const void* sin, const int64_t* css, void* oq, const int64_t* oqs, void* ok,
              const int64_t* oks, int B, int T, int NH, int NKVH, int D, float eps) {
  if (!ltvqkv_host::valid_dtype(dtype)) return LTVQKV_ERR_DTYPE;
  if (B < 0 || T < 0 || NH < 0 || NKVH < 0 || D < 1 || D > 32 * 2 * kRotMaxPer ||
      ((D & 1) && D > 32 * kRotMaxPer))
    return LTVQKV_ERR_SHAPE;
  if (!cos || !sin || !css || (NH > 0 && (!q || !qs || !oq || !oqs)) || (NKVH > 0 && (!k || !ks || !ok || !oks)))
    return LTVQKV_ERR_INVALID_ARG;
  a = RotArgs{};
  a.x[0] = q; a.x[1] = k; a.out[0] = oq; a.out[1] = ok;
  for (int i = 0; i < 4; ++i) {
    a.xs[0][i] = qs ? qs[i] : 0; a.xs[1][i] = ks ? ks[i] : 0;
    a.os[0][i] = oqs ? oqs[i] : 0; a.os[1][i] = oks ? oks[i] : 0;
  }
  a.cos = cos; a.sin = sin; a.cs[0] = css[0]; a.cs[1] = css[1];
  a.B = B; a.T = T; a.NH = NH; a.NKVH = NKVH; a.D = D; a.eps = eps;
  // paired accesses: D % 4 == 0, unit d stride and even other strides, pointers aligned to a pair
  const size_t pair = dtype == LTVQKV_DTYPE_F32 ? 8 : 4;
  auto ok4 = [&](const void* p, const long long* st) {
    return p == nullptr || ((reinterpret_cast<uintptr_t>(p) % pair) == 0 && st[3] == 1 && st[0] % 2 == 0 &&
                            st[1] % 2 == 0 && st[2] % 2 == 0);
  };
  a.vec = D % 4 == 0 && css[1] == 1 && css[0] % 2 == 0 && reinterpret_cast<uintptr_t>(cos) % pair == 0 &&
          reinterpret_cast<uintptr_t>(sin) % pair == 0 && ok4(q, a.xs[0]) && ok4(k, a.xs[1]) && ok4(oq, a.os[0]) &&
          ok4(ok, a.os[1]);
  return LTVQKV_OK;
}

}  // namespace
}  // namespace ltvqkv

using namespace ltvqkv;

extern "C" int ltvqkv_rotary_qk_norm_fwd(int dtype, const void* q, const int64_t* q_strides, const void* k,
                                         const int64_t* k_strides, const void* cos, const void* sin,
                                         const int64_t* cs_strides, void* out_q, const int64_t* oq_strides,
                                         void* out_k, const int64_t* ok_strides, int B, int T, int NH, int NKVH,
                                         int D, float eps, void* stream) {
  RotArgs a;
  int rc = rot_setup(a, dtype, q, q_strides, k, k_strides, cos, sin, cs_strides, out_q, oq_strides, out_k,
                     ok_strides, B, T, NH, NKVH, D, eps);
  if (rc != LTVQKV_OK) return rc;
  const long long rows = (long long)B * T * (NH + NKVH);
  if (rows == 0) return LTVQKV_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // x: token tiles (each warp walks tokens w, w + 8 gridDim.x, ...), y: the q and k head rows
  const dim3 grid((unsigned int)std::min(64, (T + 63) / 64), (unsigned int)(B * (NH + NKVH)));
  if (B * (NH + NKVH) > 65535) return LTVQKV_ERR_SHAPE;
  if (dtype == LTVQKV_DTYPE_F32) rotary_norm_fwd_kernel<float><<<grid, 256, 0, s>>>(a);
  else if (a.vec && D == 128) rotary_norm_fwd128_kernel<<<grid, 256, 0, s>>>(a);
  else rotary_norm_fwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(a);
  return ltvqkv_host::check_launch();
}

extern "C" int ltvqkv_rotary_qk_norm_bwd_ckpt(int dtype, const void* combined, const void* inits, int64_t inits_bs,
                                              const float* logit_bias, const float* ckpt, const void* rope_cos,
                                              const void* rope_sin, int64_t rope_stride, float eps,
                                              const void* grad_q, const int64_t* gq_strides, const void* grad_k,
                                              const int64_t* gk_strides, void* dq, const int64_t* dq_strides,
                                              void* dk, const int64_t* dk_strides, int B, int T, int NH, int NKVH,
                                              int Da, int r, int use_sigmoid, void* stream) {
  if (dtype != LTVQKV_DTYPE_BF16) return LTVQKV_ERR_DTYPE;
  if (B < 0 || T < 0 || NH < 0 || NKVH < 0 || Da != 1 || r != 128 || T % kRopeTT != 0) return LTVQKV_ERR_SHAPE;
  const int H = NH + 2 * NKVH;
  if (!combined || !inits || !logit_bias || !ckpt || !rope_cos || !rope_sin) return LTVQKV_ERR_INVALID_ARG;
  if ((NH > 0 && (!grad_q || !gq_strides || !dq || !dq_strides)) ||
      (NKVH > 0 && (!grad_k || !gk_strides || !dk || !dk_strides)))
    return LTVQKV_ERR_INVALID_ARG;
  if (inits_bs != 0 && inits_bs != (int64_t)H * 128) return LTVQKV_ERR_STRIDE;
  if (rope_stride < 64 || rope_stride % 2 != 0 || (reinterpret_cast<uintptr_t>(rope_cos) & 3u) != 0 ||
      (reinterpret_cast<uintptr_t>(rope_sin) & 3u) != 0)
    return LTVQKV_ERR_STRIDE;
  // the u rows are read as 16-byte pieces: combined 16-byte aligned with T % 8 == 0 (T % 32 == 0 here);
  // gradient rows as bf16 pairs: unit channel stride, even other strides, 4-byte aligned
  if ((reinterpret_cast<uintptr_t>(combined) & 15u) != 0) return LTVQKV_ERR_ALIGN;
  auto pairs_ok = [](const void* p, const int64_t* st) {
    return p == nullptr || ((reinterpret_cast<uintptr_t>(p) & 3u) == 0 && st[3] == 1 && st[0] % 2 == 0 &&
                            st[1] % 2 == 0 && st[2] % 2 == 0);
  };
  if (!pairs_ok(NH > 0 ? grad_q : nullptr, gq_strides) || !pairs_ok(NKVH > 0 ? grad_k : nullptr, gk_strides) ||
      !pairs_ok(NH > 0 ? dq : nullptr, dq_strides) || !pairs_ok(NKVH > 0 ? dk : nullptr, dk_strides))
    return LTVQKV_ERR_STRIDE;
  const long long ctas = (long long)B * (NH + NKVH) * (T / kRopeTT);
  if (ctas == 0) return LTVQKV_OK;
  if (ctas > 0x7fffffffLL) return LTVQKV_ERR_SHAPE;
  RopeCkptArgs a = {};
  a.combined = reinterpret_cast<const __nv_bfloat16*>(combined);
  a.inits = reinterpret_cast<const __nv_bfloat16*>(inits);
  a.inits_bs = inits_bs;
  a.logit_bias = logit_bias;
  a.ckpt = ckpt;
  a.cos = reinterpret_cast<const __nv_bfloat16*>(rope_cos);
  a.sin = reinterpret_cast<const __nv_bfloat16*>(rope_sin);
  a.cs = rope_stride;
  a.g[0] = reinterpret_cast<const __nv_bfloat16*>(grad_q);
  a.g[1] = reinterpret_cast<const __nv_bfloat16*>(grad_k);
  a.d[0] = reinterpret_cast<__nv_bfloat16*>(dq);
  a.d[1] = reinterpret_cast<__nv_bfloat16*>(dk);
  for (int i = 0; i < 4; ++i) {
    a.gs[0][i] = gq_strides ? gq_strides[i] : 0; a.gs[1][i] = gk_strides ? gk_strides[i] : 0;
    a.ds[0][i] = dq_strides ? dq_strides[i] : 0; a.ds[1][i] = dk_strides ? dk_strides[i] : 0;
  }
  a.B = B; a.T = T; a.NH = NH; a.NKVH = NKVH; a.H = H; a.F = H * 129; a.nchunks = T / kRopeTT;
  a.use_sigmoid = use_sigmoid; a.eps = eps;
  rope_bwd_ckpt_kernel<<<(unsigned int)ctas, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return ltvqkv_host::check_launch();
}

extern "C" int ltvqkv_rotary_qk_norm_bwd(int dtype, const void* q, const int64_t* q_strides, const void* k,
                                         const int64_t* k_strides, const void* cos, const void* sin,
                                         const int64_t* cs_strides, const void* grad_q, const int64_t* gq_strides,
                                         const void* grad_k, const int64_t* gk_strides, void* dq,
                                         const int64_t* dq_strides, void* dk, const int64_t* dk_strides, int B,
                                         int T, int NH, int NKVH, int D, float eps, void* stream) {
  RotArgs a;
  int rc = rot_setup(a, dtype, q, q_strides, k, k_strides, cos, sin, cs_strides, dq, dq_strides, dk, dk_strides,
                     B, T, NH, NKVH, D, eps);
  if (rc != LTVQKV_OK) return rc;
  if ((NH > 0 && (!grad_q || !gq_strides)) || (NKVH > 0 && (!grad_k || !gk_strides))) return LTVQKV_ERR_INVALID_ARG;
  a.g[0] = grad_q; a.g[1] = grad_k;
  for (int i = 0; i < 4; ++i) {
    a.gs[0][i] = gq_strides ? gq_strides[i] : 0;
    a.gs[1][i] = gk_strides ? gk_strides[i] : 0;
  }
  const size_t pair = dtype == LTVQKV_DTYPE_F32 ? 8 : 4;
  for (int w = 0; w < 2; ++w)
    if (a.g[w] && ((reinterpret_cast<uintptr_t>(a.g[w]) % pair) != 0 || a.gs[w][3] != 1 || a.gs[w][0] % 2 ||
                   a.gs[w][1] % 2 || a.gs[w][2] % 2))
      a.vec = 0;
  const long long rows = (long long)B * T * (NH + NKVH);
  if (rows == 0) return LTVQKV_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // x: token tiles (each warp walks tokens w, w + 8 gridDim.x, ...), y: the q and k head rows
  const dim3 grid((unsigned int)std::min(64, (T + 63) / 64), (unsigned int)(B * (NH + NKVH)));
  if (B * (NH + NKVH) > 65535) return LTVQKV_ERR_SHAPE;
  if (dtype == LTVQKV_DTYPE_F32) rotary_norm_bwd_kernel<float><<<grid, 256, 0, s>>>(a);
  else if (a.vec && D == 128) rotary_norm_bwd128_kernel<<<grid, 256, 0, s>>>(a);
  else rotary_norm_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(a);
  return ltvqkv_host::check_launch();
}
