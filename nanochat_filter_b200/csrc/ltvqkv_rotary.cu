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
template <typename S>
LTVQKV_DEVICE float rq(float v) {  // rounding to the storage dtype
  if constexpr (sizeof(S) == 4) return v;
  else return __bfloat162float(__float2bfloat16_rn(v));
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

// The rotated row element pair (j, j + d) in the storage dtype's rounding.
template <typename S>
LTVQKV_DEVICE void rotate(float x1, float x2, float c, float s, float& y1, float& y2) {
  y1 = rq<S>(__fadd_rn(rq<S>(__fmul_rn(x1, c)), rq<S>(__fmul_rn(x2, s))));
  y2 = rq<S>(__fadd_rn(rq<S>(__fmul_rn(x1, rq<S>(-s))), rq<S>(__fmul_rn(x2, c))));
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
        const float2 c = rld2<S>(a.cos, t * a.cs[0] + j), sn = rld2<S>(a.sin, t * a.cs[0] + j);
        const float2 x1 = rld2<S>(a.x[w], xb + j), x2 = rld2<S>(a.x[w], xb + j + d);
        rotate<S>(x1.x, x2.x, c.x, sn.x, y[0][n], y[2][n]);
        rotate<S>(x1.y, x2.y, c.y, sn.y, y[1][n], y[3][n]);
#pragma unroll
        for (int e = 0; e < 4; ++e) ss = __fmaf_rn(y[e][n], y[e][n], ss);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss / (float)a.D + a.eps);
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
  const float inv = rsqrtf(ss / (float)a.D + a.eps);
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
        const float2 x1 = rld2<S>(a.x[w], xb + j), x2 = rld2<S>(a.x[w], xb + j + d);
        rotate<S>(x1.x, x2.x, c.x, sn.x, y[0][n], y[2][n]);
        rotate<S>(x1.y, x2.y, c.y, sn.y, y[1][n], y[3][n]);
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
    const float r = rsqrtf(ss / (float)a.D + a.eps);
    const float k3 = r * r * r * gy / (float)a.D;
#pragma unroll
    for (int n = 0; n < NP; ++n) {
      const int j = 2 * (lane + 32 * n);
      if (j < d) {
        float dx1[2], dx2[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float dy1 = r * g[e][n] - y[e][n] * k3, dy2 = r * g[2 + e][n] - y[2 + e][n] * k3;
          dx1[e] = dy1 * c2[e][n] - dy2 * s2[e][n];
          dx2[e] = dy1 * s2[e][n] + dy2 * c2[e][n];
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
  const float r = rsqrtf(ss / (float)a.D + a.eps);
  const float k3 = r * r * r * gy / (float)a.D;
#pragma unroll
  for (int n = 0; n < kRotMaxPer; ++n) {
    const int j = lane + 32 * n;
    if (j < half) {
      const float dy1 = r * g1[n] - y1[n] * k3;
      if (rot) {
        const float dy2 = r * g2[n] - y2[n] * k3;
        rst<S>(a.out[w], ob + j * os[3], dy1 * cs_[n] - dy2 * sn_[n]);
        rst<S>(a.out[w], ob + (j + d) * os[3], dy1 * sn_[n] + dy2 * cs_[n]);
      } else {
        rst<S>(a.out[w], ob + j * os[3], dy1);
      }
    }
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
  else rotary_norm_fwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(a);
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
  else rotary_norm_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(a);
  return ltvqkv_host::check_launch();
}
