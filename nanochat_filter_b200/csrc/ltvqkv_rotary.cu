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
LTVQKV_DEVICE float rq(float v) {  // rounding to the storage dtype
  if constexpr (sizeof(S) == 4) return v;
  else return __bfloat162float(__float2bfloat16_rn(v));
}

// Row index -> (tensor, b, t, head); one warp per row, q rows first.
LTVQKV_DEVICE bool rot_row(const RotArgs& a, long long row, int& w, int& b, int& t, int& hh) {
  const long long nq = (long long)a.B * a.T * a.NH, nk = (long long)a.B * a.T * a.NKVH;
  if (row >= nq + nk) return false;
  w = row < nq ? 0 : 1;
  long long r = row < nq ? row : row - nq;
  const int nh = w == 0 ? a.NH : a.NKVH;
  hh = (int)(r % nh);
  r /= nh;
  t = (int)(r % a.T);
  b = (int)(r / a.T);
  return true;
}

// The rotated row element pair (j, j + d) in the storage dtype's rounding.
template <typename S>
LTVQKV_DEVICE void rotate(float x1, float x2, float c, float s, float& y1, float& y2) {
  y1 = rq<S>(__fadd_rn(rq<S>(__fmul_rn(x1, c)), rq<S>(__fmul_rn(x2, s))));
  y2 = rq<S>(__fadd_rn(rq<S>(__fmul_rn(x1, rq<S>(-s))), rq<S>(__fmul_rn(x2, c))));
}

constexpr int kRotMaxPer = 8;  // elements per lane and half (D <= 512; odd D <= 256)

template <typename S>
__global__ void __launch_bounds__(256) rotary_norm_fwd_kernel(RotArgs a) {
  const long long row = (long long)blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  int w, b, t, hh;
  if (!rot_row(a, row, w, b, t, hh)) return;
  const long long* xs = a.xs[w];
  const long long xb = b * xs[0] + t * xs[1] + hh * xs[2];
  const long long* os = a.os[w];
  const long long ob = b * os[0] + t * os[1] + hh * os[2];
  const bool rot = (a.D & 1) == 0;
  const int d = a.D / 2;
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

// Backward: z = y r, r = (mean(y^2) + eps)^(-1/2):  dy = r g - y r^3 (sum g y) / D;
// rotation transposed: dx1 = dy1 cos - dy2 sin,  dx2 = dy1 sin + dy2 cos.
template <typename S>
__global__ void __launch_bounds__(256) rotary_norm_bwd_kernel(RotArgs a) {
  const long long row = (long long)blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  int w, b, t, hh;
  if (!rot_row(a, row, w, b, t, hh)) return;
  const long long* xs = a.xs[w];
  const long long xb = b * xs[0] + t * xs[1] + hh * xs[2];
  const long long* gs = a.gs[w];
  const long long gb = b * gs[0] + t * gs[1] + hh * gs[2];
  const long long* os = a.os[w];
  const long long ob = b * os[0] + t * os[1] + hh * os[2];
  const bool rot = (a.D & 1) == 0;
  const int d = a.D / 2;
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
  const unsigned int grid = (unsigned int)((rows + 7) / 8);
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
  const long long rows = (long long)B * T * (NH + NKVH);
  if (rows == 0) return LTVQKV_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned int grid = (unsigned int)((rows + 7) / 8);
  if (dtype == LTVQKV_DTYPE_F32) rotary_norm_bwd_kernel<float><<<grid, 256, 0, s>>>(a);
  else rotary_norm_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(a);
  return ltvqkv_host::check_launch();
}
