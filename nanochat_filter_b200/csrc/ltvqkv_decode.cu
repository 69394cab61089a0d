// One decode step of the filtered-QKV layer (T == 1 with cached filter state), in one launch.
//
// The reference runs this as fused_linear_transpose with T=1 (a [B,F,1] buffer rounded to the
// compute dtype), then the scan kernel with T=1, then three index_put copies into the KV cache
// (nanochat/ltv_cuda_fused_concat_head_major_register_cast_blelloch_scan_qkv_filter.py:24-73,
// nanochat/ltv_combined_qkv_computer_module.py:28-41, nanochat/kv_cache.py:212-257).
// Here one kernel computes, per (head, 16-channel slice), the projection rows it needs (the
// slice's value rows plus the logit rows of the groups they belong to) for every token,
// rounds them to the storage dtype exactly as the reference's projection buffer does, applies
// the gate and the single recurrence step h = (1 - alpha) h_prev + alpha u, and writes the
// new state (which may alias the previous state).
#include "ltvqkv_common.cuh"

namespace ltvqkv {

constexpr int kDecSlice = 16;   // value channels per CTA
constexpr int kDecBTile = 64;   // tokens per inner pass
constexpr int kDecThreads = 256;

struct DecodeArgs {
  const void* x;
  const void* w;
  const float* logit_bias;
  const void* prev[3];
  long long ps[3][3];
  const void* init_param;
  void* out[3];
  long long os[3][3];
  int B, C, NH, NKVH, Da, r, D, H, use_sigmoid;
};

LTVQKV_DEVICE void dec_split_head(int h, int NH, int NKVH, int& which, int& hloc) {
  if (h < NH) { which = 0; hloc = h; }
  else if (h < NH + NKVH) { which = 1; hloc = h - NH; }
  else { which = 2; hloc = h - NH - NKVH; }
}

// Dot product of two rows, accumulated in fp32 for bf16 storage and in double for fp32 storage
// (the oracle's definition of the fp32 projection).
template <typename T> struct DecAcc { using type = float; };
template <> struct DecAcc<float> { using type = double; };

template <typename T>
LTVQKV_DEVICE float dot_row(const T* __restrict__ a, const T* __restrict__ b, int C, int lane) {
  using Acc = typename DecAcc<T>::type;
  Acc acc = 0;
  for (int k = lane; k < C; k += 32) acc += (Acc)Elem<T>::load(a + k) * (Acc)Elem<T>::load(b + k);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  return (float)acc;
}

template <typename T>
__global__ void __launch_bounds__(kDecThreads) decode_step_kernel(DecodeArgs a) {
  __shared__ float res[2 * kDecSlice][kDecBTile];  // projected rows (rounded to T) per token
  const int h = blockIdx.x;
  const int c0 = blockIdx.y * kDecSlice;
  const int c1 = min(c0 + kDecSlice, a.D);
  const int nv = c1 - c0;
  const int g0 = c0 / a.r, g1 = (c1 - 1) / a.r;
  const int ng = g1 - g0 + 1;
  const int rows = nv + ng;
  const int head_row = h * (a.D + a.Da);
  const T* X = reinterpret_cast<const T*>(a.x);
  const T* W = reinterpret_cast<const T*>(a.w);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  int which, hloc;
  dec_split_head(h, a.NH, a.NKVH, which, hloc);

  for (int b0 = 0; b0 < a.B; b0 += kDecBTile) {
    const int nb = min(kDecBTile, a.B - b0);
    for (int pair = warp; pair < rows * nb; pair += kDecThreads / 32) {
      const int row = pair / nb, bb = pair - (pair / nb) * nb;
      const int wrow = row < nv ? head_row + c0 + row : head_row + a.D + g0 + (row - nv);
      float v = dot_row<T>(W + (long long)wrow * a.C, X + (long long)(b0 + bb) * a.C, a.C, lane);
      if (lane == 0) res[row][bb] = Elem<T>::to_f(Elem<T>::from_f(v));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nv * nb; i += kDecThreads) {
      const int cc = i / nb, bb = i - (i / nb) * nb;
      const int c = c0 + cc, b = b0 + bb;
      const int g = c / a.r;
      float l = __fadd_rn(res[nv + (g - g0)][bb], a.logit_bias[h * a.Da + g]);
      float al = l;
      if (a.use_sigmoid) al = sizeof(T) == 4 ? sigmoid_f32_exact(l) : sigmoid_f32(l);
      float hp;
      if (a.prev[0] != nullptr) {
        const long long* ps = a.ps[which];
        hp = Elem<T>::load(reinterpret_cast<const T*>(a.prev[which]) + b * ps[0] + hloc * ps[1] + c * ps[2]);
      } else {
        hp = Elem<T>::load(reinterpret_cast<const T*>(a.init_param) + (long long)h * a.D + c);
      }
      // separately rounded products and sum, the reference's fp32 update order
      float hn = __fadd_rn(__fmul_rn(__fsub_rn(1.0f, al), hp), __fmul_rn(al, res[cc][bb]));
      const long long* os = a.os[which];
      Elem<T>::store(reinterpret_cast<T*>(a.out[which]) + b * os[0] + hloc * os[1] + c * os[2], hn);
    }
    __syncthreads();
  }
}

}  // namespace ltvqkv

using namespace ltvqkv;

extern "C" int ltvqkv_decode_step(int dtype, const void* x, const void* weight, const float* logit_bias,
                                  const void* prev_q, const int64_t* pq_strides, const void* prev_k,
                                  const int64_t* pk_strides, const void* prev_v, const int64_t* pv_strides,
                                  const void* init_param, void* out_q, const int64_t* oq_strides, void* out_k,
                                  const int64_t* ok_strides, void* out_v, const int64_t* ov_strides, int B, int C,
                                  int NH, int NKVH, int Da, int r, int use_sigmoid, void* stream) {
  if (!ltvqkv_host::valid_dtype(dtype)) return LTVQKV_ERR_DTYPE;
  if (B < 0 || C < 0 || NH < 0 || NKVH < 0 || Da <= 0 || r <= 0 || NH + 2 * NKVH <= 0) return LTVQKV_ERR_SHAPE;
  if (B == 0) return LTVQKV_OK;
  if (!x || !weight || !logit_bias) return LTVQKV_ERR_INVALID_ARG;
  if (!prev_q && !init_param) return LTVQKV_ERR_INVALID_ARG;
  if (prev_q && (!pq_strides || (NKVH > 0 && (!prev_k || !prev_v || !pk_strides || !pv_strides))))
    return LTVQKV_ERR_INVALID_ARG;
  if ((NH > 0 && (!out_q || !oq_strides)) || (NKVH > 0 && (!out_k || !out_v || !ok_strides || !ov_strides)))
    return LTVQKV_ERR_INVALID_ARG;
  DecodeArgs a;
  a.x = x; a.w = weight; a.logit_bias = logit_bias;
  a.prev[0] = prev_q; a.prev[1] = prev_k; a.prev[2] = prev_v;
  a.out[0] = out_q; a.out[1] = out_k; a.out[2] = out_v;
  const int64_t* ps[3] = {pq_strides, pk_strides, pv_strides};
  const int64_t* os[3] = {oq_strides, ok_strides, ov_strides};
  for (int i = 0; i < 3; ++i)
    for (int k = 0; k < 3; ++k) {
      a.ps[i][k] = (prev_q && ps[i]) ? ps[i][k] : 0;
      a.os[i][k] = os[i] ? os[i][k] : 0;
    }
  a.init_param = init_param;
  a.B = B; a.C = C; a.NH = NH; a.NKVH = NKVH; a.Da = Da; a.r = r; a.D = Da * r;
  a.H = NH + 2 * NKVH; a.use_sigmoid = use_sigmoid;
  dim3 grid(a.H, (a.D + kDecSlice - 1) / kDecSlice);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == LTVQKV_DTYPE_BF16) decode_step_kernel<__nv_bfloat16><<<grid, kDecThreads, 0, s>>>(a);
  else decode_step_kernel<float><<<grid, kDecThreads, 0, s>>>(a);
  return ltvqkv_host::check_launch();
}
