// Projection GEMMs of the filtered-QKV layer on sm_100a tensor cores.
//
//   forward  (reference cpp_ewma/src/fused_linear_transpose_forward.cu:23-58):
//     out[b, f, t] = sum_k W[f, k] x[b, t, k]
//       single-CTA tiles 128 f x 256 t (ltvqkv_gemm_fwd.cuh)
//   backward (reference cpp_ewma/src/fused_linear_transpose_backward.cu:22-132, which issues
//   2*B serial cuBLAS calls): in ONE launch
//     dW[f, k]    = sum_b sum_t g[b, f, t] x[b, t, k]   tiles: M = k, N = f, K = t over the batches;
//                   fp32 dW takes the batches in two halves: the half that finishes first stores
//                   its tile, the other adds its own to it (two addends, so the result is the same
//                   on every run; no zero fill, no floating-point atomics)
//     dx[b, t, k] = sum_f g[b, f, t] W[f, k]           tiles: M = t, N = k, K = f
// The backward's tensor-core kernel (CTA pairs, tcgen05 cta_group::2) is in ltvqkv_gemm_pair.cuh.
#include <algorithm>
#include <mutex>
#include <set>
#include <utility>

#include "ltvqkv_common.cuh"
#include "ltvqkv_gemm_fwd.cuh"
#include "ltvqkv_gemm_pair.cuh"
#include "ltvqkv_proj_scan.cuh"

namespace ltvqkv {

// ------------------------------------------------------------------------------------------
// CUDA-core GEMM for fp32 and for bf16 shapes the TMA path cannot address (row pitches not a
// multiple of 16 bytes).
//   C[ob][m][n] = sum_rb sum_k A[ob,rb][m][k] * B[ob,rb][n][k]
// fp32 inputs accumulate in double (a product of two floats is exact in double), so the fp32
// result is the correctly rounded sum up to double rounding — the oracle's definition; bf16
// inputs accumulate in fp32 like the tensor-core path.
// ------------------------------------------------------------------------------------------
template <typename Tin> struct AccOf { using type = float; };
template <> struct AccOf<float> { using type = double; };

struct SimtArgs {
  const void* A;
  const void* B;
  void* C;
  long long a_ob, a_rb, a_m, a_k;
  long long b_ob, b_rb, b_n, b_k;
  long long c_ob, c_m, c_n;
  int M, N, K, red_batches;
};

template <typename Tin, typename Tout>
__global__ void __launch_bounds__(256) gemm_simt_kernel(SimtArgs a) {
  constexpr int TM = 64, TN = 64, TK = 16;
  __shared__ float As[TK][TM + 4];
  __shared__ float Bs[TK][TN + 4];
  const int ob = blockIdx.z;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  using Acc = typename AccOf<Tin>::type;
  Acc acc[4][4] = {};
  const Tin* Ab = reinterpret_cast<const Tin*>(a.A) + ob * a.a_ob;
  const Tin* Bb = reinterpret_cast<const Tin*>(a.B) + ob * a.b_ob;
  for (int rb = 0; rb < a.red_batches; ++rb) {
    const Tin* Ar = Ab + rb * a.a_rb;
    const Tin* Br = Bb + rb * a.b_rb;
    for (int k0 = 0; k0 < a.K; k0 += TK) {
      for (int i = threadIdx.x; i < TK * TM; i += 256) {
        int kk, mm;
        if (a.a_k == 1) { mm = i / TK; kk = i % TK; } else { kk = i / TM; mm = i % TM; }
        int m = m0 + mm, k = k0 + kk;
        As[kk][mm] = (m < a.M && k < a.K) ? Elem<Tin>::load(Ar + m * a.a_m + k * a.a_k) : 0.f;
      }
      for (int i = threadIdx.x; i < TK * TN; i += 256) {
        int kk, nn;
        if (a.b_k == 1) { nn = i / TK; kk = i % TK; } else { kk = i / TN; nn = i % TN; }
        int n = n0 + nn, k = k0 + kk;
        Bs[kk][nn] = (n < a.N && k < a.K) ? Elem<Tin>::load(Br + n * a.b_n + k * a.b_k) : 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < TK; ++kk) {
        float av[4], bv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = (Acc)av[i] * (Acc)bv[j] + acc[i][j];
      }
      __syncthreads();
    }
  }
  Tout* Cb = reinterpret_cast<Tout*>(a.C) + ob * a.c_ob;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
      if (m < a.M && n < a.N) Elem<Tout>::store(Cb + m * a.c_m + n * a.c_n, (float)acc[i][j]);
    }
}

}  // namespace ltvqkv

using namespace ltvqkv;

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------
namespace {

// MN-major operand of the pair GEMM as one 16 KB box: element (mn, k, batch) of a tensor whose mn
// index is contiguous (extent mn_ext, a multiple of 64), k rows `k_pitch` bytes apart and batches
// `b_pitch` bytes apart, viewed as 4-D {64 mn_lo, k, mn_ext / 64 mn_hi, batch}; box {64, 64, 2, 1}
// fills shared memory as [mn_hi][k][mn_lo] with the 128-byte swizzle, the canonical MN-major layout
// of two 64-wide blocks that two separate 3-D boxes would write.
bool make_mn_blk_map(CUtensorMap* m, const void* base, uint64_t mn_ext, uint64_t k_ext, uint64_t batches,
                     uint64_t k_pitch, uint64_t b_pitch) {
  const uint64_t dims[4] = {64, k_ext, mn_ext / 64, batches};
  const uint64_t strides[3] = {k_pitch, 128, b_pitch};
  const uint32_t box[4] = {64, 64, 2, 1};
  return ltvqkv_host::encode_tiled_map(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box,
                                       CU_TENSOR_MAP_SWIZZLE_128B);
}

// 3-D tiled map: dims (d0 innermost, d1, d2), byte strides of d1 and d2, box (box0, box1, 1).
bool make_map(CUtensorMap* m, bool f32, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
              uint64_t s2, uint32_t box0, uint32_t box1, bool swizzle = true) {
  const uint64_t dims[3] = {d0, d1, d2};
  const uint64_t strides[2] = {s1, s2};
  const uint32_t box[3] = {box0, box1, 1};
  return ltvqkv_host::encode_tiled_map(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                                       base, dims, strides, box,
                                       swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE);
}

void finalize_pair(PairProblem& p, int K) {
  p.m_tiles = (p.M + 255) / 256;
  p.n_tiles = (p.N + kPairBN - 1) / kPairBN;
  p.k_blocks = (K + kPairBK - 1) / kPairBK;
  p.num_tiles = p.out_batches * p.splits * p.m_tiles * p.n_tiles;
}

// Persistent launch: one cluster (CTA pair) per SM pair that can be resident, at most one per tile.
// maps: A and B of problem 0, then A and B of problem 1.
int launch_pair(PairParams& prm, const CUtensorMap* maps /*[4]*/, cudaStream_t s) {
  prm.total_tiles = 0;
  for (int i = 0; i < prm.nprob; ++i) prm.total_tiles += prm.p[i].num_tiles;
  if (prm.total_tiles == 0) return LTVQKV_OK;
  static std::mutex mu;
  static int pairs_by_device[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ltvqkv_host::check_launch();
  int npairs;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (pairs_by_device[dev] == 0) {
      if (cudaFuncSetAttribute(gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPairSmemBytes) !=
          cudaSuccess)
        return ltvqkv_host::check_launch();
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * (ltvqkv_host::num_sms() / 2), 1, 1);
      cfg.blockDim = dim3(kPairThreads, 1, 1);
      cfg.dynamicSmemBytes = kPairSmemBytes;
      int nclusters = 0;
      if (cudaOccupancyMaxActiveClusters(&nclusters, gemm_pair_kernel, &cfg) != cudaSuccess || nclusters < 1) {
        cudaGetLastError();
        nclusters = ltvqkv_host::num_sms() / 2;
      }
      pairs_by_device[dev] = nclusters;
    }
    npairs = pairs_by_device[dev];
  }
  npairs = std::max(1, std::min(npairs, prm.total_tiles));
  gemm_pair_kernel<<<2 * npairs, kPairThreads, kPairSmemBytes, s>>>(maps[0], maps[1], maps[2], maps[3], prm);
  return ltvqkv_host::check_launch();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Opts `kernel` into `bytes` of dynamic shared memory on the current device (once per device).
int smem_opt_in(const void* kernel, size_t bytes) {
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ltvqkv_host::check_launch();
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({dev, kernel})) return LTVQKV_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
    return ltvqkv_host::check_launch();
  done.insert({dev, kernel});
  return LTVQKV_OK;
}

// Resident clusters of the fused projection + scan kernel on the current device (cached); 0 on a
// CUDA error.
int ps_clusters() {
  static std::mutex mu;
  static int by_device[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (by_device[dev] == 0) {
    if (cudaFuncSetAttribute(proj_scan_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPsSmemBytes) !=
        cudaSuccess)
      return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (ltvqkv_host::num_sms() / 2), 1, 1);
    cfg.blockDim = dim3(kPsThreads, 1, 1);
    cfg.dynamicSmemBytes = kPsSmemBytes;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, proj_scan_fwd_kernel, &cfg) != cudaSuccess || n < 1) {
      cudaGetLastError();
      n = ltvqkv_host::num_sms() / 2;
    }
    by_device[dev] = n;
  }
  return by_device[dev];
}

// The forward GEMM kernel on prepared maps (out rows = prm.F).
int launch_gemm_fwd(const CUtensorMap& tmW, const CUtensorMap& tmX, const CUtensorMap& tmOut, const FwdParams& prm,
                    cudaStream_t s) {
  const int rc = smem_opt_in((const void*)gemm_fwd_kernel, kFwdSmemBytes);
  if (rc != LTVQKV_OK) return rc;
  const int grid = std::min(prm.num_tiles, ltvqkv_host::num_sms());
  gemm_fwd_kernel<<<grid, kFwdThreads, kFwdSmemBytes, s>>>(tmW, tmX, tmOut, prm);
  return ltvqkv_host::check_launch();
}

template <typename Tin, typename Tout>
int launch_simt(const SimtArgs& a, int out_batches, cudaStream_t s) {
  if (a.M == 0 || a.N == 0 || out_batches == 0) return LTVQKV_OK;
  dim3 grid((a.N + 63) / 64, (a.M + 63) / 64, out_batches);
  gemm_simt_kernel<Tin, Tout><<<grid, 256, 0, s>>>(a);
  return ltvqkv_host::check_launch();
}

__global__ void zero_fill_kernel(void* p, long long nbytes) {
  long long i = (blockIdx.x * (long long)blockDim.x + threadIdx.x);
  if (i < nbytes) reinterpret_cast<unsigned char*>(p)[i] = 0;
}

}  // namespace

// Header, then the per-(output tile, CTA, warp) counters of the projection backward's two-split fp32
// dW (kOutColsF32Pair): enough for 2048 dW tiles of 256 x 256 (larger problems take one split).
constexpr size_t kGemmCombineWords = 2048 * 8;
extern "C" size_t ltvqkv_gemm_workspace_bytes(void) { return 256 + kGemmCombineWords * 4; }

extern "C" int ltvqkv_gemm_fwd(int dtype, const void* x, const void* weight, void* out, int B, int T, int K, int F,
                               void* workspace, size_t workspace_bytes, void* stream) {
  if (!ltvqkv_host::valid_dtype(dtype)) return LTVQKV_ERR_DTYPE;
  if (B < 0 || T < 0 || K < 0 || F < 0) return LTVQKV_ERR_SHAPE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if ((long long)B * T * F == 0) return LTVQKV_OK;
  if (!x || !weight || !out) return LTVQKV_ERR_INVALID_ARG;
  const bool bf16 = dtype == LTVQKV_DTYPE_BF16;
  const bool tc_ok = bf16 && K > 0 && K % 8 == 0 && T % 8 == 0 && aligned16(x) && aligned16(weight) && aligned16(out);
  if (!tc_ok) {
    SimtArgs a;
    a.A = weight; a.B = x; a.C = out;
    a.a_ob = 0; a.a_rb = 0; a.a_m = K; a.a_k = 1;
    a.b_ob = (long long)T * K; a.b_rb = 0; a.b_n = K; a.b_k = 1;
    a.c_ob = (long long)F * T; a.c_m = T; a.c_n = 1;
    a.M = F; a.N = T; a.K = K; a.red_batches = 1;
    return bf16 ? launch_simt<__nv_bfloat16, __nv_bfloat16>(a, B, s) : launch_simt<float, float>(a, B, s);
  }
  if (!workspace || workspace_bytes < ltvqkv_gemm_workspace_bytes()) return LTVQKV_ERR_WORKSPACE;
  FwdParams prm = {};
  prm.F = F; prm.T = T; prm.B = B;
  prm.m_tiles = (F + kFwdBM - 1) / kFwdBM;
  prm.n_tiles = (T + kFwdBN - 1) / kFwdBN;
  prm.k_blocks = (K + kFwdBK - 1) / kFwdBK;
  prm.num_tiles = B * prm.m_tiles * prm.n_tiles;
  prm.ws = reinterpret_cast<WorkspaceHeader*>(workspace);
  CUtensorMap tmW, tmX, tmOut;
  if (!make_map(&tmW, false, weight, K, F, 1, (uint64_t)K * 2, (uint64_t)K * F * 2, 64, kFwdBM) ||
      !make_map(&tmX, false, x, K, T, B, (uint64_t)K * 2, (uint64_t)K * T * 2, 64, kFwdBN) ||
      !make_map(&tmOut, false, out, T, F, B, (uint64_t)T * 2, (uint64_t)T * F * 2, 64, 32))
    return LTVQKV_ERR_LAUNCH;
  return launch_gemm_fwd(tmW, tmX, tmOut, prm, s);
}

namespace {
struct RopeTables {  // rotary tables of the fused forward's q / k prologue (cos == nullptr: none)
  const void* cos = nullptr;
  const void* sin = nullptr;
  int64_t cs = 0;
  float eps = 0.f;
};
int proj_scan_fwd_impl(int dtype, const void* x, const void* weight, const void* inits, int64_t inits_bs,
                       const float* logit_bias, void* combined, void* out_q, void* out_k, void* out_v, float* ckpt,
                       int B, int T, int C, int NH, int NKVH, int Da, int r, int use_sigmoid, void* workspace,
                       size_t workspace_bytes, void* stream, const RopeTables& rope = RopeTables());
}  // namespace

extern "C" int ltvqkv_proj_scan_fwd(int dtype, const void* x, const void* weight, const void* inits,
                                    const float* logit_bias, void* combined, void* out_q, void* out_k, void* out_v,
                                    int B, int T, int C, int NH, int NKVH, int Da, int r, int use_sigmoid,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  return proj_scan_fwd_impl(dtype, x, weight, inits, -1, logit_bias, combined, out_q, out_k, out_v, nullptr, B, T, C,
                            NH, NKVH, Da, r, use_sigmoid, workspace, workspace_bytes, stream);
}

extern "C" int ltvqkv_proj_scan_fwd_ckpt(int dtype, const void* x, const void* weight, const void* inits,
                                         int64_t inits_bs, const float* logit_bias, void* combined, void* out_q,
                                         void* out_k, void* out_v, float* ckpt, int B, int T, int C, int NH,
                                         int NKVH, int Da, int r, int use_sigmoid, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  if (!ckpt || (reinterpret_cast<uintptr_t>(ckpt) & 15u) != 0) return LTVQKV_ERR_INVALID_ARG;
  if (inits_bs != 0 && inits_bs != (int64_t)(NH + 2 * NKVH) * Da * r) return LTVQKV_ERR_STRIDE;
  return proj_scan_fwd_impl(dtype, x, weight, inits, inits_bs, logit_bias, combined, out_q, out_k, out_v, ckpt, B, T,
                            C, NH, NKVH, Da, r, use_sigmoid, workspace, workspace_bytes, stream);
}

extern "C" int ltvqkv_proj_scan_fwd_ckpt_rope(int dtype, const void* x, const void* weight, const void* inits,
                                              int64_t inits_bs, const float* logit_bias, void* combined, void* out_q,
                                              void* out_k, void* out_v, float* ckpt, const void* rope_cos,
                                              const void* rope_sin, int64_t rope_stride, float eps, int B, int T,
                                              int C, int NH, int NKVH, int Da, int r, int use_sigmoid,
                                              void* workspace, size_t workspace_bytes, void* stream) {
  if (!ckpt || (reinterpret_cast<uintptr_t>(ckpt) & 15u) != 0) return LTVQKV_ERR_INVALID_ARG;
  if (!rope_cos || !rope_sin) return LTVQKV_ERR_INVALID_ARG;
  // the epilogue reads each token's table row as 32 bf16 pairs
  if (rope_stride < Da * r / 2 || rope_stride % 2 != 0 || (reinterpret_cast<uintptr_t>(rope_cos) & 3u) != 0 ||
      (reinterpret_cast<uintptr_t>(rope_sin) & 3u) != 0)
    return LTVQKV_ERR_STRIDE;
  if (inits_bs != 0 && inits_bs != (int64_t)(NH + 2 * NKVH) * Da * r) return LTVQKV_ERR_STRIDE;
  RopeTables rope;
  rope.cos = rope_cos; rope.sin = rope_sin; rope.cs = rope_stride; rope.eps = eps;
  return proj_scan_fwd_impl(dtype, x, weight, inits, inits_bs, logit_bias, combined, out_q, out_k, out_v, ckpt, B, T,
                            C, NH, NKVH, Da, r, use_sigmoid, workspace, workspace_bytes, stream, rope);
}

namespace {
// inits_bs: elements between the sequences' initial states (0: one state for every sequence, fused
// kernel only; < 0: contiguous [B][H][D]).
int proj_scan_fwd_impl(int dtype, const void* x, const void* weight, const void* inits, int64_t inits_bs,
                       const float* logit_bias, void* combined, void* out_q, void* out_k, void* out_v, float* ckpt,
                       int B, int T, int C, int NH, int NKVH, int Da, int r, int use_sigmoid, void* workspace,
                       size_t workspace_bytes, void* stream, const RopeTables& rope) {
  if (!ltvqkv_host::valid_dtype(dtype)) return LTVQKV_ERR_DTYPE;
  if (B < 0 || T < 0 || C < 0 || NH < 0 || NKVH < 0 || Da < 1 || r < 1) return LTVQKV_ERR_SHAPE;
  const int H = NH + 2 * NKVH, D = Da * r, F = H * (D + Da);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // Fused when the scan operator would take its row-streaming kernel for these shapes (at least
  // two (batch, head) rows per SM), whose arithmetic the fused epilogue repeats step for step.
  const bool fused = dtype == LTVQKV_DTYPE_BF16 && D == kPsD && Da == 1 && H >= 1 && H <= kFwdBM && B > 0 &&
                     (long long)B * H >= 2LL * ltvqkv_host::num_sms() &&
                     T > 0 && T % 32 == 0 && C > 0 && C % 8 == 0 && x && weight && inits && logit_bias &&
                     combined && aligned16(x) && aligned16(weight) && aligned16(combined) &&
                     (NH == 0 || (out_q && aligned16(out_q))) &&
                     (NKVH == 0 || (out_k && out_v && aligned16(out_k) && aligned16(out_v)));
  // checkpoints and a shared initial state come from the fused kernel only
  if (!fused && (ckpt != nullptr || inits_bs == 0)) return LTVQKV_ERR_UNSUPPORTED;
  if (inits_bs < 0) inits_bs = (int64_t)H * D;
  if (!fused) {
    // the two operators in sequence: projection into `combined`, then the scan reading it
    int rc = ltvqkv_gemm_fwd(dtype, x, weight, combined, B, T, C, F, workspace, workspace_bytes, stream);
    if (rc != LTVQKV_OK) return rc;
    return ltvqkv_scan_fwd(dtype, combined, (int64_t)F * T, 1, T, inits, logit_bias, out_q, out_k, out_v, B, T, NH,
                           NKVH, Da, r, use_sigmoid, workspace, workspace_bytes, stream);
  }
  if (!workspace || workspace_bytes < ltvqkv_gemm_workspace_bytes()) return LTVQKV_ERR_WORKSPACE;
  WorkspaceHeader* ws = reinterpret_cast<WorkspaceHeader*>(workspace);
  const char* wb = reinterpret_cast<const char*>(weight);
  char* cb = reinterpret_cast<char*>(combined);
  // 1. the H decay-logit rows (row h*(D+1) + D of W and of `combined`) through the forward GEMM:
  //    strided 2-D views that skip the value rows; rows beyond H read zeros and are not stored
  FwdParams lp = {};
  lp.F = H; lp.T = T; lp.B = B;
  lp.m_tiles = 1;
  lp.n_tiles = (T + kFwdBN - 1) / kFwdBN;
  lp.k_blocks = (C + kFwdBK - 1) / kFwdBK;
  lp.num_tiles = B * lp.n_tiles;
  lp.ws = ws;
  CUtensorMap tmWl, tmX, tmOl;
  if (!make_map(&tmWl, false, wb + (size_t)D * C * 2, C, H, 1, (uint64_t)(D + 1) * C * 2, (uint64_t)F * C * 2, 64,
                kFwdBM) ||
      !make_map(&tmX, false, x, C, T, B, (uint64_t)C * 2, (uint64_t)C * T * 2, 64, kFwdBN) ||
      !make_map(&tmOl, false, cb + (size_t)D * T * 2, T, H, B, (uint64_t)(D + 1) * T * 2, (uint64_t)F * T * 2, 64,
                32))
    return LTVQKV_ERR_LAUNCH;
  int rc = launch_gemm_fwd(tmWl, tmX, tmOl, lp, s);
  if (rc != LTVQKV_OK) return rc;
  // 2. value rows and the scan, one head pair per ticket on a CTA pair
  PsParams pp = {};
  pp.B = B; pp.T = T; pp.H = H; pp.NH = NH; pp.NKVH = NKVH; pp.F = F;
  pp.n_tiles = (T + kPsBN - 1) / kPsBN;
  pp.k_blocks = lp.k_blocks;
  pp.npairs = B * ((H + 1) / 2);
  pp.use_sigmoid = use_sigmoid;
  pp.combined = reinterpret_cast<__nv_bfloat16*>(combined);
  pp.inits = reinterpret_cast<const __nv_bfloat16*>(inits);
  pp.logit_bias = logit_bias;
  pp.out[0] = reinterpret_cast<__nv_bfloat16*>(out_q);
  pp.out[1] = reinterpret_cast<__nv_bfloat16*>(out_k);
  pp.out[2] = reinterpret_cast<__nv_bfloat16*>(out_v);
  pp.ckpt = ckpt;
  pp.inits_bs = inits_bs;
  pp.rope_cos = reinterpret_cast<const __nv_bfloat16*>(rope.cos);
  pp.rope_sin = reinterpret_cast<const __nv_bfloat16*>(rope.sin);
  pp.rope_cs = rope.cs;
  pp.rope_eps = rope.eps;
  pp.ws = ws;
  CUtensorMap tmW, tmXh;
  if (!make_map(&tmW, false, weight, C, F, 1, (uint64_t)C * 2, (uint64_t)C * F * 2, 64, 128) ||
      !make_map(&tmXh, false, x, C, T, B, (uint64_t)C * 2, (uint64_t)C * T * 2, 64, kPsBN / 2))
    return LTVQKV_ERR_LAUNCH;
  const int nclusters = ps_clusters();
  if (nclusters < 1) return ltvqkv_host::check_launch();
  // two head pairs per cluster at a time
  const int grid = 2 * std::max(1, std::min(nclusters, (pp.npairs + 1) / 2));
  proj_scan_fwd_kernel<<<grid, kPsThreads, kPsSmemBytes, s>>>(tmW, tmXh, pp);
  return ltvqkv_host::check_launch();
}
}  // namespace

extern "C" int ltvqkv_gemm_bwd(int dtype, const void* x, const void* weight, const void* grad_out, int64_t go_b,
                               int64_t go_f, int64_t go_t, void* grad_x, void* grad_weight, int grad_weight_dtype,
                               int B, int T, int K, int F, void* workspace, size_t workspace_bytes, void* stream) {
  if (!ltvqkv_host::valid_dtype(dtype) || !ltvqkv_host::valid_dtype(grad_weight_dtype)) return LTVQKV_ERR_DTYPE;
  if (B < 0 || T < 0 || K < 0 || F < 0) return LTVQKV_ERR_SHAPE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool bf16 = dtype == LTVQKV_DTYPE_BF16;
  const bool gw_f32 = grad_weight_dtype == LTVQKV_DTYPE_F32;
  const bool go_contig = (go_t == 1 && go_f == T);
  const bool go_trans = (go_f == 1 && go_t == F);
  if (!(go_contig || go_trans) || go_b != (int64_t)F * T) return LTVQKV_ERR_STRIDE;
  // Degenerate sizes: outputs of zero extent, or an empty reduction (zero-filled).
  if ((long long)B * T * K > 0 && F == 0) {
    long long n = (long long)B * T * K * (bf16 ? 2 : 4);
    zero_fill_kernel<<<(unsigned int)((n + 255) / 256), 256, 0, s>>>(grad_x, n);
  }
  if ((long long)F * K > 0 && (long long)B * T == 0) {
    long long n = (long long)F * K * (gw_f32 ? 4 : 2);
    zero_fill_kernel<<<(unsigned int)((n + 255) / 256), 256, 0, s>>>(grad_weight, n);
  }
  if ((long long)B * T * F * K == 0) return ltvqkv_host::check_launch();
  if (!x || !weight || !grad_out || !grad_x || !grad_weight) return LTVQKV_ERR_INVALID_ARG;

  // TMA needs 16-byte row pitches: K for x / W / dx / dW, and the unit-stride extent of grad_out.
  const bool tc_ok = bf16 && K % 8 == 0 && (go_contig ? T % 8 == 0 : F % 8 == 0) && aligned16(x) &&
                     aligned16(weight) && aligned16(grad_out) && aligned16(grad_x) && aligned16(grad_weight);
  if (!tc_ok) {
    // dx[b][t][k] = sum_f g[b][f][t] W[f][k]: A = g (m=t, k=f), B = W (n=k, k=f)
    SimtArgs a;
    a.A = grad_out; a.B = weight; a.C = grad_x;
    a.a_ob = go_b; a.a_rb = 0; a.a_m = go_t; a.a_k = go_f;
    a.b_ob = 0; a.b_rb = 0; a.b_n = 1; a.b_k = K;
    a.c_ob = (long long)T * K; a.c_m = K; a.c_n = 1;
    a.M = T; a.N = K; a.K = F; a.red_batches = 1;
    int rc = bf16 ? launch_simt<__nv_bfloat16, __nv_bfloat16>(a, B, s) : launch_simt<float, float>(a, B, s);
    if (rc != LTVQKV_OK) return rc;
    // dW[f][k] = sum_b sum_t g[b][f][t] x[b][t][k]: A = g (m=f, k=t), B = x (n=k, k=t), reduce over b
    SimtArgs w;
    w.A = grad_out; w.B = x; w.C = grad_weight;
    w.a_ob = 0; w.a_rb = go_b; w.a_m = go_f; w.a_k = go_t;
    w.b_ob = 0; w.b_rb = (long long)T * K; w.b_n = 1; w.b_k = K;
    w.c_ob = 0; w.c_m = K; w.c_n = 1;
    w.M = F; w.N = K; w.K = T; w.red_batches = B;
    if (bf16)
      return gw_f32 ? launch_simt<__nv_bfloat16, float>(w, 1, s) : launch_simt<__nv_bfloat16, __nv_bfloat16>(w, 1, s);
    return gw_f32 ? launch_simt<float, float>(w, 1, s) : launch_simt<float, __nv_bfloat16>(w, 1, s);
  }
  if (!workspace || workspace_bytes < ltvqkv_gemm_workspace_bytes()) return LTVQKV_ERR_WORKSPACE;

  PairParams prm = {};
  prm.nprob = 2;
  prm.ws = reinterpret_cast<WorkspaceHeader*>(workspace);
  CUtensorMap maps[4];
  // Problem 0: dW tiles. M = k (lanes), N = f, reduction over the B batches x T tokens; fp32 dW
  // takes the batches in two halves (two tiles per output tile, so the long dW tiles balance the dx
  // tiles across the clusters), combined by the epilogues: the first half to finish stores, the
  // second adds (no zero fill, no floating-point atomics).
  PairProblem& w = prm.p[0];
  const long long dw_tiles = (long long)((K + 255) / 256) * ((F + kPairBN - 1) / kPairBN);
  const int splits = (gw_f32 && B % 2 == 0 && dw_tiles * 8 <= (long long)kGemmCombineWords) ? 2 : 1;
  w.M = K; w.N = F; w.out_batches = 1; w.splits = splits; w.red_batches = B / splits;
  w.a_mn = 1; w.b_mn = go_contig ? 0 : 1; w.a_bmode = 2; w.b_bmode = 2;
  w.out_mode = splits == 2 ? kOutColsF32Pair : (gw_f32 ? kOutColsF32 : kOutColsBf16);
  w.out = grad_weight; w.out_ld = K; w.out_bs = 0;  // dW [F][K]
  w.combine = reinterpret_cast<unsigned int*>(reinterpret_cast<char*>(workspace) + 256);
  finalize_pair(w, T);
  // Problem 1: dx tiles. M = t (lanes), N = k, reduction over F.
  PairProblem& d = prm.p[1];
  d.M = T; d.N = K; d.out_batches = B; d.splits = 1; d.red_batches = 1;
  d.a_mn = go_contig ? 1 : 0; d.b_mn = 1; d.a_bmode = 1; d.b_bmode = 0; d.out_mode = kOutRows;
  d.out = grad_x; d.out_ld = K; d.out_bs = (long long)T * K;  // dx [B][T][K]
  finalize_pair(d, F);
  bool ok = true;
  // MN-major operands whose contiguous extent is a multiple of 64 load as one 4-D box per stage
  w.a_blk = K % 64 == 0;
  w.b_blk = !go_contig && F % 64 == 0;
  d.a_blk = go_contig && T % 64 == 0;
  d.b_blk = K % 64 == 0;
  // x as [B][T][K]: MN-major A operand of dW (m = k, k = t).
  ok = ok && (w.a_blk ? make_mn_blk_map(&maps[0], x, K, T, B, (uint64_t)K * 2, (uint64_t)T * K * 2)
                      : make_map(&maps[0], false, x, K, T, B, (uint64_t)K * 2, (uint64_t)T * K * 2, 64, 64));
  if (go_contig) {
    // g as [B][F][T]: K-major B of dW (n = f, k = t), MN-major A of dx (m = t, k = f).
    ok = ok && make_map(&maps[1], false, grad_out, T, F, B, (uint64_t)T * 2, (uint64_t)go_b * 2, 64, 128);
    ok = ok && (d.a_blk ? make_mn_blk_map(&maps[2], grad_out, T, F, B, (uint64_t)T * 2, (uint64_t)go_b * 2)
                        : make_map(&maps[2], false, grad_out, T, F, B, (uint64_t)T * 2, (uint64_t)go_b * 2, 64, 64));
  } else {
    // g as [B][T][F]: MN-major B of dW (n = f, k = t), K-major A of dx (m = t, k = f).
    ok = ok && (w.b_blk ? make_mn_blk_map(&maps[1], grad_out, F, T, B, (uint64_t)F * 2, (uint64_t)go_b * 2)
                        : make_map(&maps[1], false, grad_out, F, T, B, (uint64_t)F * 2, (uint64_t)go_b * 2, 64, 64));
    ok = ok && make_map(&maps[2], false, grad_out, F, T, B, (uint64_t)F * 2, (uint64_t)go_b * 2, 64, 128);
  }
  // W as [F][K]: MN-major B operand of dx (n = k, k = f).
  ok = ok && (d.b_blk ? make_mn_blk_map(&maps[3], weight, K, F, 1, (uint64_t)K * 2, (uint64_t)K * F * 2)
                      : make_map(&maps[3], false, weight, K, F, 1, (uint64_t)K * 2, (uint64_t)K * F * 2, 64, 64));
  if (!ok) return LTVQKV_ERR_LAUNCH;
  return launch_pair(prm, maps, s);
}
