// Projection GEMMs of the filtered-QKV layer on sm_100a tensor cores.
//
//   forward  (reference cpp_ewma/src/fused_linear_transpose_forward.cu:23-58):
//     out[b, f, t] = sum_k W[f, k] x[b, t, k]
//   backward (reference cpp_ewma/src/fused_linear_transpose_backward.cu:22-132, which issues
//   2*B serial cuBLAS calls): in ONE launch
//     dx[b, t, k] = sum_f g[b, f, t] W[f, k]          (dx tiles)
//     dW[f, k]    = sum_b sum_t g[b, f, t] x[b, t, k] (dW tiles, reduction over all B*T tokens
//                                                      inside one CTA's TMEM accumulator)
//
// Kernel structure (one CTA per SM, persistent, 192 threads):
//   warp 0      TMA producer: draws tile tickets, loads A/B k-blocks (64 bf16 = 128 B wide,
//               128B swizzle) into a 4-stage smem ring (mbarrier full/empty pairs).
//   warp 1      allocates 512 TMEM columns; one lane issues tcgen05.mma (M=128, N=bn, K=16,
//               bf16 x bf16 -> fp32) into one of two TMEM accumulators and commits stages.
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, convert, stage into a swizzled
//               4 KB smem buffer (double-buffered per warp) and TMA-store to global.
// A tile is described by two operand "problems" so the dx and dW GEMMs share one launch; the
// long dW tiles are drawn first and the short dx tiles fill the remaining SMs.
// Every mbarrier wait is bounded (2 s); a timeout records LTVQKV_ERR_TIMEOUT in the workspace
// and all roles leave their loops, then TMEM is freed.
#include <algorithm>

#include "ltvqkv_common.cuh"

namespace ltvqkv {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr int kAStageBytes = kBM * kBK * 2;           // 16 KB
constexpr int kBStageBytesMax = 256 * kBK * 2;        // 32 KB
constexpr int kStageBytes = kAStageBytes + kBStageBytesMax;
constexpr int kEpiWarps = 4;
constexpr int kEpiBufBytes = 32 * 128;                // 32 rows x 128 B
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;     // 192
constexpr int kTmemCols = 512;
constexpr int kAccStride = 256;                       // TMEM columns between the two accumulators
constexpr int kSchedDepth = 2;
constexpr size_t kGemmSmemBytes =
    1024 /*alignment slack*/ + (size_t)kStages * kStageBytes + (size_t)kEpiWarps * 2 * kEpiBufBytes + 256;

struct GemmProblem {
  int M, N;           // output extents (rows: TMEM lanes; cols: contiguous in the output)
  int out_batches;    // independent output slices (third TMA coordinate of D)
  int red_batches;    // reduction batches, outer K loop
  int K;              // reduction extent per batch
  int bn;             // N tile: 128 or 256
  int a_mn, b_mn;     // 1 = operand stored MN-major (M/N contiguous), 0 = K-major
  int a_bmode, b_bmode;  // third TMA coordinate: 0 none, 1 output batch, 2 reduction batch
  int out_f32;        // output element type
  int m_tiles, n_tiles, k_blocks, num_tiles;
};

struct GemmParams {
  GemmProblem p[2];
  int nprob;
  int total_tiles;
  WorkspaceHeader* ws;
};

struct TileCoord {
  int prob, ob, m0, n0;
};

LTVQKV_DEVICE TileCoord decode_tile(const GemmParams& prm, int tile) {
  TileCoord tc;
  int local = tile;
  tc.prob = 0;
  if (prm.nprob > 1 && local >= prm.p[0].num_tiles) {
    local -= prm.p[0].num_tiles;
    tc.prob = 1;
  }
  const GemmProblem& P = prm.p[tc.prob];
  // Row tiles fastest when the B operand is the large streamed one (forward: all row tiles of
  // one x block run together); column tiles fastest otherwise (dx: one g block feeds all
  // column tiles).
  int mt, nt;
  if (P.n_tiles <= P.m_tiles && P.a_bmode == 0) {
    mt = local % P.m_tiles;
    int rest = local / P.m_tiles;
    nt = rest % P.n_tiles;
    tc.ob = rest / P.n_tiles;
  } else {
    nt = local % P.n_tiles;
    int rest = local / P.n_tiles;
    mt = rest % P.m_tiles;
    tc.ob = rest / P.m_tiles;
  }
  tc.m0 = mt * kBM;
  tc.n0 = nt * P.bn;
  return tc;
}

LTVQKV_DEVICE int batch_coord(int mode, int ob, int rb) { return mode == 1 ? ob : (mode == 2 ? rb : 0); }

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmB0,
                   const __grid_constant__ CUtensorMap tmD0, const __grid_constant__ CUtensorMap tmA1,
                   const __grid_constant__ CUtensorMap tmB1, const __grid_constant__ CUtensorMap tmD1,
                   const GemmParams prm) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* stages = smem;
  unsigned char* epi = stages + kStages * kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi + kEpiWarps * 2 * kEpiBufBytes);
  uint64_t* full_bar = bars;                       // [kStages]
  uint64_t* empty_bar = full_bar + kStages;        // [kStages]
  uint64_t* tfull_bar = empty_bar + kStages;       // [2]
  uint64_t* tempty_bar = tfull_bar + 2;            // [2]
  uint64_t* sfull_bar = tempty_bar + 2;            // [kSchedDepth]
  uint64_t* sempty_bar = sfull_bar + kSchedDepth;  // [kSchedDepth]
  int* sched_tile = reinterpret_cast<int*>(sempty_bar + kSchedDepth);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sched_tile + kSchedDepth);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  WorkspaceHeader* ws = prm.ws;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], kEpiWarps);
    }
    for (int i = 0; i < kSchedDepth; ++i) {
      mbar_init(&sfull_bar[i], 1);
      mbar_init(&sempty_bar[i], 1 + kEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA0); tma_prefetch_desc(&tmB0); tma_prefetch_desc(&tmD0);
    if (prm.nprob > 1) { tma_prefetch_desc(&tmA1); tma_prefetch_desc(&tmB1); tma_prefetch_desc(&tmD1); }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- scheduler + TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int i = 0;; ++i) {
        const int slot = i % kSchedDepth;
        const uint32_t sph = (uint32_t)(i / kSchedDepth) & 1u;
        if (!mbar_wait(&sempty_bar[slot], sph ^ 1u, abort_flag, ws, 0x6001)) break;
        int tile = (int)draw_ticket(ws);
        if (tile >= prm.total_tiles) tile = -1;
        sched_tile[slot] = tile;
        mbar_arrive(&sfull_bar[slot]);
        if (tile < 0) break;
        const TileCoord tc = decode_tile(prm, tile);
        const GemmProblem& P = prm.p[tc.prob];
        const CUtensorMap* mA = tc.prob ? &tmA1 : &tmA0;
        const CUtensorMap* mB = tc.prob ? &tmB1 : &tmB0;
        const uint32_t bytes = (uint32_t)(kAStageBytes + P.bn * kBK * 2);
        bool ok = true;
        for (int rb = 0; rb < P.red_batches && ok; ++rb) {
          const int ca = batch_coord(P.a_bmode, tc.ob, rb);
          const int cbz = batch_coord(P.b_bmode, tc.ob, rb);
          for (int kb = 0; kb < P.k_blocks; ++kb) {
            if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, ws, 0x6002)) { ok = false; break; }
            unsigned char* sA = stages + stage * kStageBytes;
            unsigned char* sB = sA + kAStageBytes;
            mbar_arrive_expect_tx(&full_bar[stage], bytes);
            const int k0 = kb * kBK;
            if (P.a_mn) {
              tma_load_3d(sA, mA, &full_bar[stage], tc.m0, k0, ca);
              tma_load_3d(sA + 8192, mA, &full_bar[stage], tc.m0 + 64, k0, ca);
            } else {
              tma_load_3d(sA, mA, &full_bar[stage], k0, tc.m0, ca);
            }
            if (P.b_mn) {
              for (int i2 = 0; i2 < P.bn / 64; ++i2)
                tma_load_3d(sB + i2 * 8192, mB, &full_bar[stage], tc.n0 + 64 * i2, k0, cbz);
            } else {
              tma_load_3d(sB, mB, &full_bar[stage], k0, tc.n0, cbz);
            }
            if (++stage == kStages) { stage = 0; phase ^= 1u; }
          }
        }
        if (!ok) break;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int i = 0;; ++i) {
        const int slot = i % kSchedDepth;
        const uint32_t sph = (uint32_t)(i / kSchedDepth) & 1u;
        if (!mbar_wait(&sfull_bar[slot], sph, abort_flag, ws, 0x6101)) break;
        const int tile = sched_tile[slot];
        mbar_arrive(&sempty_bar[slot]);
        if (tile < 0) break;
        const TileCoord tc = decode_tile(prm, tile);
        const GemmProblem& P = prm.p[tc.prob];
        const uint32_t idesc = umma_idesc_bf16(kBM, P.bn, P.a_mn, P.b_mn);
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, ws, 0x6102)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * kAccStride);
        const int total_kb = P.red_batches * P.k_blocks;
        bool ok = true;
        for (int it = 0; it < total_kb; ++it) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, ws, 0x6103)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stages + stage * kStageBytes);
          const uint32_t b_addr = a_addr + kAStageBytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t adesc = P.a_mn ? umma_desc_sw128(a_addr + kk * 2048, 8192, 1024)
                                          : umma_desc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bdesc = P.b_mn ? umma_desc_sw128(b_addr + kk * 2048, 8192, 1024)
                                          : umma_desc_sw128(b_addr + kk * 32, 16, 1024);
            umma_bf16(d_tmem, adesc, bdesc, idesc, (it > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue warps ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    unsigned char* buf0 = epi + (warp - 2) * 2 * kEpiBufBytes;
    int acc = 0;
    uint32_t acc_phase = 0;
    int nbuf = 0;
    for (int i = 0;; ++i) {
      const int slot = i % kSchedDepth;
      const uint32_t sph = (uint32_t)(i / kSchedDepth) & 1u;
      bool ok = mbar_wait(&sfull_bar[slot], sph, abort_flag, ws, 0x6201);
      if (!ok) break;
      const int tile = sched_tile[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty_bar[slot]);
      if (tile < 0) break;
      const TileCoord tc = decode_tile(prm, tile);
      const GemmProblem& P = prm.p[tc.prob];
      const CUtensorMap* mD = tc.prob ? &tmD1 : &tmD0;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, ws, 0x6202)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * kAccStride);
      const int row0 = tc.m0 + q * 32;
      const int cols_per_chunk = P.out_f32 ? 32 : 64;
      // Row slabs entirely beyond M hold nothing to store (and issue no bulk store, which keeps
      // the two staging buffers strictly alternating between committed groups).
      const int nchunks = row0 < P.M ? P.bn / cols_per_chunk : 0;
      for (int ch = 0; ch < nchunks; ++ch) {
        unsigned char* buf = buf0 + nbuf * kEpiBufBytes;
        // Make sure the bulk store that last read this buffer has finished reading it.
        if (lane == 0) tma_store_wait_read1();
        __syncwarp();
        unsigned char* rowp = buf + lane * 128;
        if (P.out_f32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_row + (uint32_t)(ch * 32), v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 w = make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            *reinterpret_cast<uint4*>(rowp + ((j ^ (lane & 7)) * 16)) = w;
          }
        } else {
          uint32_t v0[32], v1[32];
          tmem_ld_32x32b_x32(t_row + (uint32_t)(ch * 64), v0);
          tmem_ld_32x32b_x32(t_row + (uint32_t)(ch * 64 + 32), v1);
          tmem_wait_ld();
          uint32_t pk[32];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            __nv_bfloat162 p2 = __floats2bfloat162_rn(__uint_as_float(v0[2 * j]), __uint_as_float(v0[2 * j + 1]));
            pk[j] = *reinterpret_cast<uint32_t*>(&p2);
            __nv_bfloat162 p3 = __floats2bfloat162_rn(__uint_as_float(v1[2 * j]), __uint_as_float(v1[2 * j + 1]));
            pk[16 + j] = *reinterpret_cast<uint32_t*>(&p3);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 w = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
            *reinterpret_cast<uint4*>(rowp + ((j ^ (lane & 7)) * 16)) = w;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(mD, buf, tc.n0 + ch * cols_per_chunk, row0, tc.ob);
          tma_store_commit();
        }
        nbuf ^= 1;
      }
      // All TMEM reads of this accumulator are complete (tcgen05.wait::ld above).
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
    if (lane == 0) tma_store_wait0();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
  if (threadIdx.x == 0) finish_launch(ws, gridDim.x);
}

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

// 3-D tiled map: dims (d0 innermost, d1, d2), byte strides of d1 and d2, box (box0, box1, 1).
bool make_map(CUtensorMap* m, bool f32, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
              uint64_t s2, uint32_t box0, uint32_t box1) {
  const uint64_t dims[3] = {d0, d1, d2};
  const uint64_t strides[2] = {s1, s2};
  const uint32_t box[3] = {box0, box1, 1};
  return ltvqkv_host::encode_tiled_map(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                                       base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

void finalize_problem(GemmProblem& p) {
  p.m_tiles = (p.M + kBM - 1) / kBM;
  p.n_tiles = (p.N + p.bn - 1) / p.bn;
  p.k_blocks = (p.K + kBK - 1) / kBK;
  p.num_tiles = p.out_batches * p.m_tiles * p.n_tiles;
}

int launch_tc(GemmParams& prm, const CUtensorMap* maps /*[6]*/, cudaStream_t s) {
  prm.total_tiles = 0;
  for (int i = 0; i < prm.nprob; ++i) prm.total_tiles += prm.p[i].num_tiles;
  if (prm.total_tiles == 0) return LTVQKV_OK;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmemBytes);
    attr_set = true;
  }
  int grid = std::min(prm.total_tiles, ltvqkv_host::num_sms());
  gemm_tc_kernel<<<grid, kGemmThreads, kGemmSmemBytes, s>>>(maps[0], maps[1], maps[2], maps[3], maps[4], maps[5],
                                                          prm);
  return ltvqkv_host::check_launch();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

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

extern "C" size_t ltvqkv_gemm_workspace_bytes(void) { return 256; }

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
  GemmParams prm = {};
  prm.nprob = 1;
  prm.ws = reinterpret_cast<WorkspaceHeader*>(workspace);
  GemmProblem& p = prm.p[0];
  p.M = F; p.N = T; p.out_batches = B; p.red_batches = 1; p.K = K; p.bn = 256;
  p.a_mn = 0; p.b_mn = 0; p.a_bmode = 0; p.b_bmode = 1; p.out_f32 = 0;
  finalize_problem(p);
  CUtensorMap maps[6];
  bool ok = make_map(&maps[0], false, weight, K, F, 1, (uint64_t)K * 2, (uint64_t)K * F * 2, 64, 128) &&
            make_map(&maps[1], false, x, K, T, B, (uint64_t)K * 2, (uint64_t)K * T * 2, 64, 256) &&
            make_map(&maps[2], false, out, T, F, B, (uint64_t)T * 2, (uint64_t)T * F * 2, 64, 32);
  if (!ok) return LTVQKV_ERR_LAUNCH;
  maps[3] = maps[0]; maps[4] = maps[1]; maps[5] = maps[2];
  return launch_tc(prm, maps, s);
}

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

  GemmParams prm = {};
  prm.nprob = 2;
  prm.ws = reinterpret_cast<WorkspaceHeader*>(workspace);
  CUtensorMap maps[6];
  // Problem 0: dW tiles (M = F rows, N = K columns, reduction over B batches x T tokens).
  GemmProblem& w = prm.p[0];
  w.M = F; w.N = K; w.out_batches = 1; w.red_batches = B; w.K = T; w.bn = 128;
  w.a_bmode = 2; w.b_bmode = 2; w.b_mn = 1; w.out_f32 = gw_f32 ? 1 : 0;
  // Problem 1: dx tiles (M = T tokens per batch, N = K columns, reduction over F).
  GemmProblem& d = prm.p[1];
  d.M = T; d.N = K; d.out_batches = B; d.red_batches = 1; d.K = F; d.bn = 256;
  d.a_bmode = 1; d.b_bmode = 0; d.b_mn = 1; d.out_f32 = 0;
  bool ok = true;
  if (go_contig) {
    // g as [B][F][T]: K-major for dW (k = t), MN-major for dx (m = t).
    w.a_mn = 0;
    ok = ok && make_map(&maps[0], false, grad_out, T, F, B, (uint64_t)T * 2, (uint64_t)go_b * 2, 64, 128);
    d.a_mn = 1;
    ok = ok && make_map(&maps[3], false, grad_out, T, F, B, (uint64_t)T * 2, (uint64_t)go_b * 2, 64, 64);
  } else {
    // g as [B][T][F]: MN-major for dW (m = f), K-major for dx (k = f).
    w.a_mn = 1;
    ok = ok && make_map(&maps[0], false, grad_out, F, T, B, (uint64_t)F * 2, (uint64_t)go_b * 2, 64, 64);
    d.a_mn = 0;
    ok = ok && make_map(&maps[3], false, grad_out, F, T, B, (uint64_t)F * 2, (uint64_t)go_b * 2, 64, 128);
  }
  // x as [B][T][K]: MN-major B operand of dW (n = k, k = t).
  ok = ok && make_map(&maps[1], false, x, K, T, B, (uint64_t)K * 2, (uint64_t)T * K * 2, 64, 64);
  // dW output [F][K].
  ok = ok && (gw_f32 ? make_map(&maps[2], true, grad_weight, K, F, 1, (uint64_t)K * 4, (uint64_t)K * F * 4, 32, 32)
                     : make_map(&maps[2], false, grad_weight, K, F, 1, (uint64_t)K * 2, (uint64_t)K * F * 2, 64, 32));
  // W as [F][K]: MN-major B operand of dx (n = k, k = f).
  ok = ok && make_map(&maps[4], false, weight, K, F, 1, (uint64_t)K * 2, (uint64_t)K * F * 2, 64, 64);
  // dx output [B][T][K].
  ok = ok && make_map(&maps[5], false, grad_x, K, T, B, (uint64_t)K * 2, (uint64_t)T * K * 2, 64, 32);
  if (!ok) return LTVQKV_ERR_LAUNCH;
  finalize_problem(w);
  finalize_problem(d);
  return launch_tc(prm, maps, s);
}
