// Forward projection on single CTAs (included by ltvqkv_gemm.cu):
//   out[b, f, t] = sum_k W[f, k] x[b, t, k]
// tiles of 128 head channels (A = W, K-major) x 256 tokens (B = x, K-major), K = model dim.
//
// Measured on B200 at the config-2 shape against the CTA-pair kernel of the backward: with K as
// short as 768 a tile is 12 k-blocks, and the pair kernel's operand feed (both CTAs' halves must
// land before the leader may issue) left its tensor pipe waiting; one CTA per SM with a 48 KB
// k-block keeps more bytes per SM in flight and finishes the forward ~15% sooner.
//
// Kernel structure (one CTA per SM, persistent, 192 threads):
//   warp 0      TMA producer: draws tile tickets, loads A/B k-blocks (64 bf16 = 128 B wide,
//               128B swizzle) into a 4-stage smem ring (mbarrier full/empty pairs).
//   warp 1      allocates 512 TMEM columns; one lane issues tcgen05.mma (M=128, N=256, K=16,
//               bf16 x bf16 -> fp32) into one of two TMEM accumulators and commits stages.
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 64 columns, convert to bf16, stage into a
//               swizzled 4 KB smem buffer (double-buffered per warp) and TMA-store to global.
// Tiles run channel-tile fastest, so the 19 channel tiles that read one x block do so together
// and the block is read from DRAM once. Every mbarrier wait is bounded (2 s); a timeout records
// LTVQKV_ERR_TIMEOUT in the workspace and all roles leave their loops, then TMEM is freed.
#pragma once

namespace ltvqkv {

constexpr int kFwdBM = 128;
constexpr int kFwdBN = 256;
constexpr int kFwdBK = 64;
constexpr int kFwdStages = 4;
constexpr int kFwdAStageBytes = kFwdBM * kFwdBK * 2;  // 16 KB
constexpr int kFwdStageBytes = kFwdAStageBytes + kFwdBN * kFwdBK * 2;  // + 32 KB
constexpr int kFwdEpiBufBytes = 32 * 128;             // 32 rows x 128 B
constexpr int kFwdThreads = 192;
constexpr int kFwdSchedDepth = 2;
constexpr size_t kFwdSmemBytes = 1024 + (size_t)kFwdStages * kFwdStageBytes + 4 * 2 * (size_t)kFwdEpiBufBytes + 256;

struct FwdParams {
  int F, T, B;                         // output [B][F][T]
  int m_tiles, n_tiles, k_blocks, num_tiles;
  WorkspaceHeader* ws;
};

__global__ void __launch_bounds__(kFwdThreads, 1)
    gemm_fwd_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                    const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ FwdParams prm) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = smem_align<unsigned char>(smem_raw, 1024);
  unsigned char* stages = smem;
  unsigned char* epi = stages + kFwdStages * kFwdStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi + 4 * 2 * kFwdEpiBufBytes);
  uint64_t* full_bar = bars;                          // [kFwdStages]
  uint64_t* empty_bar = full_bar + kFwdStages;        // [kFwdStages]
  uint64_t* tfull_bar = empty_bar + kFwdStages;       // [2]
  uint64_t* tempty_bar = tfull_bar + 2;               // [2]
  uint64_t* sfull_bar = tempty_bar + 2;               // [kFwdSchedDepth]
  uint64_t* sempty_bar = sfull_bar + kFwdSchedDepth;  // [kFwdSchedDepth]
  int* sched_tile = reinterpret_cast<int*>(sempty_bar + kFwdSchedDepth);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sched_tile + kFwdSchedDepth);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  WorkspaceHeader* ws = prm.ws;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFwdStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], 4);
    }
    for (int i = 0; i < kFwdSchedDepth; ++i) {
      mbar_init(&sfull_bar[i], 1);
      mbar_init(&sempty_bar[i], 1 + 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW); tma_prefetch_desc(&tmX); tma_prefetch_desc(&tmOut);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // tile -> (batch, channel tile, token tile), channel tiles fastest
  auto decode = [&](int tile, int& b, int& m0, int& n0) {
    const int mt = tile % prm.m_tiles;
    const int rest = tile / prm.m_tiles;
    n0 = (rest % prm.n_tiles) * kFwdBN;
    b = rest / prm.n_tiles;
    m0 = mt * kFwdBM;
  };

  if (warp == 0) {
    // ---------------- scheduler + TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int i = 0;; ++i) {
        const int slot = i % kFwdSchedDepth;
        const uint32_t sph = (uint32_t)(i / kFwdSchedDepth) & 1u;
        if (!mbar_wait(&sempty_bar[slot], sph ^ 1u, abort_flag, ws, 0x6001)) break;
        int tile = (int)draw_ticket(ws);
        if (tile >= prm.num_tiles) tile = -1;
        sched_tile[slot] = tile;
        mbar_arrive(&sfull_bar[slot]);
        if (tile < 0) break;
        int b, m0, n0;
        decode(tile, b, m0, n0);
        bool ok = true;
        for (int kb = 0; kb < prm.k_blocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, ws, 0x6002)) { ok = false; break; }
          unsigned char* sA = stages + stage * kFwdStageBytes;
          mbar_arrive_expect_tx(&full_bar[stage], (uint32_t)kFwdStageBytes);
          tma_load_3d(sA, &tmW, &full_bar[stage], kb * kFwdBK, m0, 0);
          tma_load_3d(sA + kFwdAStageBytes, &tmX, &full_bar[stage], kb * kFwdBK, n0, b);
          if (++stage == kFwdStages) { stage = 0; phase ^= 1u; }
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
      const uint32_t idesc = umma_idesc_bf16(kFwdBM, kFwdBN, 0, 0);
      for (int i = 0;; ++i) {
        const int slot = i % kFwdSchedDepth;
        const uint32_t sph = (uint32_t)(i / kFwdSchedDepth) & 1u;
        if (!mbar_wait(&sfull_bar[slot], sph, abort_flag, ws, 0x6101)) break;
        const int tile = sched_tile[slot];
        mbar_arrive(&sempty_bar[slot]);
        if (tile < 0) break;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, ws, 0x6102)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * kFwdBN);
        bool ok = true;
        for (int kb = 0; kb < prm.k_blocks; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, ws, 0x6103)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stages + stage * kFwdStageBytes);
          const uint32_t b_addr = a_addr + kFwdAStageBytes;
#pragma unroll
          for (int kk = 0; kk < kFwdBK / 16; ++kk) {
            umma_bf16(d_tmem, umma_desc_sw128(a_addr + kk * 32, 16, 1024), umma_desc_sw128(b_addr + kk * 32, 16, 1024),
                      idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == kFwdStages) { stage = 0; phase ^= 1u; }
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
    unsigned char* buf0 = epi + (warp - 2) * 2 * kFwdEpiBufBytes;
    int acc = 0;
    uint32_t acc_phase = 0;
    int nbuf = 0;
    for (int i = 0;; ++i) {
      const int slot = i % kFwdSchedDepth;
      const uint32_t sph = (uint32_t)(i / kFwdSchedDepth) & 1u;
      if (!mbar_wait(&sfull_bar[slot], sph, abort_flag, ws, 0x6201)) break;
      const int tile = sched_tile[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty_bar[slot]);
      if (tile < 0) break;
      int b, m0, n0;
      decode(tile, b, m0, n0);
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, ws, 0x6202)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * kFwdBN);
      const int row0 = m0 + q * 32;
      // row slabs entirely beyond F hold nothing to store (and issue no bulk store, which keeps
      // the two staging buffers strictly alternating between committed groups)
      const int nchunks = row0 < prm.F ? kFwdBN / 64 : 0;
      for (int ch = 0; ch < nchunks; ++ch) {
        unsigned char* buf = buf0 + nbuf * kFwdEpiBufBytes;
        // the bulk store that last read this buffer must have finished reading it
        if (lane == 0) tma_store_wait_read1();
        __syncwarp();
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
        unsigned char* rowp = buf + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint4 w = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
          *reinterpret_cast<uint4*>(rowp + ((j ^ (lane & 7)) * 16)) = w;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(&tmOut, buf, n0 + ch * 64, row0, b);
          tma_store_commit();
        }
        nbuf ^= 1;
      }
      // all TMEM reads of this accumulator are complete (tcgen05.wait::ld above)
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
  if (warp == 1) tmem_dealloc(tmem_base, 512);
  if (threadIdx.x == 0) finish_launch(ws, gridDim.x);
}

}  // namespace ltvqkv
