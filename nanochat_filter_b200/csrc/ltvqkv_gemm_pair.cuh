// Projection GEMMs on CTA pairs (included by ltvqkv_gemm.cu).
//
// A cluster of two CTAs on two SMs computes one 256 x bn output tile with tcgen05.mma
// cta_group::2 (M = 256: 128 rows in each CTA's TMEM; the B tile split by N between the two
// CTAs' shared memory), so each SM streams half of A and half of B per k-block: 32 KB per
// 2 * 256 * 256 * 64 FLOP, 1.5x the arithmetic intensity of a single-CTA 128 x 256 tile.
//
// Roles (256 threads per CTA, persistent, one cluster per SM pair; every role that waits in a loop
// has a warp of its own, so no waiting lane holds up a sibling of its warp):
//   warp 0      the leader's lane 0: tile scheduler (draws a ticket, forwards it to the peer's ring
//               through distributed shared memory).
//   warps 1..2  lane 0 of each, both CTAs: TMA producers, each loading every other stage of the
//               ring (this CTA's halves of A and B, one 16 KB box each; completion is counted on
//               the leader's full barrier, which the leader's producer arms with both CTAs'
//               bytes). One thread issues about one bulk-tensor copy per few hundred cycles, short
//               of the 64 B/clock per SM a 256 x 256 pair tile consumes; two issuing threads
//               measured 10% faster at the config-2 backward than one (three or four: no better).
//   warp 3      TMEM allocation (cta_group::2, both CTAs); the leader's lane 0 issues the MMAs and
//               commits (multicast to both CTAs) the stage-empty and accumulator-full barriers.
//   warps 4..7  epilogue of each CTA over its 128 TMEM lanes: tcgen05.ld, convert, and store
//               straight from registers (16-byte row pieces, or one coalesced 128-byte row of the
//               output per TMEM column); then report the accumulator free to the leader. No
//               shared-memory staging: all of it goes to a 7-stage operand ring.
// A reduction split in two tiles (the fp32 dW of the backward, batches in two halves) is combined
// without floating-point atomics or a zero fill: per output tile and epilogue warp, the split that
// finishes first stores its partial sums, the second adds its own to them (two addends, so the
// result does not depend on which finished first).
// Tiles of up to two problems share one launch; problem 0 is drawn first (the long dW tiles of
// the backward). Every wait is bounded (2 s); a timeout records LTVQKV_ERR_TIMEOUT and all roles
// leave their loops.
#pragma once

namespace ltvqkv {

constexpr int kPairStages = 7;
constexpr int kPairBK = 64;
constexpr int kPairBN = 256;
constexpr int kPairAHalf = 128 * kPairBK * 2;                 // 16 KB: this CTA's 128 rows of A
constexpr int kPairBHalf = (kPairBN / 2) * kPairBK * 2;       // 16 KB: this CTA's half of B
constexpr int kPairStageBytes = kPairAHalf + kPairBHalf;
constexpr int kPairProducers = 2;                        // producer warps (lane 0 of each)
constexpr int kPairProdWarp = 1;                         // warp 0 schedules
constexpr int kPairMmaWarp = kPairProdWarp + kPairProducers;
constexpr int kPairEpiWarp = kPairMmaWarp + 1;           // four epilogue warps
constexpr int kPairThreads = 32 * (kPairEpiWarp + 4);
constexpr int kPairSchedDepth = 2;
// readers of a scheduler slot: the producers of both CTAs, the leader's MMA lane, 4 epilogue warps per CTA
constexpr int kPairSchedReaders = 2 * kPairProducers + 1 + 8;
constexpr size_t kPairSmemBytes = 1024 + (size_t)kPairStages * kPairStageBytes + 256;

// Epilogue forms (output element (row, col) at out[ob * out_bs + row * out_ld + col]).
//   kOutRows:      TMEM lane = output row (m), TMEM column = col (n); bf16
//   kOutColsBf16:  TMEM lane = col (m), TMEM column = output row (n); bf16
//   kOutColsF32:   as kOutColsBf16, fp32
//   kOutColsF32Pair: as kOutColsF32 for a reduction split in two tiles: the first of the two to
//                   finish stores, the second adds (per 32-lane warp slice, through `combine`)
enum PairOut { kOutRows = 0, kOutColsBf16 = 1, kOutColsF32 = 2, kOutColsF32Pair = 3 };

struct PairProblem {
  int M, N;              // tile space: M rows (TMEM lanes), N columns
  int out_batches;       // independent output slices (third TMA coordinate of the output)
  int splits;            // reduction batches are split into this many tiles (results added)
  int red_batches;       // reduction batches per split
  int k_blocks;          // 64-wide k-blocks per reduction batch
  int a_mn, b_mn;        // operand stored MN-major (1) or K-major (0)
  int a_blk, b_blk;      // MN-major operand loaded as one 4-D box {64, 64, 2, 1} (extent a multiple of 64)
  int a_bmode, b_bmode;  // third operand coordinate: 0 none, 1 output batch, 2 reduction batch
  int out_mode;          // PairOut
  int m_tiles, n_tiles, num_tiles;
  void* out;
  long long out_ld, out_bs;  // elements
  unsigned int* combine;     // kOutColsF32Pair: [m_tiles * n_tiles][2 CTAs][4 warps] counters, zero at launch
};

struct PairParams {
  PairProblem p[2];
  int nprob;
  int total_tiles;
  WorkspaceHeader* ws;
};

struct PairTile {
  int prob, ob, split, m0, n0, bn;
};

LTVQKV_DEVICE PairTile pair_decode(const PairParams& prm, int tile) {
  PairTile t;
  int local = tile;
  t.prob = 0;
  if (prm.nprob > 1 && local >= prm.p[0].num_tiles) {
    local -= prm.p[0].num_tiles;
    t.prob = 1;
  }
  const PairProblem& P = prm.p[t.prob];
  // column tiles fastest: consecutive tiles reuse the same A rows from L2
  const int nt = local % P.n_tiles;
  int rest = local / P.n_tiles;
  const int mt = rest % P.m_tiles;
  rest /= P.m_tiles;
  t.split = rest % P.splits;
  t.ob = rest / P.splits;
  t.m0 = mt * 256;
  t.n0 = nt * kPairBN;
  const int left = P.N - t.n0;
  // narrow last column tile: a multiple of 16 (K-major B), or of 128 (MN-major B, so that each
  // CTA's half is whole 64-column swizzle atoms)
  const int step = P.b_mn ? 128 : 16;
  t.bn = left >= kPairBN ? kPairBN : ((left + step - 1) / step) * step;
  return t;
}

LTVQKV_DEVICE int pair_bcoord(int mode, int ob, int rb) { return mode == 1 ? ob : (mode == 2 ? rb : 0); }

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmB0,
                     const __grid_constant__ CUtensorMap tmA1, const __grid_constant__ CUtensorMap tmB1,
                     const __grid_constant__ PairParams prm) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = smem_align<unsigned char>(smem_raw, 1024);
  unsigned char* stages = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(stages + kPairStages * kPairStageBytes);
  uint64_t* full_bar = bars;                           // [kPairStages] (leader's counts the pair's bytes)
  uint64_t* empty_bar = full_bar + kPairStages;        // [kPairStages]
  uint64_t* tfull_bar = empty_bar + kPairStages;       // [2]
  uint64_t* tempty_bar = tfull_bar + 2;                // [2] (leader: 4 local + 4 peer epilogue warps)
  uint64_t* sfull_bar = tempty_bar + 2;                // [kPairSchedDepth]
  uint64_t* sempty_bar = sfull_bar + kPairSchedDepth;  // [kPairSchedDepth] (leader: every reader of both CTAs)
  int* sched_tile = reinterpret_cast<int*>(sempty_bar + kPairSchedDepth);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sched_tile + kPairSchedDepth);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  WorkspaceHeader* ws = prm.ws;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], 8);
    }
    for (int i = 0; i < kPairSchedDepth; ++i) {
      mbar_init(&sfull_bar[i], 1);
      mbar_init(&sempty_bar[i], kPairSchedReaders);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA0); tma_prefetch_desc(&tmB0);
    if (prm.nprob > 1) { tma_prefetch_desc(&tmA1); tma_prefetch_desc(&tmB1); }
  }
  if (warp == kPairMmaWarp) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Sched ring readers: wait on the local full barrier, then release the slot on the leader.
  auto sched_take = [&](int i, int& tile, unsigned int where) -> bool {
    const int slot = i % kPairSchedDepth;
    const uint32_t sph = (uint32_t)(i / kPairSchedDepth) & 1u;
    if (!mbar_wait_cluster(&sfull_bar[slot], sph, abort_flag, ws, where)) return false;
    tile = sched_tile[slot];
    return true;
  };
  auto sched_release = [&](int i) {
    const int slot = i % kPairSchedDepth;
    if (leader) mbar_arrive(&sempty_bar[slot]);
    else mbar_arrive_cluster(mapa_shared(&sempty_bar[slot], 0));
  };

  // Epilogue of one split of a two-split reduction (kOutColsF32Pair). Per (output tile, CTA, warp)
  // counter: the claim (+1) orders the two splits; the first stores its partials and then publishes
  // (+1 after a fence); the second waits until it sees all three increments and adds its partials to
  // the stored ones. The first never waits, so a wait always ends once the (already running) first
  // split's cluster finishes its epilogue. The CTA that finishes the launch last zeroes the counters
  // for the next launch on the workspace.
  auto pair_epilogue = [&](const PairProblem& P, const PairTile& tc, uint32_t t_row, int m) -> bool {
    const int ncols = min(tc.bn, P.N - tc.n0);
    const bool in_m = m < P.M;
    unsigned int* ctr = P.combine + (((tc.m0 / 256) * P.n_tiles + tc.n0 / kPairBN) * 2 + (int)rank) * 4 + (warp & 3);
    unsigned int claim = 0;
    if (lane == 0) claim = atomicAdd(ctr, 1u);
    claim = __shfl_sync(0xffffffffu, claim, 0);
    float* o = reinterpret_cast<float*>(P.out) + (long long)tc.n0 * P.out_ld + m;
    if (claim == 0) {
      for (int ch = 0; ch * 32 < ncols; ++ch) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_row + (uint32_t)(ch * 32), v);
        tmem_wait_ld();
        const int nj = min(32, ncols - ch * 32);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (in_m && j < nj) __stcg(o + (long long)(ch * 32 + j) * P.out_ld, __uint_as_float(v[j]));
      }
      __threadfence();
      __syncwarp();
      if (lane == 0) atomicAdd(ctr, 1u);
      return true;
    }
    bool ok = true;
    if (lane == 0 && claim != 2u) {
      const unsigned long long t0 = global_timer_ns();
      while (ld_acquire_u32(ctr) != 3u) {
        if (*abort_flag || global_timer_ns() - t0 > kWaitLimitNs) {
          record_timeout(ws, 0x6703);
          *abort_flag = 1;
          ok = false;
          break;
        }
        __nanosleep(64);
      }
    }
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    if (!ok) return false;
    (void)ld_acquire_u32(ctr);  // every lane: the first split's stores happen-before its reads below
    for (int ch = 0; ch * 32 < ncols; ++ch) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_row + (uint32_t)(ch * 32), v);
      tmem_wait_ld();
      const int nj = min(32, ncols - ch * 32);
      float* oc = o + (long long)(ch * 32) * P.out_ld;
      float prev[32];  // every load issued before any store: one L2 round trip per chunk
#pragma unroll
      for (int j = 0; j < 32; ++j) prev[j] = (in_m && j < nj) ? __ldcg(oc + (long long)j * P.out_ld) : 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (in_m && j < nj) oc[(long long)j * P.out_ld] = prev[j] + __uint_as_float(v[j]);
    }
    return true;
  };

  if (warp == 0) {
    if (leader && lane == 0) {
      // ---------------- scheduler (leader): tickets into the ring of both CTAs ----------------
      for (int i = 0;; ++i) {
        const int slot = i % kPairSchedDepth;
        const uint32_t sph = (uint32_t)(i / kPairSchedDepth) & 1u;
        if (!mbar_wait(&sempty_bar[slot], sph ^ 1u, abort_flag, ws, 0x6501)) break;
        int tile = (int)draw_ticket(ws);
        if (tile >= prm.total_tiles) tile = -1;
        sched_tile[slot] = tile;
        st_cluster_u32(mapa_shared(&sched_tile[slot], 1), (uint32_t)tile);
        mbar_arrive(&sfull_bar[slot]);
        mbar_arrive_cluster(mapa_shared(&sfull_bar[slot], 1));
        if (tile < 0) break;
      }
    }
    __syncwarp();
  } else if (warp < kPairMmaWarp) {
    if (lane == 0) {
      // ---------------- TMA producers (both CTAs): stage g is loaded by producer g % kPairProducers ----------------
      const int pw = warp - kPairProdWarp;
      const uint32_t full_leader0 = mapa_shared(&full_bar[0], 0);
      int g = 0;  // stages of every tile so far (the same count in every producer lane)
      for (int i = 0;; ++i) {
        int tile;
        if (!sched_take(i, tile, 0x6502)) break;
        sched_release(i);
        if (tile < 0) break;
        const PairTile tc = pair_decode(prm, tile);
        const PairProblem& P = prm.p[tc.prob];
        const CUtensorMap* mA = tc.prob ? &tmA1 : &tmA0;
        const CUtensorMap* mB = tc.prob ? &tmB1 : &tmB0;
        const int am = tc.m0 + (int)rank * 128;         // this CTA's A rows
        const int bnh = tc.bn / 2;
        const int bn0 = tc.n0 + (int)rank * bnh;        // this CTA's B rows (N half)
        const int rb0 = tc.split * P.red_batches;
        const int nst = P.red_batches * P.k_blocks;
        bool ok = true;
        // this producer's first stage of the tile, then every kPairProducers-th
        for (int j = (pw - g % kPairProducers + kPairProducers) % kPairProducers; j < nst; j += kPairProducers) {
          const int gs = g + j;
          const int stage = gs % kPairStages;
          const uint32_t phase = (uint32_t)(gs / kPairStages) & 1u;
          const int rb = rb0 + j / P.k_blocks, kb = j % P.k_blocks;
          const int ca = pair_bcoord(P.a_bmode, tc.ob, rb);
          const int cbz = pair_bcoord(P.b_bmode, tc.ob, rb);
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, ws, 0x6503)) { ok = false; break; }
          unsigned char* sA = stages + stage * kPairStageBytes;
          unsigned char* sB = sA + kPairAHalf;
          const uint32_t fb = full_leader0 + (uint32_t)(stage * 8);
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], (uint32_t)(2 * kPairStageBytes));
          const int k0 = kb * kPairBK;
          if (!P.a_mn) {
            tma_load_3d_pair(sA, mA, fb, k0, am, ca);
          } else if (P.a_blk) {
            tma_load_4d_pair(sA, mA, fb, 0, k0, am / 64, ca);
          } else {
            tma_load_3d_pair(sA, mA, fb, am, k0, ca);
            tma_load_3d_pair(sA + 8192, mA, fb, am + 64, k0, ca);
          }
          if (!P.b_mn) {
            tma_load_3d_pair(sB, mB, fb, k0, bn0, cbz);
          } else if (P.b_blk) {
            tma_load_4d_pair(sB, mB, fb, 0, k0, bn0 / 64, cbz);
          } else {
            tma_load_3d_pair(sB, mB, fb, bn0, k0, cbz);
            tma_load_3d_pair(sB + 8192, mB, fb, bn0 + 64, k0, cbz);
          }
        }
        if (!ok) break;
        g += nst;
      }
    }
    __syncwarp();
  } else if (warp == kPairMmaWarp) {
    // ---------------- MMA issuer (leader) ----------------
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int i = 0;; ++i) {
        int tile;
        if (!sched_take(i, tile, 0x6601)) break;
        sched_release(i);
        if (tile < 0) break;
        const PairTile tc = pair_decode(prm, tile);
        const PairProblem& P = prm.p[tc.prob];
        const uint32_t idesc = umma_idesc_bf16(256, tc.bn, P.a_mn, P.b_mn);
        if (!mbar_wait_cluster(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, ws, 0x6602)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * kPairBN);
        const int total_kb = P.red_batches * P.k_blocks;
        bool ok = true;
        for (int it = 0; it < total_kb; ++it) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, ws, 0x6603)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stages + stage * kPairStageBytes);
          const uint32_t b_addr = a_addr + kPairAHalf;
#pragma unroll
          for (int kk = 0; kk < kPairBK / 16; ++kk) {
            const uint64_t adesc = P.a_mn ? umma_desc_sw128(a_addr + kk * 2048, 8192, 1024)
                                          : umma_desc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bdesc = P.b_mn ? umma_desc_sw128(b_addr + kk * 2048, 8192, 1024)
                                          : umma_desc_sw128(b_addr + kk * 32, 16, 1024);
            umma_bf16_pair(d_tmem, adesc, bdesc, idesc, (it > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit_pair(&empty_bar[stage], 0x3);
          if (++stage == kPairStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit_pair(&tfull_bar[acc], 0x3);
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue warps ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t tempty_leader0 = mapa_shared(&tempty_bar[0], 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int i = 0;; ++i) {
      int tile = -1;
      bool ok = true;
      if (lane == 0) ok = sched_take(i, tile, 0x6701);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      tile = __shfl_sync(0xffffffffu, tile, 0);
      if (!ok) break;
      if (lane == 0) sched_release(i);
      if (tile < 0) break;
      const PairTile tc = pair_decode(prm, tile);
      const PairProblem& P = prm.p[tc.prob];
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, ws, 0x6702)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * kPairBN);
      const int m = tc.m0 + (int)rank * 128 + q * 32 + lane;  // this thread's TMEM lane (tile row)
      const int ncols = min(tc.bn, P.N - tc.n0);               // valid columns of the tile
      if (P.out_mode == kOutColsF32Pair) {
        if (!pair_epilogue(P, tc, t_row, m)) break;
      } else if (P.out_mode == kOutRows) {
        // this thread writes row m: 64 columns (128 bytes) per chunk as eight 16-byte stores
        __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(P.out) + (long long)tc.ob * P.out_bs +
                              (long long)m * P.out_ld + tc.n0;
        for (int ch = 0; ch * 64 < ncols; ++ch) {
          uint32_t v0[32], v1[32];
          tmem_ld_32x32b_x32(t_row + (uint32_t)(ch * 64), v0);
          tmem_ld_32x32b_x32(t_row + (uint32_t)(ch * 64 + 32), v1);
          tmem_wait_ld();
          if (m < P.M) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint32_t* src = j < 4 ? v0 + 8 * j : v1 + 8 * (j - 4);
              uint4 w;
              __nv_bfloat162 p0 = __floats2bfloat162_rn(__uint_as_float(src[0]), __uint_as_float(src[1]));
              __nv_bfloat162 p1 = __floats2bfloat162_rn(__uint_as_float(src[2]), __uint_as_float(src[3]));
              __nv_bfloat162 p2 = __floats2bfloat162_rn(__uint_as_float(src[4]), __uint_as_float(src[5]));
              __nv_bfloat162 p3 = __floats2bfloat162_rn(__uint_as_float(src[6]), __uint_as_float(src[7]));
              w.x = *reinterpret_cast<uint32_t*>(&p0); w.y = *reinterpret_cast<uint32_t*>(&p1);
              w.z = *reinterpret_cast<uint32_t*>(&p2); w.w = *reinterpret_cast<uint32_t*>(&p3);
              if (ch * 64 + 8 * j < ncols) *reinterpret_cast<uint4*>(orow + ch * 64 + 8 * j) = w;
            }
          }
        }
      } else {
        // TMEM column j is output row n0 + j; the warp's 32 lanes write 32 consecutive elements of it
        const bool in_m = m < P.M;
        for (int ch = 0; ch * 32 < ncols; ++ch) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_row + (uint32_t)(ch * 32), v);
          tmem_wait_ld();
          const long long base = (long long)tc.ob * P.out_bs + (long long)(tc.n0 + ch * 32) * P.out_ld + m;
          const int nj = min(32, ncols - ch * 32);
          if (P.out_mode == kOutColsBf16) {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(P.out) + base;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (in_m && j < nj) o[(long long)j * P.out_ld] = __float2bfloat16_rn(__uint_as_float(v[j]));
          } else {
            float* o = reinterpret_cast<float*>(P.out) + base;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (in_m && j < nj) o[(long long)j * P.out_ld] = __uint_as_float(v[j]);
          }
        }
      }
      // all TMEM reads of this accumulator are complete (tcgen05.wait::ld above)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(&tempty_bar[acc]);
        else mbar_arrive_cluster_relaxed(tempty_leader0 + (uint32_t)(acc * 8));
      }
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
  }

  tc_fence_before();
  cluster_sync_all();  // no CTA of the pair touches the other's memory or TMEM after this
  tc_fence_after();
  if (warp == kPairMmaWarp) tmem_dealloc_pair(tmem_base, 512);
  const PairProblem& P0 = prm.p[0];
  if (P0.out_mode != kOutColsF32Pair) {
    if (threadIdx.x == 0) finish_launch(ws, gridDim.x);
    return;
  }
  __shared__ int last_cta;
  if (threadIdx.x == 0) last_cta = finish_launch_last(ws, gridDim.x) ? 1 : 0;
  __syncthreads();
  if (last_cta) {
    const int n = P0.m_tiles * P0.n_tiles * 8;
    for (int i = threadIdx.x; i < n; i += blockDim.x) P0.combine[i] = 0u;
  }
}

}  // namespace ltvqkv
