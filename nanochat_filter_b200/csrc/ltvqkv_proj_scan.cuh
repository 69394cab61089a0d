// Fused projection + scan forward (included by ltvqkv_gemm.cu), for head dim 128 with one decay
// group per head (Da = 1):
//   combined[b, h*129 + c, t] = sum_k W[h*129 + c, k] x[b, t, k]        (value rows, c < 128)
//   h_t = (1 - a_t) h_{t-1} + a_t u_t,  a_t = sigmoid(combined[b, h*129 + 128, t] + bias[h])
//
// Work unit: a head pair (heads 2j, 2j+1 of one batch; ticket counter) on a cluster of two CTAs.
// The tensor cores compute both heads' value rows with one tcgen05.mma cta_group::2 per k step
// (M = 256: head 2j's 128 rows in CTA 0's TMEM, head 2j+1's in CTA 1's; the 256-token x tile
// split by N between the two CTAs' shared memory), so each SM streams 16 KB of W and 16 KB of x
// per 64-wide k-block. A cluster holds two head pairs at a time (two tickets, "slots"), walks
// their 256-token tiles in time order and alternates between them: the tensor cores fill one
// slot's accumulator (256 TMEM columns each) while an epilogue warpgroup reads the other's. In a
// warpgroup each warp owns 32 channels (its TMEM lane quarter): a thread reads its channel's
// accumulator, rounds u to bf16 (the stored projection value the reference's scan reads),
// writes it to `combined` and continues the recurrence in a register across tiles, so the scan
// never re-reads `combined` from HBM. The decay-logit rows come from a pre-pass (the forward
// GEMM kernel on the H logit rows) and are read back from L2, one tile ahead. Results equal the
// unfused ltvqkv_gemm_fwd + row-streaming ltvqkv_scan_fwd bit for bit (same MMA order, same
// rounding steps).
//
// Roles (320 threads per CTA, persistent, one cluster per SM pair):
//   warp 0      scheduler (leader: draws two tickets per round and forwards them to the peer's
//               ring through distributed shared memory) and TMA producer (both CTAs: W rows of
//               the CTA's head and its half of the x tile into a 6-stage ring; completion counted
//               on the leader's full barrier, armed with both CTAs' bytes).
//   warp 1      TMEM allocation (cta_group::2); the leader's lane 0 issues the MMAs and commits
//               (multicast to both CTAs) the stage-empty and accumulator-full barriers.
//   warps 2..5  epilogue of slot 0, warps 6..9 of slot 1 (this CTA's head of the slot's pair):
//               `combined` rows through a per-warp 2 KB transpose (64-byte row pieces per store),
//               q/k/v straight from the walk (a warp stores 64 contiguous bytes per token); then
//               report the accumulator free to the leader.
// Every wait is bounded (2 s); a timeout records LTVQKV_ERR_TIMEOUT and all roles leave.
#pragma once

namespace ltvqkv {

constexpr int kPsStages = 6;
constexpr int kPsBN = 256;                         // tokens per tile
constexpr int kPsD = 128;                          // head dim = threads of an epilogue warpgroup
constexpr int kPsBK = 64;
constexpr int kPsThreads = 64 + 2 * kPsD;          // producer, MMA, two epilogue warpgroups
constexpr int kPsWHalf = 128 * kPsBK * 2;          // 16 KB: the CTA's head's 128 W rows
constexpr int kPsXHalf = (kPsBN / 2) * kPsBK * 2;  // 16 KB: the CTA's 128 tokens of x
constexpr int kPsStageBytes = kPsWHalf + kPsXHalf;
constexpr int kPsXposeBytes = 32 * 64;             // one warp's 32 channels x 32 tokens, bf16
constexpr int kPsSchedDepth = 2;
constexpr int kPsEpiWarps = 8;
constexpr size_t kPsSmemBytes = 1024 + (size_t)kPsStages * kPsStageBytes + kPsEpiWarps * (size_t)kPsXposeBytes +
                                kPsEpiWarps * (size_t)kPsBN * 8 + 256;

struct PsParams {
  int B, T, H, NH, NKVH, F;  // F = H * 129
  int n_tiles, k_blocks;
  int npairs;                // B * ceil(H / 2)
  int use_sigmoid;
  __nv_bfloat16* combined;        // [B][F][T]: logit rows written by the pre-pass, value rows here
  const __nv_bfloat16* inits;     // [B][H][128], sequences inits_bs elements apart (0: shared)
  long long inits_bs;
  const float* logit_bias;        // [H]
  __nv_bfloat16* out[3];          // [B][heads][T][128]
  float* ckpt;                    // optional [B][H][T / 32][128]: the fp32 state after every 32nd token
  // optional rotary tables [T][64] (rows rope_cs elements apart): q and k then leave rotated and
  // RMS-normalised (the reference attention's prologue, nanochat/gpt.py:224-230) instead of raw
  const __nv_bfloat16* rope_cos;
  const __nv_bfloat16* rope_sin;
  long long rope_cs;
  float rope_eps;
  WorkspaceHeader* ws;
};

// Eight decay logits (tokens t0 .. t0+7 of one logit row), 16-byte aligned; zeros beyond T.
LTVQKV_DEVICE uint4 ps_load_logits(const __nv_bfloat16* lrow, int t0, int T) {
  if (t0 >= T) return make_uint4(0, 0, 0, 0);
  return __ldg(reinterpret_cast<const uint4*>(lrow + t0));
}

// Rotary table pairs (2 lane, 2 lane + 1) of tokens t0 .. t0 + 7.
LTVQKV_DEVICE void ps_rope_rows(const PsParams& prm, int t0, int lane, uint32_t (&c)[8], uint32_t (&s)[8]) {
#pragma unroll
  for (int tt = 0; tt < 8; ++tt) {
    const long long ti = (long long)(t0 + tt) * prm.rope_cs;
    c[tt] = __ldg(reinterpret_cast<const uint32_t*>(prm.rope_cos + ti) + lane);
    s[tt] = __ldg(reinterpret_cast<const uint32_t*>(prm.rope_sin + ti) + lane);
  }
}

// Head pair p -> batch and first head (the second, h0 + 1, exists when h0 + 1 < H).
LTVQKV_DEVICE void ps_pair(int p, int H, int& b, int& h0) {
  const int hp = (H + 1) / 2;
  b = p / hp;
  h0 = 2 * (p % hp);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPsThreads, 1)
    proj_scan_fwd_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                         const __grid_constant__ PsParams prm) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = smem_align<unsigned char>(smem_raw, 1024);
  unsigned char* stages = smem;
  unsigned char* xpose = stages + kPsStages * kPsStageBytes;                       // [8 warps][32][64 B]
  float2* gates = reinterpret_cast<float2*>(xpose + kPsEpiWarps * kPsXposeBytes);  // [8 warps][256]
  uint64_t* bars = reinterpret_cast<uint64_t*>(gates + kPsEpiWarps * kPsBN);
  uint64_t* full_bar = bars;                          // [kPsStages] (leader's counts the pair's bytes)
  uint64_t* empty_bar = full_bar + kPsStages;         // [kPsStages]
  uint64_t* tfull_bar = empty_bar + kPsStages;        // [2]: slot accumulator ready
  uint64_t* tempty_bar = tfull_bar + 2;               // [2]: slot accumulator read (leader: 4 + 4 warps)
  uint64_t* sfull_bar = tempty_bar + 2;               // [kPsSchedDepth]
  uint64_t* sempty_bar = sfull_bar + kPsSchedDepth;   // [kPsSchedDepth] (leader: 9 local + 9 peer readers)
  int* sched = reinterpret_cast<int*>(sempty_bar + kPsSchedDepth);  // [kPsSchedDepth][2] tickets
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sched + 2 * kPsSchedDepth);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  WorkspaceHeader* ws = prm.ws;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPsStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], 8);
    }
    for (int i = 0; i < kPsSchedDepth; ++i) {
      mbar_init(&sfull_bar[i], 1);
      mbar_init(&sempty_bar[i], 2 * (1 + kPsEpiWarps));
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW); tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Sched ring readers: wait on the local full barrier, read the round's two tickets, release
  // the slot on the leader.
  auto sched_take = [&](int i, int& t0, int& t1, unsigned int where) -> bool {
    const int slot = i % kPsSchedDepth;
    const uint32_t sph = (uint32_t)(i / kPsSchedDepth) & 1u;
    if (!mbar_wait_cluster(&sfull_bar[slot], sph, abort_flag, ws, where)) return false;
    t0 = sched[2 * slot];
    t1 = sched[2 * slot + 1];
    return true;
  };
  auto sched_release = [&](int i) {
    const int slot = i % kPsSchedDepth;
    if (leader) mbar_arrive(&sempty_bar[slot]);
    else mbar_arrive_cluster(mapa_shared(&sempty_bar[slot], 0));
  };

  if (warp == 0) {
    // ---------------- scheduler (leader) + TMA producer (both) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const uint32_t full_leader0 = mapa_shared(&full_bar[0], 0);
      for (int i = 0;; ++i) {
        int tk[2];
        if (leader) {
          const int slot = i % kPsSchedDepth;
          const uint32_t sph = (uint32_t)(i / kPsSchedDepth) & 1u;
          if (!mbar_wait(&sempty_bar[slot], sph ^ 1u, abort_flag, ws, 0x6801)) break;
          tk[0] = (int)draw_ticket(ws);
          tk[1] = tk[0] < prm.npairs ? (int)draw_ticket(ws) : prm.npairs;
          if (tk[0] >= prm.npairs) tk[0] = -1;  // end
          if (tk[1] >= prm.npairs) tk[1] = -2;  // slot 1 idle this round
          sched[2 * slot] = tk[0];
          sched[2 * slot + 1] = tk[1];
          st_cluster_u32(mapa_shared(&sched[2 * slot], 1), (uint32_t)tk[0]);
          st_cluster_u32(mapa_shared(&sched[2 * slot + 1], 1), (uint32_t)tk[1]);
          mbar_arrive(&sfull_bar[slot]);
          mbar_arrive_cluster(mapa_shared(&sfull_bar[slot], 1));
        } else {
          if (!sched_take(i, tk[0], tk[1], 0x6802)) break;
          sched_release(i);
        }
        if (tk[0] < 0) break;
        const int nslots = tk[1] >= 0 ? 2 : 1;
        // this CTA's head of each slot's pair (rows beyond F read zeros for an odd H)
        int b0, h0, b1 = 0, h1 = 0;
        ps_pair(tk[0], prm.H, b0, h0);
        if (nslots > 1) ps_pair(tk[1], prm.H, b1, h1);
        h0 += (int)rank;
        h1 += (int)rank;
        bool ok = true;
        for (int nt = 0; nt < prm.n_tiles && ok; ++nt) {
          for (int sl = 0; sl < nslots && ok; ++sl) {
            const int bsl = sl ? b1 : b0, hsl = sl ? h1 : h0;
            for (int kb = 0; kb < prm.k_blocks; ++kb) {
              if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, ws, 0x6803)) { ok = false; break; }
              unsigned char* sW = stages + stage * kPsStageBytes;
              const uint32_t fb = full_leader0 + (uint32_t)(stage * 8);
              if (leader) mbar_arrive_expect_tx(&full_bar[stage], (uint32_t)(2 * kPsStageBytes));
              tma_load_3d_pair(sW, &tmW, fb, kb * kPsBK, hsl * (kPsD + 1), 0);
              tma_load_3d_pair(sW + kPsWHalf, &tmX, fb, kb * kPsBK, nt * kPsBN + (int)rank * (kPsBN / 2), bsl);
              if (++stage == kPsStages) { stage = 0; phase ^= 1u; }
            }
          }
        }
        if (!ok) break;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader) ----------------
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_phase[2] = {0, 0};
      const uint32_t idesc = umma_idesc_bf16(256, kPsBN, 0, 0);
      bool ok = true;
      for (int i = 0; ok; ++i) {
        int tk[2];
        if (!sched_take(i, tk[0], tk[1], 0x6901)) break;
        sched_release(i);
        if (tk[0] < 0) break;
        const int nslots = tk[1] >= 0 ? 2 : 1;
        for (int nt = 0; nt < prm.n_tiles && ok; ++nt) {
          for (int sl = 0; sl < nslots && ok; ++sl) {
            if (!mbar_wait_cluster(&tempty_bar[sl], acc_phase[sl] ^ 1u, abort_flag, ws, 0x6902)) { ok = false; break; }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + (uint32_t)(sl * kPsBN);
            for (int kb = 0; kb < prm.k_blocks; ++kb) {
              if (!mbar_wait(&full_bar[stage], phase, abort_flag, ws, 0x6903)) { ok = false; break; }
              tc_fence_after();
              const uint32_t a_addr = smem_u32(stages + stage * kPsStageBytes);
              const uint32_t b_addr = a_addr + kPsWHalf;
#pragma unroll
              for (int kk = 0; kk < kPsBK / 16; ++kk) {
                umma_bf16_pair(d_tmem, umma_desc_sw128(a_addr + kk * 32, 16, 1024),
                               umma_desc_sw128(b_addr + kk * 32, 16, 1024), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
              }
              umma_commit_pair(&empty_bar[stage], 0x3);
              if (++stage == kPsStages) { stage = 0; phase ^= 1u; }
            }
            if (!ok) break;
            umma_commit_pair(&tfull_bar[sl], 0x3);
            acc_phase[sl] ^= 1u;
          }
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: warpgroup sl = slot sl; warp = 32 channels of this CTA's head ----------------
    const int ew = warp - 2;           // 0..7
    const int sl = ew / 4;             // slot
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int c = q * 32 + lane;       // channel = TMEM lane
    unsigned char* xp = xpose + ew * kPsXposeBytes;
    float2* gw = gates + ew * kPsBN;
    const uint32_t tempty_leader = mapa_shared(&tempty_bar[sl], 0);
    uint32_t acc_phase = 0;
    // Rotary + norm: the warpgroup's four transpose buffers (8 KB, contiguous) hold a [32 token][128
    // channel] bf16 tile of the walk's outputs between two barriers of the group (named barrier 1 +
    // slot, 128 threads); each warp then finishes 8 of its tokens, lane l holding the channel pairs
    // (2l, 2l + 1) and (2l + 64, 2l + 65), i.e. the rotation's pairs. The group leaves its loops
    // together: the outcome of every bounded wait is OR-reduced over the group at a barrier, so no
    // warp can wait at a group barrier for a warp that has left.
    unsigned char* stg = xpose + (size_t)sl * 4 * kPsXposeBytes;
    const int gbar = 1 + sl;
    for (int i = 0;; ++i) {
      int tk[2] = {-1, -1};
      bool got = true;
      if (lane == 0) got = sched_take(i, tk[0], tk[1], 0x6a01);
      got = !named_barrier_or(gbar, 128, __shfl_sync(0xffffffffu, got ? 0 : 1, 0) != 0);
      const int tick0 = __shfl_sync(0xffffffffu, tk[0], 0);
      const int tick = __shfl_sync(0xffffffffu, sl ? tk[1] : tk[0], 0);
      if (!got) break;
      if (lane == 0) sched_release(i);
      if (tick0 < 0) break;
      if (tick < 0) continue;  // this slot idles this round
      int b, h;
      ps_pair(tick, prm.H, b, h);
      h += (int)rank;
      const bool live = h < prm.H;  // odd H: the pair's second head does not exist
      int which = 0, hloc = 0, nheads = 1;
      if (live) split_head(h, prm.NH, prm.NKVH, which, hloc, nheads);
      const int hh = live ? h : 0;
      __nv_bfloat16* orow = (which == 0 ? prm.out[0] : (which == 1 ? prm.out[1] : prm.out[2])) +
                            ((long long)b * nheads + hloc) * prm.T * kPsD;  // the head's [T][128] output
      __nv_bfloat16* obase = orow + c;
      const bool rope = prm.rope_cos != nullptr && which < 2;  // the same for the warpgroup's four warps
      const long long vrow0 = (long long)b * prm.F + hh * (kPsD + 1) + q * 32;  // the warp's first value row
      const __nv_bfloat16* lrow = prm.combined + ((long long)b * prm.F + hh * (kPsD + 1) + kPsD) * prm.T;
      const float lb = prm.logit_bias[hh];
      float E = __bfloat162float(prm.inits[(long long)b * prm.inits_bs + (long long)hh * kPsD + c]);
      uint4 lg = live ? ps_load_logits(lrow, lane * 8, prm.T) : make_uint4(0, 0, 0, 0);
      bool ok = true;
      for (int nt = 0; nt < prm.n_tiles; ++nt) {
        const int n0 = nt * kPsBN;
        if (live) {
          // gates of the tile's 256 tokens, 8 per lane (identity beyond T); then the next tile's logits
          __syncwarp();  // the previous tile's walk has read every gate
          const uint32_t w4[4] = {lg.x, lg.y, lg.z, lg.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int t = lane * 8 + 2 * j;
            const float l0 = __uint_as_float(w4[j] << 16) + lb, l1 = __uint_as_float(w4[j] & 0xffff0000u) + lb;
            float a0 = 0.f, a1 = 0.f;
            if (n0 + t < prm.T) {
              a0 = prm.use_sigmoid ? sigmoid_f32(l0) : l0;
              a1 = prm.use_sigmoid ? sigmoid_f32(l1) : l1;
            }
            *reinterpret_cast<float4*>(gw + t) = make_float4(1.0f - a0, a0, 1.0f - a1, a1);
          }
          if (nt + 1 < prm.n_tiles) lg = ps_load_logits(lrow, n0 + kPsBN + lane * 8, prm.T);
          __syncwarp();
        }
        const bool got2 = mbar_wait(&tfull_bar[sl], acc_phase, abort_flag, ws, 0x6a02);
        if (rope ? named_barrier_or(gbar, 128, !got2) : __any_sync(0xffffffffu, !got2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(sl * kPsBN);
        uint32_t pcos[8], psin[8];  // rotary: the next block's table pairs, carried across iterations
#pragma unroll 1
        for (int hb = 0; hb < kPsBN / 32; ++hb) {
          const int c0 = n0 + hb * 32;
          if (!live || c0 >= prm.T) break;  // uniform; T % 32 == 0, so the 32 tokens are all inside T
          // rotary: this warp's 8 tokens' table pairs of this block (loaded one block ahead) and the next's
          uint32_t rcos[8], rsin[8], ncos[8], nsin[8];
          if (rope) {
            if (hb == 0) ps_rope_rows(prm, c0 + q * 8, lane, rcos, rsin);
            else {
#pragma unroll
              for (int tt = 0; tt < 8; ++tt) { rcos[tt] = pcos[tt]; rsin[tt] = psin[tt]; }
            }
            if (hb + 1 < kPsBN / 32 && c0 + 32 < prm.T) ps_rope_rows(prm, c0 + 32 + q * 8, lane, ncos, nsin);
          }
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_row + (uint32_t)(hb * 32), v);
          tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            __nv_bfloat162 p2 = __floats2bfloat162_rn(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
            pk[j] = *reinterpret_cast<uint32_t*>(&p2);
          }
          // ---- u = bf16(acc) into `combined`: this thread's channel row holds 32 tokens (64 B);
          //      the transpose lets each store instruction write eight 64-byte row pieces ----
#pragma unroll
          for (int j = 0; j < 4; ++j)
            *reinterpret_cast<uint4*>(xp + lane * 64 + ((j ^ ((lane >> 1) & 3)) * 16)) =
                make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int r8 = k * 8 + lane / 4, jj = lane & 3;
            const uint4 val = *reinterpret_cast<const uint4*>(xp + r8 * 64 + ((jj ^ ((r8 >> 1) & 3)) * 16));
            *reinterpret_cast<uint4*>(prm.combined + (vrow0 + r8) * prm.T + c0 + jj * 8) = val;
          }
          __syncwarp();  // the buffer is free for the next 32 tokens
          const int tb = hb * 32;
          if (!rope) {
            // ---- the recurrence over the same 32 tokens; a warp stores 64 contiguous bytes per token ----
            __nv_bfloat16* op = obase + (long long)c0 * kPsD;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const uint32_t w = pk[j];
              const float u0 = __uint_as_float(w << 16), u1 = __uint_as_float(w & 0xffff0000u);
              const float4 g = *reinterpret_cast<const float4*>(gw + tb + 2 * j);
              E = __fmaf_rn(g.x, E, __fmul_rn(g.y, u0));
              op[(2 * j) * kPsD] = __float2bfloat16_rn(E);
              E = __fmaf_rn(g.z, E, __fmul_rn(g.w, u1));
              op[(2 * j + 1) * kPsD] = __float2bfloat16_rn(E);
            }
          } else {
            // ---- the recurrence into the group's [32][128] tile, then rotary + norm per token ----
            named_barrier(gbar, 128);  // every transpose buffer of the group is read
            __nv_bfloat16* sg = reinterpret_cast<__nv_bfloat16*>(stg) + c;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const uint32_t w = pk[j];
              const float u0 = __uint_as_float(w << 16), u1 = __uint_as_float(w & 0xffff0000u);
              const float4 g = *reinterpret_cast<const float4*>(gw + tb + 2 * j);
              E = __fmaf_rn(g.x, E, __fmul_rn(g.y, u0));
              sg[(2 * j) * kPsD] = __float2bfloat16_rn(E);
              E = __fmaf_rn(g.z, E, __fmul_rn(g.w, u1));
              sg[(2 * j + 1) * kPsD] = __float2bfloat16_rn(E);
            }
            named_barrier(gbar, 128);  // the tile is complete
            const uint32_t* s32 = reinterpret_cast<const uint32_t*>(stg);
            float y[8][4], ss[8];
#pragma unroll
            for (int tt = 0; tt < 8; ++tt) {
              const int t = q * 8 + tt;
              uint32_t r1, r2;
              rope_rotate_bf16x2(s32[t * (kPsD / 2) + lane], s32[t * (kPsD / 2) + 32 + lane], rcos[tt], rsin[tt],
                                 r1, r2);
              y[tt][0] = bf16_lo(r1); y[tt][1] = bf16_hi(r1); y[tt][2] = bf16_lo(r2); y[tt][3] = bf16_hi(r2);
              ss[tt] = 0.f;
#pragma unroll
              for (int e = 0; e < 4; ++e) ss[tt] = __fmaf_rn(y[tt][e], y[tt][e], ss[tt]);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
              for (int tt = 0; tt < 8; ++tt) ss[tt] += __shfl_xor_sync(0xffffffffu, ss[tt], o);
            }
#pragma unroll
            for (int tt = 0; tt < 8; ++tt) {
              const float inv = rope_inv_rms(ss[tt], kPsD, prm.rope_eps);
              uint32_t* orow32 = reinterpret_cast<uint32_t*>(orow + (long long)(c0 + q * 8 + tt) * kPsD);
              orow32[lane] = pack_bf16x2(y[tt][0] * inv, y[tt][1] * inv);
              orow32[32 + lane] = pack_bf16x2(y[tt][2] * inv, y[tt][3] * inv);
            }
            named_barrier(gbar, 128);  // the tile is read: the buffers are free again
#pragma unroll
            for (int tt = 0; tt < 8; ++tt) { pcos[tt] = ncos[tt]; psin[tt] = nsin[tt]; }
          }
          // the state entering the next 32 tokens: the backward replays each 32-token chunk from
          // it instead of re-reading the chunk's outputs (a warp writes 128 contiguous bytes)
          if (prm.ckpt != nullptr && c0 + 32 < prm.T)
            prm.ckpt[(((long long)b * prm.H + hh) * (prm.T / 32) + c0 / 32) * kPsD + c] = E;
        }
        if (!ok) break;
        // all TMEM reads of this accumulator are complete (tcgen05.wait::ld above)
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster_relaxed(tempty_leader);
        acc_phase ^= 1u;
      }
      if (!ok) break;
    }
    __syncwarp();
  }

  tc_fence_before();
  cluster_sync_all();  // no CTA of the pair touches the other's memory or TMEM after this
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, 512);
  if (threadIdx.x == 0) finish_launch(ws, gridDim.x);
}

}  // namespace ltvqkv
