// Row-streaming, TMA-fed bf16 scan kernels for the exact production layout (included by
// ltvqkv_scan.cu): combined / grad_combined are the transposed view of a contiguous [B, F, T]
// buffer, so one 2-D tensor map [B*F rows, T columns] addresses every head's value and logit rows.
//
// A persistent CTA owns whole (batch, head) rows (the forward draws them from a ticket counter, the
// backward takes rows blockIdx.x, blockIdx.x + gridDim.x, ...: rows cost the same), and walks each row
// chunk by chunk (kTT = 32 or 64 tokens; forward in time order, backward in reverse). Consumer
// thread c owns channel c and walks all kTT tokens of a chunk, so the carry never leaves its
// register: no look-back, no inter-CTA communication, results fixed by construction. One producer
// warp streams the row's chunks into a ring of shared-memory stages with cp.async.bulk.tensor
// (mbarrier full/empty pairs): the value tile (128- or 64-byte swizzle), the logit rows, and at a
// row's first chunk the row's initial state (plain bulk copy). The logit bias of every head sits
// in shared memory for the whole launch, so no global load is on a chunk's critical path.
//
// Forward: the chunk's output tile [kTT][D] is written over the value tile it came from (every
// value row is in registers by then) and leaves as one contiguous bulk store; the stage is handed
// back to the producer once that store has read it (one chunk later).
// Backward: thread c alone reads its channel's slots of the chunk's value tile (16 bytes per 8
// tokens), gradient tile G and state tile H (2 bytes per token each), so once it has read them it
// reuses them: du goes back into the value-tile slot (the tile then leaves as one bulk tensor store
// into grad_combined) and dalpha(t, c) as an fp32 split into its high and low halves into G[t][c]
// and H[t][c]; the per-(group, token) sums read that table after one barrier.
// Chosen when there are enough rows to fill the GPU (B * heads >= 2 * SMs); fewer, longer rows
// take the chunk-parallel look-back kernels. Every wait is bounded (2 s) and reports
// LTVQKV_ERR_TIMEOUT through the workspace.
#pragma once

namespace ltvqkv {

constexpr int kRowMaxStages = 8;
constexpr int kRowMaxBias = 4096;  // heads * Da logit-bias entries held in shared memory

struct TmaFwdArgs {
  const __nv_bfloat16* inits;
  const float* logit_bias;
  __nv_bfloat16* out[3];
  int B, T, NH, NKVH, Da, r, D, H, F, nchunks, nrows, use_sigmoid;
  int stages;  // shared-memory ring depth (2..kRowMaxStages)
  WorkspaceHeader* ws;
};

struct TmaBwdArgs {
  const __nv_bfloat16* inits;
  const float* logit_bias;
  __nv_bfloat16* grad_combined;
  __nv_bfloat16* grad_inits;
  float* bias_part;  // [B][H][Da]: one partial per row
  float* grad_bias;  // backward: [H][Da], the partials' sums are added here by the last CTA
  const float* ckpt; // backward from checkpoints: [B][H][nchunks][D], the fp32 state entering chunk j + 1
  long long inits_bs;    // elements between sequences' initial states (0: one state shared by the batch)
  // shared initial state: per-row gradients (each rounded to bf16) go to init_part [B][H][D], and
  // the row that completes a head's batch sums them in batch order into grad_init_sum [H][D] (fp32)
  float* init_part;
  unsigned int* init_cnt;  // [H] rows of each head done (zero at launch)
  float* grad_init_sum;
  int bias_overwrite;      // grad_bias = sum (1) or grad_bias += sum (0)
  int B, T, NH, NKVH, Da, r, D, H, F, nchunks, nrows, use_sigmoid;
  int stages;  // shared-memory ring depth (2..kRowMaxStages)
  WorkspaceHeader* ws;
};

struct RowTile {  // written by the producer for each staged chunk; row < 0 ends the stream
  int row, b, h, j, t0, tlen, which, hloc, nheads;
};

__host__ __device__ constexpr int row_align(int v, int a) { return (v + a - 1) / a * a; }
// Logit box of the backward: the chunk's kTT tokens plus the next chunk's first, padded to 16 bytes.
__host__ __device__ constexpr int row_bwd_logit_box(int tt) { return tt + 8; }

// Forward stage: value tile [D][kTT] (swizzled) | logits [Da][kTT] | initial state [D].
__host__ __device__ constexpr int row_fwd_logit_off(int D, int tt) { return D * tt * 2; }
__host__ __device__ constexpr int row_fwd_init_off(int D, int Da, int tt) {
  return row_fwd_logit_off(D, tt) + row_align(Da * tt * 2, 128);
}
__host__ __device__ constexpr int row_fwd_stage_bytes(int D, int Da, int tt) {
  return row_align(row_fwd_init_off(D, Da, tt) + D * 2, 1024);
}
// Backward stage: value tile [D][kTT] | logits [Da][kTT + 8] | G [kTT][D] | H [kTT][D] | initial state [D].
__host__ __device__ constexpr int row_bwd_logit_off(int D, int tt) { return D * tt * 2; }
__host__ __device__ constexpr int row_bwd_g_off(int D, int Da, int tt) {
  return row_bwd_logit_off(D, tt) + row_align(Da * row_bwd_logit_box(tt) * 2, 128);
}
__host__ __device__ constexpr int row_bwd_h_off(int D, int Da, int tt) { return row_bwd_g_off(D, Da, tt) + tt * D * 2; }
__host__ __device__ constexpr int row_bwd_init_off(int D, int Da, int tt) {
  return row_bwd_h_off(D, Da, tt) + tt * D * 2;
}
__host__ __device__ constexpr int row_bwd_stage_bytes(int D, int Da, int tt) {
  return row_align(row_bwd_init_off(D, Da, tt) + D * 2, 1024);
}

inline size_t row_fwd_smem_bytes(int D, int Da, int H, int tt, int stages) {
  return 1024 + (size_t)stages * row_fwd_stage_bytes(D, Da, tt) + (size_t)row_align(H * Da, 4) * 4 +
         (size_t)8 * Da * tt + sizeof(RowTile) * stages + 16 + 16 * stages + 64;
}
inline size_t row_bwd_smem_bytes(int D, int Da, int H, int tt, int stages) {
  return 1024 + (size_t)stages * row_bwd_stage_bytes(D, Da, tt) + (size_t)row_align(H * Da, 4) * 4 +
         (size_t)16 * Da * tt * stages + (size_t)4 * (D / 32) * tt + (size_t)4 * Da * tt + sizeof(RowTile) * stages + 16 +
         24 * stages + 64;
}


// Occupancy targets (CTAs per SM) for __launch_bounds__, from the Da = 1 shared-memory footprint
// and a floor of 64 (forward) / 96 (backward) registers per thread.
constexpr int row_min_blocks(int smem, int threads, int regs) {
  const int by_smem = (225 * 1024) / smem;
  const int by_regs = 65536 / (threads * regs);
  const int b = by_smem < by_regs ? by_smem : by_regs;
  return b < 1 ? 1 : (b > 8 ? 8 : b);
}
constexpr int row_fwd_min_blocks(int D, int tt) {
  return row_min_blocks(4 * row_fwd_stage_bytes(D, 1, tt) + 3072, D + 32, 64);
}
constexpr int row_bwd_min_blocks(int D, int tt, bool ckpt) {
  return row_min_blocks(2 * row_bwd_stage_bytes(D, 1, tt) + 3072, D / 2 + (ckpt ? 64 : 32), 128);
}


// 16-byte chunk k of row `row` in a tile of kTT bf16 per row, as TMA writes it with the 128-byte
// (kTT = 64) or 64-byte (kTT = 32) swizzle.

template <int kTT>
LTVQKV_DEVICE const uint4* swz_chunk(const uint8_t* tile, int row, int k) {
  if constexpr (kTT == 64) {
    return reinterpret_cast<const uint4*>(tile + row * 128 + ((k ^ (row & 7)) << 4));
  } else {
    return reinterpret_cast<const uint4*>(tile + row * 64 + ((k ^ ((row >> 1) & 3)) << 4));
  }
}

// ------------------------------------------------------------------------------------------
// Forward
// ------------------------------------------------------------------------------------------
template <int kD, int kTT>  // head dim = consumer threads; constants, so smem offsets are immediates
__global__ void __launch_bounds__(kD + 32, row_fwd_min_blocks(kD, kTT))
    scan_fwd_rows_kernel(const __grid_constant__ CUtensorMap tm_u, const __grid_constant__ CUtensorMap tm_l,
                         const TmaFwdArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint8_t* base = smem_align<uint8_t>(smem_raw, 1024);
  constexpr int D = kD, ncons = kD;
  const int S = a.stages;
  const int Da = a.Da;
  const int sbytes = row_fwd_stage_bytes(D, Da, kTT);
  constexpr int loff = row_fwd_logit_off(D, kTT);
  const int ioff = row_fwd_init_off(D, Da, kTT);
  const int nlb = a.H * Da;
  uint8_t* stages = base;
  float* lb_s = reinterpret_cast<float*>(stages + S * sbytes);               // [H][Da]
  float2* gates = reinterpret_cast<float2*>(lb_s + row_align(nlb, 4));       // [Da][kTT]: (1 - a, a)
  RowTile* info = reinterpret_cast<RowTile*>(gates + Da * kTT);              // [S]
  uint64_t* full = smem_align<uint64_t>(info + S, 16);
  uint64_t* empty = full + S;
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);  // released by thread 0 once the chunk's bulk store has read the stage
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  for (int q = tid; q < nlb; q += blockDim.x) lb_s[q] = a.logit_bias[q];
  __syncthreads();

  if (warp == ncons / 32) {
    // ---------------- producer: rows from the ticket counter, chunks in time order ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tm_u);
      tma_prefetch_desc(&tm_l);
      int i = 0;
      bool ok = true;
      while (ok) {
        int row = (int)draw_ticket(a.ws);
        if (row >= a.nrows) row = -1;
        const int nch = row < 0 ? 1 : a.nchunks;
        const int b = row < 0 ? 0 : row / a.H, h = row < 0 ? 0 : row % a.H;
        int which = 0, hloc = 0, nheads = 0;
        if (row >= 0) split_head(h, a.NH, a.NKVH, which, hloc, nheads);
        const int frow = b * a.F + h * (D + Da);
        for (int j = 0; j < nch; ++j, ++i) {
          const int st = i % S;
          const uint32_t ph = (uint32_t)(i / S) & 1u;
          if (!mbar_wait(&empty[st], ph ^ 1u, &abort_flag, a.ws, 0x7101)) { ok = false; break; }
          RowTile& ti = info[st];
          ti.row = row;
          if (row < 0) {
            mbar_arrive(&full[st]);
            ok = false;
            break;
          }
          ti.b = b; ti.h = h; ti.j = j; ti.t0 = j * kTT; ti.tlen = min(kTT, a.T - j * kTT);
          ti.which = which; ti.hloc = hloc; ti.nheads = nheads;
          uint8_t* sb = stages + st * sbytes;
          const uint32_t bytes = (uint32_t)((D + Da) * kTT * 2 + (j == 0 ? D * 2 : 0));
          mbar_arrive_expect_tx(&full[st], bytes);
          tma_load_2d(sb, &tm_u, &full[st], j * kTT, frow);
          tma_load_2d(sb + loff, &tm_l, &full[st], j * kTT, frow + D);
          if (j == 0) bulk_load(sb + ioff, a.inits + ((long long)b * a.H + h) * D, D * 2, &full[st]);
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- consumers: thread c = channel ----------------
    const int c = tid;
    const int gi = c / a.r;
    float E = 0.f;  // row carry: h at the last token of the previous chunk
    for (int i = 0;; ++i) {
      const int st = i % S;
      const uint32_t ph = (uint32_t)(i / S) & 1u;
      if (!mbar_wait(&full[st], ph, &abort_flag, a.ws, 0x7102)) break;
      const RowTile ti = info[st];
      if (ti.row < 0) break;
      uint8_t* sb = stages + st * sbytes;
      if (ti.j == 0) E = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(sb + ioff)[c]);
      if (tid < Da * kTT) {
        const int g = tid / kTT, t = tid % kTT;
        float al = 0.f;  // beyond T: identity steps
        if (t < ti.tlen) {
          const float l = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(sb + loff)[g * kTT + t]) +
                          lb_s[ti.h * Da + g];
          al = a.use_sigmoid ? sigmoid_f32(l) : l;
        }
        gates[tid] = make_float2(1.0f - al, al);
      }
      uint4 uv[kTT / 8];
#pragma unroll
      for (int k = 0; k < kTT / 8; ++k) uv[k] = *swz_chunk<kTT>(sb, c, k);
      named_barrier(1, ncons);  // gates ready; every value row is in registers

      // the output tile [kTT][D] overwrites the value tile
      const float2* grow = gates + gi * kTT;
      __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(sb) + c;
#pragma unroll
      for (int k = 0; k < kTT / 8; ++k) {
        float f[8];
        unpack8(uv[k], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float2 g2 = grow[8 * k + e];
          E = __fmaf_rn(g2.x, E, __fmul_rn(g2.y, f[e]));
          ob[(8 * k + e) * D] = __float2bfloat16_rn(E);
        }
      }
      fence_proxy_async_smem();
      named_barrier(1, ncons);
      if (tid == 0) {
        __nv_bfloat16* o0 = ti.which == 0 ? a.out[0] : (ti.which == 1 ? a.out[1] : a.out[2]);
        __nv_bfloat16* go = o0 + (((long long)ti.b * ti.nheads + ti.hloc) * a.T + ti.t0) * D;
        bulk_store(go, sb, (uint32_t)(ti.tlen * D * 2));
        tma_store_commit();
        if (i > 0) {  // the previous chunk's store has read its stage: hand it back
          tma_store_wait_read1();
          mbar_arrive(&empty[(i - 1) % S]);
        }
      }
    }
    if (tid == 0) tma_store_wait0();
  }
  __syncthreads();
  if (tid == 0) finish_launch(a.ws, gridDim.x);
}

// ------------------------------------------------------------------------------------------
// Backward
// ------------------------------------------------------------------------------------------
// kCkpt: h_{t-1} is not read from the forward's outputs but replayed per chunk from the fp32 state
// the forward stored at the chunk's start (its recurrence step for step, so the replayed outputs are
// the forward's bit for bit); the chunk's 8 KB output tile becomes a 512-byte state read. A fourth
// warp replays each chunk while the consumers walk the previous one, so the consumers' per-chunk
// path is unchanged.
template <int kD, int kTT, bool kCkpt>
__global__ void __launch_bounds__(kD / 2 + (kCkpt ? 64 : 32), row_bwd_min_blocks(kD, kTT, kCkpt))
    scan_bwd_rows_kernel(const __grid_constant__ CUtensorMap tm_u, const __grid_constant__ CUtensorMap tm_l,
                         const __grid_constant__ CUtensorMap tm_du,
                         const __grid_constant__ CUtensorMap tm_gq, const __grid_constant__ CUtensorMap tm_gk,
                         const __grid_constant__ CUtensorMap tm_gv, const __grid_constant__ CUtensorMap tm_hq,
                         const __grid_constant__ CUtensorMap tm_hk, const __grid_constant__ CUtensorMap tm_hv,
                         const TmaBwdArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint8_t* base = smem_align<uint8_t>(smem_raw, 1024);
  constexpr int D = kD, ncons = kD / 2, LB = row_bwd_logit_box(kTT);  // a consumer owns two channels
  const int S = a.stages;
  const int Da = a.Da;
  const int sbytes = row_bwd_stage_bytes(D, Da, kTT);
  constexpr int loff = row_bwd_logit_off(D, kTT);
  const int goff = row_bwd_g_off(D, Da, kTT), hoff = row_bwd_h_off(D, Da, kTT), ioff = row_bwd_init_off(D, Da, kTT);
  const int nlb = a.H * Da;
  uint8_t* stages = base;
  float* lb_s = reinterpret_cast<float*>(stages + S * sbytes);               // [H][Da]
  // per stage: (1 - alpha_{t+1}, alpha_t, alpha_t (1 - alpha_t)) of the chunk's tokens, written by the
  // consumers, or with checkpoints by the replay warp one chunk ahead of them
  float4* gates = reinterpret_cast<float4*>(lb_s + row_align(nlb, 4));       // [S][Da][kTT]
  // dalpha partial sums per lane segment (see below) and per-row logit-bias sums
  float* part = reinterpret_cast<float*>(gates + S * Da * kTT);              // [D / 32][kTT]
  float* bsum = part + (D / 32) * kTT;                                        // [Da][kTT]
  RowTile* info = reinterpret_cast<RowTile*>(bsum + Da * kTT);               // [S]
  uint64_t* full = smem_align<uint64_t>(info + S, 16);
  uint64_t* empty = full + S;
  uint64_t* hfull = empty + S;  // kCkpt: the stage's replayed outputs are in place (32 replay lanes)
  __shared__ volatile int abort_flag;
  __shared__ int init_last;  // this row completed its head's batch (shared initial state)

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], ncons / 32);
      if (kCkpt) mbar_init(&hfull[i], 32);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  for (int q = tid; q < nlb; q += blockDim.x) lb_s[q] = a.logit_bias[q];
  __syncthreads();

  if (warp == ncons / 32) {
    // ---------------- producers: rows blockIdx.x, + gridDim.x, ...; chunks in reverse time order ----------------
    // Lanes 0-3 walk the same chunk sequence and each issues one of a chunk's copies (lane 0: the
    // value tile, with the stage's bookkeeping; 1: the logit rows; 2: the gradient tile; 3: the
    // state tile or checkpoint, and the initial state): one thread issues about one bulk-tensor copy
    // per few hundred cycles, so the four land together instead of one after another.
    if (lane < 4) {
      if (lane == 0) {
        tma_prefetch_desc(&tm_u);
        tma_prefetch_desc(&tm_l);
      }
      int i = 0;
      bool ok = true;
      for (int row = (int)blockIdx.x; ok; row += (int)gridDim.x) {
        const bool end = row >= a.nrows;
        const int nch = end ? 1 : a.nchunks;
        const int b = end ? 0 : row / a.H, h = end ? 0 : row % a.H;
        int which = 0, hloc = 0, nheads = 0;
        if (!end) split_head(h, a.NH, a.NKVH, which, hloc, nheads);
        const int frow = b * a.F + h * (D + Da);
        const CUtensorMap* mg = which == 0 ? &tm_gq : (which == 1 ? &tm_gk : &tm_gv);
        const CUtensorMap* mh = which == 0 ? &tm_hq : (which == 1 ? &tm_hk : &tm_hv);
        for (int q = 0; q < nch; ++q, ++i) {
          const int st = i % S;
          const uint32_t ph = (uint32_t)(i / S) & 1u;
          if (!mbar_wait(&empty[st], ph ^ 1u, &abort_flag, a.ws, 0x7201)) { ok = false; break; }
          if (end) {
            if (lane == 0) {
              info[st].row = -1;
              mbar_arrive(&full[st]);
            }
            ok = false;
            break;
          }
          const int j = a.nchunks - 1 - q;
          const int t0 = j * kTT;
          uint8_t* sb = stages + st * sbytes;
          if (lane == 0) {
            RowTile& ti = info[st];
            ti.row = row;
            ti.b = b; ti.h = h; ti.j = j; ti.t0 = t0; ti.tlen = min(kTT, a.T - t0);
            ti.which = which; ti.hloc = hloc; ti.nheads = nheads;
            const uint32_t hbytes = kCkpt ? (j > 0 ? D * 4 : 0) : kTT * D * 2;
            const uint32_t bytes = (uint32_t)(D * kTT * 2 + Da * LB * 2 + kTT * D * 2 + hbytes + (q == 0 ? D * 2 : 0));
            mbar_arrive_expect_tx(&full[st], bytes);
            tma_load_2d(sb, &tm_u, &full[st], t0, frow);
          } else if (lane == 1) {
            tma_load_2d(sb + loff, &tm_l, &full[st], t0, frow + D);
          } else if (lane == 2) {
            tma_load_4d(sb + goff, mg, &full[st], 0, t0, hloc, b);
          } else {
            if (!kCkpt)
              tma_load_4d(sb + hoff, mh, &full[st], 0, t0 - 1, hloc, b);
            else if (j > 0)
              bulk_load(sb + hoff, a.ckpt + (((long long)b * a.H + h) * a.nchunks + (j - 1)) * D, D * 4, &full[st]);
            if (q == 0) bulk_load(sb + ioff, a.inits + (long long)b * a.inits_bs + (long long)h * D, D * 2, &full[st]);
          }
        }
      }
    }
    __syncwarp();
  } else if (kCkpt && warp == ncons / 32 + 1) {
    // ---------------- replay (kCkpt): H32 row t = h_{t0 + t - 1}, from the chunk's entering state ----------------
    // Lane l does the work of consumers l and l + 32 (channel pairs (2l, 2l + 1) and (2l + 64,
    // 2l + 65)) with their conflict-free read order, one chunk ahead of them. The forward's
    // arithmetic step for step: alpha = sigmoid(logit + bias), E = fma(1 - alpha, E, alpha * u), h = bf16(E).
    static_assert(!kCkpt || kD == 128, "checkpoints come from the head-dim-128 fused forward");
    const int sw = (lane >> 2) & 1;
    uint32_t initA = 0, initB = 0;  // h_{-1} of the two channel pairs
    for (int i = 0;; ++i) {
      const int st = i % S;
      const uint32_t ph = (uint32_t)(i / S) & 1u;
      if (!mbar_wait(&full[st], ph, &abort_flag, a.ws, 0x7203)) break;
      const RowTile ti = info[st];
      if (ti.row < 0) break;
      uint8_t* sb = stages + st * sbytes;
      if (ti.j == a.nchunks - 1) {
        initA = reinterpret_cast<const uint32_t*>(sb + ioff)[lane];
        initB = reinterpret_cast<const uint32_t*>(sb + ioff)[lane + 32];
      }
      // alpha of token t0 + lane (one decay group; the chunk is whole: T % 32 == 0)
      const __nv_bfloat16* L_s = reinterpret_cast<const __nv_bfloat16*>(sb + loff);
      const float lg = __bfloat162float(L_s[lane]) + lb_s[ti.h];
      const float al_l = a.use_sigmoid ? sigmoid_f32(lg) : lg;
      {
        // the consumers' gates of this chunk: alpha_{t+1} from the next lane, or for the last token
        // the next chunk's first (identity beyond T), with the consumers' own arithmetic
        float an = __shfl_down_sync(0xffffffffu, al_l, 1);
        if (lane == kTT - 1) {
          an = 0.f;
          if (ti.t0 + kTT < a.T) {
            const float ln = __bfloat162float(L_s[kTT]) + lb_s[ti.h];
            an = a.use_sigmoid ? sigmoid_f32(ln) : ln;
          }
        }
        gates[st * kTT + lane] = make_float4(1.0f - an, al_l, a.use_sigmoid ? al_l * (1.0f - al_l) : 1.0f, 0.f);
      }
      float E0, E1, E2, E3;
      if (ti.j == 0) {
        E0 = __uint_as_float(initA << 16); E1 = __uint_as_float(initA & 0xffff0000u);
        E2 = __uint_as_float(initB << 16); E3 = __uint_as_float(initB & 0xffff0000u);
      } else {
        const float2 ea = reinterpret_cast<const float2*>(sb + hoff)[lane];
        const float2 eb = reinterpret_cast<const float2*>(sb + hoff)[lane + 32];
        E0 = ea.x; E1 = ea.y; E2 = eb.x; E3 = eb.y;
      }
      __syncwarp();  // every lane has its state before row 0 is written over the stored states
      uint32_t* H32 = reinterpret_cast<uint32_t*>(sb + hoff);
      H32[lane] = pack_bf16x2(E0, E1);
      H32[lane + 32] = pack_bf16x2(E2, E3);
#pragma unroll
      for (int k = 0; k < kTT / 8; ++k) {
        const int ra = 2 * lane, rb = 2 * lane + 64;
        const uint4 a0 = *swz_chunk<kTT>(sb, ra + sw, k), a1 = *swz_chunk<kTT>(sb, ra + 1 - sw, k);
        const uint4 b0 = *swz_chunk<kTT>(sb, rb + sw, k), b1 = *swz_chunk<kTT>(sb, rb + 1 - sw, k);
        float fa0[8], fa1[8], fb0[8], fb1[8];
        unpack8(sw ? a1 : a0, fa0);
        unpack8(sw ? a0 : a1, fa1);
        unpack8(sw ? b1 : b0, fb0);
        unpack8(sw ? b0 : b1, fb1);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int t = 8 * k + e;
          if (t + 1 < kTT) {
            const float al = __shfl_sync(0xffffffffu, al_l, t);
            const float om = 1.0f - al;
            E0 = __fmaf_rn(om, E0, __fmul_rn(al, fa0[e]));
            E1 = __fmaf_rn(om, E1, __fmul_rn(al, fa1[e]));
            E2 = __fmaf_rn(om, E2, __fmul_rn(al, fb0[e]));
            E3 = __fmaf_rn(om, E3, __fmul_rn(al, fb1[e]));
            H32[(t + 1) * (D / 2) + lane] = pack_bf16x2(E0, E1);
            H32[(t + 1) * (D / 2) + lane + 32] = pack_bf16x2(E2, E3);
          }
        }
      }
      mbar_arrive(&hfull[st]);  // release: this lane's H32 and gate writes are visible to the consumers' wait
    }
    __syncwarp();
  } else {
    // ---------------- consumers: thread = channel pair (2 tid, 2 tid + 1) ----------------
    // Two adjacent channels per thread: every 16-bit G/H access of the walk becomes one 32-bit
    // access, a full 128-byte shared-memory wavefront per warp instead of half of one.
    static_assert(kTT == 32, "the backward walks 32-token chunks (four 8-token blocks)");
    const int gi = (2 * tid) / a.r;  // r is even, so both channels share the decay group
    // dalpha group sums: a "segment" of lanes covers min(r, 64) channels of one group; within a
    // warp, each 8-token block is reduced by a transposing butterfly (three halving rounds, then
    // plain rounds), so lane l ends with the segment's sum of token (l / (seg/8)) & 7 of the block.
    const int seg = a.r >= 64 ? 32 : a.r / 2;        // lanes per segment (16 or 32)
    const int m1 = seg / 2, m2 = seg / 4, m3 = seg / 8;
    const int tloc = ((lane & m1) ? 4 : 0) + ((lane & m2) ? 2 : 0) + ((lane & m3) ? 1 : 0);
    const bool canon = (lane & (m3 - 1)) == 0;        // one lane per (segment, token) writes
    const int segid = warp * (32 / seg) + lane / seg;
    const int spg = a.r / (2 * seg);                  // segments per group
    // value-tile rows 2 tid and 2 tid + 1 are read in lane-dependent order, so that the 8 lanes of
    // a shared-memory phase hit 8 different 16-byte bank groups under the tile's swizzle
    const int sw = (lane >> 2) & 1;
    float carry0 = 0.f, carry1 = 0.f;  // adjoints of h at the first token of the previous chunk
    uint32_t init2 = 0;                 // h_{-1} of both channels (bf16 pair)
    float bias_q[2] = {0.f, 0.f};       // this row's dlogit sums of (group, token) entries q = tid + i*ncons
    for (int i = 0;; ++i) {
      const int st = i % S;
      const uint32_t ph = (uint32_t)(i / S) & 1u;
      if (!mbar_wait(&full[st], ph, &abort_flag, a.ws, 0x7202)) break;
      const RowTile ti = info[st];
      if (ti.row < 0) break;
      const long long rowbase = (long long)ti.b * a.H + ti.h;
      uint8_t* sb = stages + st * sbytes;
      if (ti.j == a.nchunks - 1) {
        carry0 = carry1 = 0.f;
        bias_q[0] = bias_q[1] = 0.f;
        init2 = reinterpret_cast<const uint32_t*>(sb + ioff)[tid];
      }
      const __nv_bfloat16* L_s = reinterpret_cast<const __nv_bfloat16*>(sb + loff);
      const uint32_t* G32 = reinterpret_cast<const uint32_t*>(sb + goff);
      uint32_t* H32 = reinterpret_cast<uint32_t*>(sb + hoff);
      // h_{t-1} of the row's first token is the initial state (the tile's row -1 was filled with 0)
      if (!kCkpt && ti.t0 == 0) H32[tid] = init2;
      float4* gst = gates + st * Da * kTT;
      for (int q = tid; !kCkpt && q < Da * kTT; q += ncons) {
        const int g = q / kTT, t = q % kTT;
        const float lb = lb_s[ti.h * Da + g];
        float al = 0.f, an = 0.f;  // alpha_t and alpha_{t+1}; identity steps beyond T
        if (t < ti.tlen) {
          const float l = __bfloat162float(L_s[g * LB + t]) + lb;
          al = a.use_sigmoid ? sigmoid_f32(l) : l;
        }
        if (ti.t0 + t + 1 < a.T) {
          const float l = __bfloat162float(L_s[g * LB + t + 1]) + lb;
          an = a.use_sigmoid ? sigmoid_f32(l) : l;
        }
        gst[q] = make_float4(1.0f - an, al, a.use_sigmoid ? al * (1.0f - al) : 1.0f, 0.f);
      }
      if (!kCkpt) named_barrier(1, ncons);  // gates ready (with checkpoints: the replay warp's, below)

      const float4* grow = gst + gi * kTT;
      if (kCkpt && !mbar_wait(&hfull[st], ph, &abort_flag, a.ws, 0x7204)) break;  // replayed outputs in place

      // reverse walk: adjoint carries, du, and the per-token dalpha terms of both channels
      // one 8-token block per iteration: unrolling across blocks would let every block's loads be
      // hoisted to the top and spill
#pragma unroll 1
      for (int k = kTT / 8 - 1; k >= 0; --k) {
        uint4* slotA = const_cast<uint4*>(swz_chunk<kTT>(sb, 2 * tid + sw, k));
        uint4* slotB = const_cast<uint4*>(swz_chunk<kTT>(sb, 2 * tid + 1 - sw, k));
        const uint4 vA = *slotA, vB = *slotB;
        float f0[8], f1[8], du0[8], du1[8], ds[8];
        unpack8(sw ? vB : vA, f0);
        unpack8(sw ? vA : vB, f1);
#pragma unroll
        for (int e = 7; e >= 0; --e) {
          const int t = 8 * k + e;
          const float4 gv = grow[t];
          const uint32_t g2 = G32[t * (D / 2) + tid], h2 = H32[t * (D / 2) + tid];
          carry0 = gv.x * carry0 + __uint_as_float(g2 << 16);
          carry1 = gv.x * carry1 + __uint_as_float(g2 & 0xffff0000u);
          du0[e] = gv.y * carry0;
          du1[e] = gv.y * carry1;
          const float d0 = (f0[e] - __uint_as_float(h2 << 16)) * carry0 * gv.z;
          const float d1 = (f1[e] - __uint_as_float(h2 & 0xffff0000u)) * carry1 * gv.z;
          ds[e] = d0 + d1;
        }
        // du takes the value tile's place: the tile leaves as one bulk store
        const uint4 p0 = pack8(du0), p1 = pack8(du1);
        *slotA = sw ? p1 : p0;
        *slotB = sw ? p0 : p1;
        // the block's 8 dalpha terms summed over the segment's lanes: halving rounds keep the
        // upper half of the values in the lanes with the round's mask bit set
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const bool up = (lane & m1) != 0;
          const float send = up ? ds[j] : ds[j + 4];
          const float keep = up ? ds[j + 4] : ds[j];
          ds[j] = keep + __shfl_xor_sync(0xffffffffu, send, m1);
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const bool up = (lane & m2) != 0;
          const float send = up ? ds[j] : ds[j + 2];
          const float keep = up ? ds[j + 2] : ds[j];
          ds[j] = keep + __shfl_xor_sync(0xffffffffu, send, m2);
        }
        {
          const bool up = (lane & m3) != 0;
          const float send = up ? ds[0] : ds[1];
          const float keep = up ? ds[1] : ds[0];
          ds[0] = keep + __shfl_xor_sync(0xffffffffu, send, m3);
        }
        for (int o = m3 >> 1; o > 0; o >>= 1) ds[0] += __shfl_xor_sync(0xffffffffu, ds[0], o);
        if (canon) part[segid * kTT + 8 * k + tloc] = ds[0];
      }
      if (ti.t0 == 0) {
        const __nv_bfloat162 gi2 =
            __floats2bfloat162_rn(carry0 * (1.0f - grow[0].y), carry1 * (1.0f - grow[0].y));
        if (a.init_part == nullptr)
          reinterpret_cast<__nv_bfloat162*>(a.grad_inits + rowbase * D)[tid] = gi2;
        else
          reinterpret_cast<float2*>(a.init_part + rowbase * D)[tid] =
              make_float2(__low2float(gi2), __high2float(gi2));
      }
      fence_proxy_async_smem();
      named_barrier(1, ncons);  // the du tile and the segment sums are complete
      if (tid == 0) {
        tma_store_2d(&tm_du, sb, ti.t0, ti.b * a.F + ti.h * (D + Da));  // columns beyond T are clipped
        tma_store_commit();
      }
      // dlogit of each (group, token): the group's segment sums in a fixed order
#pragma unroll
      for (int qi = 0; qi < 2; ++qi) {
        const int q = tid + qi * ncons;
        if (q < Da * kTT) {
          const int g = q / kTT, t = q % kTT;
          float sum = 0.f;
          for (int j = 0; j < spg; ++j) sum += part[(g * spg + j) * kTT + t];
          if (t < ti.tlen) {
            a.grad_combined[((long long)ti.b * a.F + ti.h * (D + Da) + D + g) * a.T + ti.t0 + t] =
                __float2bfloat16_rn(sum);
            bias_q[qi] += sum;
          }
        }
      }
      fence_proxy_async_smem();  // order this thread's writes into the stage before the next TMA fill
      if (tid == 0) tma_store_wait_read0();  // the du tile has left the stage
      named_barrier(1, ncons);   // every segment sum has been read (`part` is rewritten next chunk)
      if (lane == 0) mbar_arrive(&empty[st]);  // the stage is free

      if (ti.j == 0) {  // row done: this row's logit-bias partials, a fixed-order sum per group
#pragma unroll
        for (int qi = 0; qi < 2; ++qi) {
          const int q = tid + qi * ncons;
          if (q < Da * kTT) bsum[q] = bias_q[qi];
        }
        named_barrier(1, ncons);
        if (tid < Da) {
          float t = 0.f;
          for (int j = 0; j < kTT; ++j) t += bsum[tid * kTT + j];
          a.bias_part[rowbase * Da + tid] = t;
        }
        if (a.init_part != nullptr) {
          // shared initial state: the row that completes its head's batch sums the head's per-row
          // gradients in batch order (each thread its two channels)
          __threadfence();
          named_barrier(1, ncons);
          if (tid == 0) init_last = atomicAdd(&a.init_cnt[ti.h], 1u) == (unsigned int)(a.B - 1) ? 1 : 0;
          named_barrier(1, ncons);
          if (init_last) {
            __threadfence();
            float s0 = 0.f, s1 = 0.f;
#pragma unroll 8
            for (int bb = 0; bb < a.B; ++bb) {
              const float2 v = __ldcg(reinterpret_cast<const float2*>(a.init_part + ((long long)bb * a.H + ti.h) * D) + tid);
              s0 += v.x;
              s1 += v.y;
            }
            reinterpret_cast<float2*>(a.grad_init_sum + (long long)ti.h * D)[tid] = make_float2(s0, s1);
          }
        }
        named_barrier(1, ncons);  // bsum (and init_last) are free again
      }
    }
    if (tid == 0) tma_store_wait0();
  }
  __syncthreads();
  // the CTA that finishes last adds the per-row logit-bias partials, batch by batch in order
  __shared__ int last_cta;
  if (tid == 0) last_cta = finish_launch_last(a.ws, gridDim.x) ? 1 : 0;
  __syncthreads();
  if (last_cta) {
    const int n = a.H * Da;
    for (int idx = tid; idx < n; idx += blockDim.x) {
      float sum = 0.f;
      for (int b = 0; b < a.B; ++b) sum += __ldcg(a.bias_part + (long long)b * n + idx);
      if (a.bias_overwrite) a.grad_bias[idx] = sum;
      else a.grad_bias[idx] += sum;
    }
  }
}

}  // namespace ltvqkv
