// Row-streaming, TMA-fed bf16 scan kernels for the exact production layout (included by
// ltvqkv_scan.cu): combined / grad_combined are the transposed view of a contiguous [B, F, T]
// buffer, so one 2-D tensor map [B*F rows, T columns] addresses every head's value and logit rows.
//
// A persistent CTA owns whole (batch, head) rows, drawn from a ticket counter, and walks each row
// chunk by chunk (64 tokens; forward in time order, backward in reverse). The carry never leaves
// registers: thread (c, s) holds channel c, tokens [32 s, 32 s + 32) of a chunk, and the two
// threads of a channel are adjacent lanes that hand the carry over with one shuffle — no
// look-back, no inter-CTA communication, results fixed by construction. One producer warp
// streams the row's chunks into a ring of shared-memory stages with cp.async.bulk.tensor
// (mbarrier full/empty pairs), so the next chunks' loads are in flight while the consumers scan
// the current one; forward outputs leave as one contiguous 16 KB bulk store per chunk, backward
// gradients as 16-byte vector stores. Chosen when there are enough rows to fill the GPU
// (B * heads >= 2 * SMs); fewer, longer rows take the chunk-parallel look-back kernels.
// Every wait is bounded (2 s) and reports LTVQKV_ERR_TIMEOUT through the workspace.
#pragma once

namespace ltvqkv {

constexpr int kTmaFwdStages = 4;
constexpr int kTmaBwdStages = 3;
constexpr int kLogitBoxBwd = 72;  // 64 tokens + the next chunk's first, padded to 16 bytes

struct TmaFwdArgs {
  const __nv_bfloat16* inits;
  const float* logit_bias;
  __nv_bfloat16* out[3];
  int B, T, NH, NKVH, Da, r, D, H, F, nchunks, nrows, use_sigmoid;
  WorkspaceHeader* ws;
};

struct TmaBwdArgs {
  const __nv_bfloat16* inits;
  const float* logit_bias;
  __nv_bfloat16* grad_combined;
  __nv_bfloat16* grad_inits;
  float* bias_part;  // [B][H][Da]: one partial per row
  int B, T, NH, NKVH, Da, r, D, H, F, nchunks, nrows, use_sigmoid;
  WorkspaceHeader* ws;
};

__host__ __device__ inline int tma_fwd_stage_bytes(int D, int Da) { return ((D + Da) * 128 + 1023) / 1024 * 1024; }
__host__ __device__ inline int tma_bwd_logit_bytes(int Da) { return (Da * kLogitBoxBwd * 2 + 127) / 128 * 128; }
__host__ __device__ inline int tma_bwd_stage_bytes(int D, int Da) {
  return (D * 128 + tma_bwd_logit_bytes(Da) + 2 * kFastTT * D * 2 + 1023) / 1024 * 1024;
}
inline size_t tma_fwd_smem_bytes(int D, int Da) {
  return 1024 + (size_t)kTmaFwdStages * tma_fwd_stage_bytes(D, Da) + 2 * (size_t)kFastTT * D * 2 +
         sizeof(float) * (size_t)Da * kFastTT + 16 * kTmaFwdStages + 64;
}
inline size_t tma_bwd_smem_bytes(int D, int Da) {
  return 1024 + (size_t)kTmaBwdStages * tma_bwd_stage_bytes(D, Da) +
         sizeof(float) * ((size_t)kFastTT * D + (size_t)Da * (kFastTT + 1) + (size_t)Da * kFastTT) +
         16 * kTmaBwdStages + 64;
}

// 16-byte chunk `chunk` of row `row` in a 128-byte-swizzled tile of 64 bf16 per row.
LTVQKV_DEVICE const uint4* sw128_chunk(const uint8_t* tile, int row, int chunk) {
  return reinterpret_cast<const uint4*>(tile + row * 128 + ((chunk ^ (row & 7)) << 4));
}

// ------------------------------------------------------------------------------------------
// Forward
// ------------------------------------------------------------------------------------------
template <int kMaxThreads>
__global__ void __launch_bounds__(kMaxThreads, 2)
    scan_fwd_rows_kernel(const __grid_constant__ CUtensorMap tm_u, const __grid_constant__ CUtensorMap tm_l,
                         const TmaFwdArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int D = a.D, Da = a.Da;
  const int ncons = 2 * D;
  const int sbytes = tma_fwd_stage_bytes(D, Da);
  uint8_t* stages = base;
  __nv_bfloat16* out_s = reinterpret_cast<__nv_bfloat16*>(stages + kTmaFwdStages * sbytes);  // [2][64][D]
  float* alpha_s = reinterpret_cast<float*>(out_s + 2 * kFastTT * D);                       // [Da][64]
  int* tile_slot = reinterpret_cast<int*>(alpha_s + Da * kFastTT);                          // [stages]
  uint64_t* full = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(tile_slot + kTmaFwdStages) + 7) & ~uintptr_t(7));
  uint64_t* empty = full + kTmaFwdStages;
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kTmaFwdStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], ncons / 32);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
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
        for (int j = 0; j < nch; ++j, ++i) {
          const int st = i % kTmaFwdStages;
          const uint32_t ph = (uint32_t)(i / kTmaFwdStages) & 1u;
          if (!mbar_wait(&empty[st], ph ^ 1u, &abort_flag, a.ws, 0x7101)) { ok = false; break; }
          if (row < 0) {
            tile_slot[st] = -1;
            mbar_arrive(&full[st]);
            ok = false;
            break;
          }
          tile_slot[st] = row * a.nchunks + j;
          const int b = row / a.H, h = row % a.H;
          const int frow = b * a.F + h * (D + Da);
          uint8_t* sb = stages + st * sbytes;
          mbar_arrive_expect_tx(&full[st], (uint32_t)((D + Da) * 128));
          tma_load_2d(sb, &tm_u, &full[st], j * kFastTT, frow);
          tma_load_2d(sb + D * 128, &tm_l, &full[st], j * kFastTT, frow + D);
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- consumers ----------------
    const int c = tid >> 1, s = tid & 1;
    int buf = 0;
    float E = 0.f;  // row carry (h at the end of the previous chunk), held by the s == 1 lane
    for (int i = 0;; ++i) {
      const int st = i % kTmaFwdStages;
      const uint32_t ph = (uint32_t)(i / kTmaFwdStages) & 1u;
      if (!mbar_wait(&full[st], ph, &abort_flag, a.ws, 0x7102)) break;
      const int tile = tile_slot[st];
      if (tile < 0) break;
      const int row = tile / a.nchunks, j = tile % a.nchunks;
      const int b = row / a.H, h = row % a.H;
      const int t0 = j * kFastTT;
      const int tlen = min(kFastTT, a.T - t0);
      const uint8_t* sb = stages + st * sbytes;
      if (j == 0 && s == 1) E = __bfloat162float(a.inits[((long long)b * a.H + h) * D + c]);
      if (tid < Da * kFastTT) {
        const int g = tid / kFastTT, t = tid % kFastTT;
        float al = 0.f;
        if (t < tlen) {
          const float l = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(sb + D * 128 + g * 128)[t]) +
                          a.logit_bias[h * Da + g];
          al = a.use_sigmoid ? sigmoid_f32(l) : l;
        }
        alpha_s[tid] = al;
      }
      uint4 uv[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) uv[k] = *sw128_chunk(sb, c, 4 * s + k);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      // out_s[buf] was last read by the bulk store issued two chunks ago
      if (tid == 0) tma_store_wait_read1();
      named_barrier(1, ncons);

      const float* al_row = alpha_s + (c / a.r) * kFastTT + s * kFastSeg;
      float sa = 1.f, sx = 0.f;
      if (s == 0) {  // the first segment's aggregate carries the chunk's entry value to its partner
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float f[8];
          unpack8(uv[k], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float al = al_row[8 * k + e];
            sx = (1.0f - al) * sx + al * f[e];
            sa *= (1.0f - al);
          }
        }
      }
      const float a0 = __shfl_sync(0xffffffffu, sa, lane & ~1);
      const float x0 = __shfl_sync(0xffffffffu, sx, lane & ~1);
      const float Ec = __shfl_sync(0xffffffffu, E, lane | 1);
      float carry = (s == 0) ? Ec : a0 * Ec + x0;

      __nv_bfloat16* ob = out_s + buf * kFastTT * D;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float f[8];
        unpack8(uv[k], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float al = al_row[8 * k + e];
          carry = (1.0f - al) * carry + al * f[e];
          ob[(s * kFastSeg + 8 * k + e) * D + c] = __float2bfloat16_rn(carry);
        }
      }
      if (s == 1) E = carry;
      fence_proxy_async_smem();
      named_barrier(1, ncons);
      if (tid == 0) {
        int which, hloc, nheads;
        split_head(h, a.NH, a.NKVH, which, hloc, nheads);
        __nv_bfloat16* go = a.out[which] + (((long long)b * nheads + hloc) * a.T + t0) * D;
        bulk_store(go, ob, (uint32_t)(tlen * D * 2));
        tma_store_commit();
      }
      buf ^= 1;
    }
    if (tid == 0) tma_store_wait0();
  }
  __syncthreads();
  if (tid == 0) finish_launch(a.ws, gridDim.x);
}

// ------------------------------------------------------------------------------------------
// Backward
// ------------------------------------------------------------------------------------------
template <int kMaxThreads>
__global__ void __launch_bounds__(kMaxThreads, 1)
    scan_bwd_rows_kernel(const __grid_constant__ CUtensorMap tm_u, const __grid_constant__ CUtensorMap tm_l,
                         const __grid_constant__ CUtensorMap tm_gq, const __grid_constant__ CUtensorMap tm_gk,
                         const __grid_constant__ CUtensorMap tm_gv, const __grid_constant__ CUtensorMap tm_hq,
                         const __grid_constant__ CUtensorMap tm_hk, const __grid_constant__ CUtensorMap tm_hv,
                         const TmaBwdArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int D = a.D, Da = a.Da;
  const int ncons = 2 * D;
  const int sbytes = tma_bwd_stage_bytes(D, Da);
  const int lbytes = tma_bwd_logit_bytes(Da);
  uint8_t* stages = base;
  float* red = reinterpret_cast<float*>(stages + kTmaBwdStages * sbytes);  // [64][D]
  float* alpha_s = red + kFastTT * D;                                      // [Da][65]
  float* dlog_s = alpha_s + Da * (kFastTT + 1);                            // [Da][64]
  int* tile_slot = reinterpret_cast<int*>(dlog_s + Da * kFastTT);
  uint64_t* full = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(tile_slot + kTmaBwdStages) + 7) & ~uintptr_t(7));
  uint64_t* empty = full + kTmaBwdStages;
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kTmaBwdStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], ncons / 32);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const int ld_a = kFastTT + 1;

  if (warp == ncons / 32) {
    // ---------------- producer: rows from the ticket counter, chunks in reverse time order ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tm_u);
      tma_prefetch_desc(&tm_l);
      int i = 0;
      bool ok = true;
      while (ok) {
        int row = (int)draw_ticket(a.ws);
        if (row >= a.nrows) row = -1;
        const int nch = row < 0 ? 1 : a.nchunks;
        for (int q = 0; q < nch; ++q, ++i) {
          const int st = i % kTmaBwdStages;
          const uint32_t ph = (uint32_t)(i / kTmaBwdStages) & 1u;
          if (!mbar_wait(&empty[st], ph ^ 1u, &abort_flag, a.ws, 0x7201)) { ok = false; break; }
          if (row < 0) {
            tile_slot[st] = -1;
            mbar_arrive(&full[st]);
            ok = false;
            break;
          }
          const int j = a.nchunks - 1 - q;
          tile_slot[st] = row * a.nchunks + j;
          const int b = row / a.H, h = row % a.H;
          int which, hloc, nheads;
          split_head(h, a.NH, a.NKVH, which, hloc, nheads);
          const int frow = b * a.F + h * (D + Da);
          const int t0 = j * kFastTT;
          uint8_t* sb = stages + st * sbytes;
          uint8_t* sl = sb + D * 128;
          uint8_t* sg = sl + lbytes;
          uint8_t* shh = sg + kFastTT * D * 2;
          const CUtensorMap* mg = which == 0 ? &tm_gq : (which == 1 ? &tm_gk : &tm_gv);
          const CUtensorMap* mh = which == 0 ? &tm_hq : (which == 1 ? &tm_hk : &tm_hv);
          mbar_arrive_expect_tx(&full[st], (uint32_t)(D * 128 + Da * kLogitBoxBwd * 2 + 2 * kFastTT * D * 2));
          tma_load_2d(sb, &tm_u, &full[st], t0, frow);
          tma_load_2d(sl, &tm_l, &full[st], t0, frow + D);
          tma_load_4d(sg, mg, &full[st], 0, t0, hloc, b);
          tma_load_4d(shh, mh, &full[st], 0, t0 - 1, hloc, b);
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- consumers ----------------
    const int c = tid >> 1, s = tid & 1;
    const int gi = c / a.r;
    float Eg = 0.f;        // g^ at the first token of the previously processed chunk (s == 0 lane)
    float bias_acc = 0.f;  // lane 0 of warp g < Da: the row's logit-bias gradient of group g
    for (int i = 0;; ++i) {
      const int st = i % kTmaBwdStages;
      const uint32_t ph = (uint32_t)(i / kTmaBwdStages) & 1u;
      if (!mbar_wait(&full[st], ph, &abort_flag, a.ws, 0x7202)) break;
      const int tile = tile_slot[st];
      if (tile < 0) break;
      const int row = tile / a.nchunks, j = tile % a.nchunks;
      const int b = row / a.H, h = row % a.H;
      const int t0 = j * kFastTT;
      const int tlen = min(kFastTT, a.T - t0);
      if (j == a.nchunks - 1) {
        Eg = 0.f;
        bias_acc = 0.f;
      }
      const uint8_t* sb = stages + st * sbytes;
      const __nv_bfloat16* L_s = reinterpret_cast<const __nv_bfloat16*>(sb + D * 128);
      const __nv_bfloat16* G_s = reinterpret_cast<const __nv_bfloat16*>(sb + D * 128 + lbytes);
      const __nv_bfloat16* H_s = G_s + kFastTT * D;
      for (int q = tid; q < Da * ld_a; q += ncons) {
        const int g = q / ld_a, t = q % ld_a;
        float al = 0.f;
        if (t <= tlen && t0 + t < a.T) {
          const float l = __bfloat162float(L_s[g * kLogitBoxBwd + t]) + a.logit_bias[h * Da + g];
          al = a.use_sigmoid ? sigmoid_f32(l) : l;
        }
        alpha_s[q] = al;
      }
      uint4 uv[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) uv[k] = *sw128_chunk(sb, c, 4 * s + k);
      named_barrier(1, ncons);

      const float* al_row = alpha_s + gi * ld_a + s * kFastSeg;
      float sa = 1.f, sx = 0.f;
      if (s == 1) {  // the second segment's aggregate carries the chunk's exit value to its partner
#pragma unroll
        for (int t = kFastSeg - 1; t >= 0; --t) {
          const float an = 1.0f - al_row[t + 1];
          sx = an * sx + __bfloat162float(G_s[(s * kFastSeg + t) * D + c]);
          sa *= an;
        }
      }
      const float a1 = __shfl_sync(0xffffffffu, sa, lane | 1);
      const float x1 = __shfl_sync(0xffffffffu, sx, lane | 1);
      const float Ec = __shfl_sync(0xffffffffu, Eg, lane & ~1);

      // final reverse walk fused with the elementwise part (g^_t, du, dlogit terms)
      {
        const float init_c = __bfloat162float(a.inits[((long long)b * a.H + h) * D + c]);
        __nv_bfloat16* grow = a.grad_combined + (long long)(b * a.F + h * (D + Da) + c) * a.T + t0 + s * kFastSeg;
        float carry = (s == 1) ? Ec : a1 * Ec + x1;
#pragma unroll
        for (int k = 3; k >= 0; --k) {
          float f[8], du[8];
          unpack8(uv[k], f);
#pragma unroll
          for (int e = 7; e >= 0; --e) {
            const int t = 8 * k + e;
            const int tl = s * kFastSeg + t;
            carry = (1.0f - al_row[t + 1]) * carry + __bfloat162float(G_s[tl * D + c]);
            const float al = al_row[t];
            du[e] = al * carry;
            const float hp = (t0 + tl == 0) ? init_c : __bfloat162float(H_s[tl * D + c]);
            const float dalpha = (f[e] - hp) * carry;
            red[tl * D + c] = a.use_sigmoid ? dalpha * (al * (1.0f - al)) : dalpha;
          }
          if (s * kFastSeg + 8 * k < tlen) *reinterpret_cast<uint4*>(grow + 8 * k) = pack8(du);
        }
        if (s == 0) Eg = carry;
        if (t0 == 0 && s == 0)
          a.grad_inits[((long long)b * a.H + h) * D + c] = __float2bfloat16_rn(carry * (1.0f - al_row[0]));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      named_barrier(1, ncons);

      {
        const int tpg = a.r / 32;
        const int npairs = Da * kFastTT;
        const int pair = tid / tpg, part = tid % tpg;
        float sum = 0.f;
        if (pair < npairs) {
          const int g = pair / kFastTT, t = pair % kFastTT;
          const float* rrow = red + t * D + g * a.r + part * 32;
          const int rot = (t + part * (32 / tpg)) & 31;
#pragma unroll 8
          for (int q = 0; q < 32; ++q) sum += rrow[(q + rot) & 31];
        }
        for (int o = tpg >> 1; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (pair < npairs && part == 0) {
          const int g = pair / kFastTT, t = pair % kFastTT;
          dlog_s[g * kFastTT + t] = sum;
          if (t < tlen)
            a.grad_combined[(long long)(b * a.F + h * (D + Da) + D + g) * a.T + t0 + t] = __float2bfloat16_rn(sum);
        }
      }
      named_barrier(1, ncons);
      if (warp < Da) {
        float v = 0.f;
        for (int t = lane; t < kFastTT; t += 32) v += (t < tlen) ? dlog_s[warp * kFastTT + t] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        bias_acc += v;
        if (j == 0 && lane == 0) a.bias_part[((long long)b * a.H + h) * Da + warp] = bias_acc;
      }
    }
  }
  __syncthreads();
  if (tid == 0) finish_launch(a.ws, gridDim.x);
}

}  // namespace ltvqkv
