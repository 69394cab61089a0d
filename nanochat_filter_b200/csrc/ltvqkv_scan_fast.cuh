// Vectorised bf16 scan kernels for the production layouts (included by ltvqkv_scan.cu).
//
// Layouts: combined / grad_combined are the transposed view of a [B, F, T] buffer (t unit
// stride), the saved outputs and their gradients are [B, heads, T, D] with d unit stride (any
// b/h/t strides, so the attention layer's transposed q/k gradients qualify).
//
// A CTA owns one (b, head, 64-token chunk) tile with 2*D threads: thread (c, s) holds channel c
// and tokens [32 s, 32 s + 32) of the chunk. t-contiguous rows are read and written straight
// from/to registers with 16-byte vector accesses (4 per thread); d-contiguous tiles pass through
// shared memory ([64][D] bf16, one contiguous 16 KB block per tile in global memory). The two
// 32-token segments of a channel are adjacent lanes and combine with one shuffle. Chunk carries:
// the forward composes them in a separate pass between two tile passes (no waits between CTAs);
// the backward uses the anchored look-back of the generic kernels. Both associations are fixed,
// so results are deterministic.
#pragma once

namespace ltvqkv {

constexpr int kFastTT = 64;   // tokens per tile
constexpr int kFastSeg = 32;  // tokens per thread
constexpr int kFastMaxDa = 8;
// CTAs per SM targeted for 256-thread tiles (head dim <= 128) by the register cap: the backward
// and the forward's aggregate pass fit 6 without spills (40 and 38 registers), the forward's
// apply pass 5 (48 registers, one 4-byte spill)
constexpr int kFastFwdAggMinBlocks256 = 6;
constexpr int kFastFwdMinBlocks256 = 5;
constexpr int kFastBwdMinBlocks256 = 6;

LTVQKV_DEVICE void unpack8(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(p[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

LTVQKV_DEVICE uint4 pack8(const float (&f)[8]) {
  uint4 v;
  __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

struct FastFwdArgs {
  const __nv_bfloat16* combined;
  long long sc_b, sc_e;  // sc_t == 1
  const __nv_bfloat16* inits;
  const float* logit_bias;
  __nv_bfloat16* out[3];
  int B, T, NH, NKVH, Da, r, D, H, nchunks, use_sigmoid;
  float* aggA;   // [tiles][Da] decay product of each tile
  float* aggX;   // [tiles][D] zero-carry scan end of each tile
  float* inclX;  // [tiles][D] state entering each tile (written by the carry pass)
};

struct FastBwdArgs {
  const __nv_bfloat16* combined;
  long long sc_b, sc_e;
  const __nv_bfloat16* inits;
  const float* logit_bias;
  const __nv_bfloat16* h[3];
  long long hs[3][3];  // b, head, t strides (d stride 1)
  const __nv_bfloat16* gh[3];
  long long gs[3][3];
  __nv_bfloat16* grad_combined;
  long long gc_b, gc_e;
  __nv_bfloat16* grad_inits;
  float* bias_part;
  int B, T, NH, NKVH, Da, r, D, H, nchunks, use_sigmoid;
  WorkspaceHeader* ws;
  unsigned int* flags;
  float* aggA;
  float* aggX;
  float* inclX;
};

// Warp 0 waits for the flags of chunk positions [m, j) of row bh (positions count from the end
// when `reverse`), one lane per flag so the polls overlap; returns (to every lane of warp 0)
// whether any wait gave up. j - m <= kAnchorStride <= 32.
LTVQKV_DEVICE bool warp_wait_flags(const unsigned int* flags, int BH, int bh, int nchunks, int m, int j, bool reverse,
                                   unsigned int epoch, WorkspaceHeader* ws, int lane) {
  bool timed_out = false;
  const int k = m + lane;
  if (k < j) {
    const int chunk = reverse ? nchunks - 1 - k : k;
    wait_flag(&flags[(long long)chunk * BH + bh], epoch, ws, &timed_out);
  }
  return __any_sync(0xffffffffu, timed_out);
}

// Carry-in of a tile: the anchor's inclusive carry composed with the aggregates of the positions
// between, in position order. All payload loads are issued before the composition.
LTVQKV_DEVICE float compose_carry(const float* inclX, const float* aggA, const float* aggX, int BH, int bh,
                                  int nchunks, int m, int j, bool reverse, int D, int Da, int c, int gi) {
  float X[kAnchorStride], A[kAnchorStride];
#pragma unroll
  for (int q = 0; q < kAnchorStride; ++q) {
    const int k = m + q;
    const long long p = (long long)(reverse ? nchunks - 1 - k : k) * BH + bh;
    X[q] = 0.f;
    A[q] = 1.f;
    if (q == 0) {
      X[q] = ld_cg_f32(&inclX[p * D + c]);
    } else if (k < j) {
      X[q] = ld_cg_f32(&aggX[p * D + c]);
      A[q] = ld_cg_f32(&aggA[p * Da + gi]);
    }
  }
  float E = X[0];
#pragma unroll
  for (int q = 1; q < kAnchorStride; ++q)
    if (m + q < j) E = A[q] * E + X[q];
  return E;
}

// ------------------------------------------------------------------------------------------
// Forward: three passes, no look-back. (1) every tile's aggregates (the decay product of each
// group and the zero-carry scan end of each channel), all tiles in parallel; (2) per (row,
// channel), the carries entering every tile, composed in tile order; (3) every tile again from its
// carry, writing the outputs. Nothing waits on another CTA; the value rows are read twice (the
// second time mostly from L2) instead of once, which costs less than the look-back chain did.
// ------------------------------------------------------------------------------------------

// Tile geometry shared by passes 1 and 3 (tile = blockIdx.x = chunk * B * H + row).
struct FastTile {
  int j, bh, b, h, t0, tlen, head_col;
};
LTVQKV_DEVICE FastTile fast_tile(const FastFwdArgs& a) {
  FastTile t;
  const int BH = a.B * a.H;
  t.j = (int)(blockIdx.x / BH);
  t.bh = (int)(blockIdx.x % BH);
  t.b = t.bh / a.H;
  t.h = t.bh % a.H;
  t.t0 = t.j * kFastTT;
  t.tlen = min(kFastTT, a.T - t.t0);
  t.head_col = t.h * (a.D + a.Da);
  return t;
}

// Gates of the tile (identity beyond T) into alpha_s [Da][64], and this thread's value-row segment.
LTVQKV_DEVICE void fast_fwd_load(const FastFwdArgs& a, const FastTile& t, float* alpha_s, int c, int s,
                                 uint4 (&uv)[4]) {
  const __nv_bfloat16* cb = a.combined + (long long)t.b * a.sc_b;
  for (int i = threadIdx.x; i < a.Da * kFastTT; i += blockDim.x) {
    const int gi = i / kFastTT, tt = i % kFastTT;
    float al = 0.f;
    if (tt < t.tlen) {
      const float l = __bfloat162float(cb[(long long)(t.head_col + a.D + gi) * a.sc_e + t.t0 + tt]) +
                      a.logit_bias[t.h * a.Da + gi];
      al = a.use_sigmoid ? sigmoid_f32(l) : l;
    }
    alpha_s[i] = al;
  }
  const __nv_bfloat16* urow = cb + (long long)(t.head_col + c) * a.sc_e + t.t0 + s * kFastSeg;
#pragma unroll
  for (int k = 0; k < 4; ++k)
    uv[k] = (s * kFastSeg + 8 * k < t.tlen) ? __ldg(reinterpret_cast<const uint4*>(urow + 8 * k))
                                            : make_uint4(0, 0, 0, 0);
}

// Zero-carry scan of this thread's segment: sa = product of (1 - alpha), sx = end state.
LTVQKV_DEVICE void fast_fwd_local(const float* al_row, const uint4 (&uv)[4], float& sa, float& sx) {
  sa = 1.f;
  sx = 0.f;
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

template <int kThreads, int kMinBlocks>
__global__ void __launch_bounds__(kThreads, kMinBlocks) scan_fwd_agg_kernel(FastFwdArgs a) {
  __shared__ float alpha_s[kFastMaxDa * kFastTT];
  const int tid = threadIdx.x, lane = tid & 31;
  const int c = tid >> 1, s = tid & 1;
  const FastTile t = fast_tile(a);
  uint4 uv[4];
  fast_fwd_load(a, t, alpha_s, c, s, uv);
  __syncthreads();
  float sa, sx;
  fast_fwd_local(alpha_s + (c / a.r) * kFastTT + s * kFastSeg, uv, sa, sx);
  // segment 0 lives in the even lane of each pair
  const float a0 = __shfl_sync(0xffffffffu, sa, lane & ~1);
  const float x0 = __shfl_sync(0xffffffffu, sx, lane & ~1);
  if (s == 1) {
    a.aggX[(long long)blockIdx.x * a.D + c] = sa * x0 + sx;
    if (c % a.r == 0) a.aggA[(long long)blockIdx.x * a.Da + c / a.r] = a0 * sa;
  }
}

// One thread per (row, channel): the state entering each tile of the row, from the initial state
// and the tiles' aggregates in tile order (16 tiles' aggregates in flight at a time).
__global__ void __launch_bounds__(256) scan_fwd_carry_kernel(FastFwdArgs a) {
  const int BH = a.B * a.H;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)BH * a.D) return;
  const int bh = (int)(i / a.D), c = (int)(i % a.D), gi = c / a.r;
  float E = __bfloat162float(a.inits[(long long)bh * a.D + c]);
  for (int j0 = 0; j0 < a.nchunks; j0 += 16) {
    float A[16], X[16];
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      const long long tile = (long long)(j0 + q) * BH + bh;
      A[q] = 1.f;
      X[q] = 0.f;
      if (j0 + q < a.nchunks) {
        A[q] = ld_cg_f32(&a.aggA[tile * a.Da + gi]);
        X[q] = ld_cg_f32(&a.aggX[tile * a.D + c]);
      }
    }
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      if (j0 + q < a.nchunks) {
        a.inclX[((long long)(j0 + q) * BH + bh) * a.D + c] = E;  // carry into tile j0 + q
        E = A[q] * E + X[q];
      }
    }
  }
}

template <int kThreads, int kMinBlocks>
__global__ void __launch_bounds__(kThreads, kMinBlocks) scan_fwd_apply_kernel(FastFwdArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int D = a.D;
  __nv_bfloat16* out_s = reinterpret_cast<__nv_bfloat16*>(smem_raw);                 // [64][D]
  float* alpha_s = reinterpret_cast<float*>(smem_raw + (size_t)kFastTT * D * 2);      // [Da][64]
  const int tid = threadIdx.x, lane = tid & 31;
  const int c = tid >> 1, s = tid & 1;
  const FastTile t = fast_tile(a);
  uint4 uv[4];
  fast_fwd_load(a, t, alpha_s, c, s, uv);
  const float E_in = a.inclX[(long long)blockIdx.x * D + c];
  __syncthreads();
  const float* al_row = alpha_s + (c / a.r) * kFastTT + s * kFastSeg;
  float sa, sx;
  fast_fwd_local(al_row, uv, sa, sx);
  const float a0 = __shfl_sync(0xffffffffu, sa, lane & ~1);
  const float x0 = __shfl_sync(0xffffffffu, sx, lane & ~1);
  float carry = (s == 0) ? E_in : a0 * E_in + x0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float f[8];
    unpack8(uv[k], f);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float al = al_row[8 * k + e];
      carry = (1.0f - al) * carry + al * f[e];
      out_s[(s * kFastSeg + 8 * k + e) * D + c] = __float2bfloat16_rn(carry);
    }
  }
  __syncthreads();

  int which, hloc, nheads;
  split_head(t.h, a.NH, a.NKVH, which, hloc, nheads);
  uint4* go = reinterpret_cast<uint4*>(a.out[which] + (((long long)t.b * nheads + hloc) * a.T + t.t0) * D);
  const uint4* so = reinterpret_cast<const uint4*>(out_s);
  const int n16 = t.tlen * D / 8;
  for (int i = tid; i < n16; i += blockDim.x) go[i] = so[i];
}

// ------------------------------------------------------------------------------------------
// Backward
// ------------------------------------------------------------------------------------------
template <int kThreads, int kMinBlocks>
__global__ void __launch_bounds__(kThreads, kMinBlocks) scan_bwd_fast_kernel(FastBwdArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int D = a.D, Da = a.Da;
  __nv_bfloat16* G_s = reinterpret_cast<__nv_bfloat16*>(smem_raw);                        // [64][D] upstream grad
  __nv_bfloat16* H_s = G_s + kFastTT * D;                                                 // [64][D] h_{t-1}
  float* part = reinterpret_cast<float*>(H_s + kFastTT * D);                              // [D/16][64] warp sums
  float* alpha_s = part + (D / 16) * kFastTT;                                             // [Da][65]
  float* dlog_s = alpha_s + Da * (kFastTT + 1);                                           // [Da][64]
  float* shE = dlog_s + Da * kFastTT;                                                     // [D]
  __shared__ unsigned int sh_tile, sh_epoch;
  __shared__ int sh_timeout;

  const int tid = threadIdx.x, lane = tid & 31;
  const int c = tid >> 1, s = tid & 1;
  if (tid == 0) {
    sh_tile = draw_ticket(a.ws);
    sh_epoch = *((volatile unsigned int*)&a.ws->epoch) & 0x3FFFFFFFu;
  }
  __syncthreads();
  const unsigned int epoch = sh_epoch;
  const int BH = a.B * a.H;
  const int j = a.nchunks - 1 - (int)(sh_tile / BH);
  const int bh = (int)(sh_tile % BH);
  const int b = bh / a.H, h = bh % a.H;
  const int t0 = j * kFastTT;
  const int tlen = min(kFastTT, a.T - t0);
  int which, hloc, nheads;
  split_head(h, a.NH, a.NKVH, which, hloc, nheads);
  const __nv_bfloat16* cb = a.combined + (long long)b * a.sc_b;
  const int head_col = h * (D + Da);
  const int ld_a = kFastTT + 1;

  // gates alpha_{t0 + t}, t = 0..tlen (the first token of the next chunk included; 0 beyond T)
  for (int i = tid; i < Da * ld_a; i += blockDim.x) {
    const int gi = i / ld_a, t = i % ld_a;
    float al = 0.f;
    if (t <= tlen && t0 + t < a.T) {
      const float l = __bfloat162float(cb[(long long)(head_col + D + gi) * a.sc_e + t0 + t]) + a.logit_bias[h * Da + gi];
      al = a.use_sigmoid ? sigmoid_f32(l) : l;
    }
    alpha_s[i] = al;
  }
  // upstream gradient rows and h_{t-1} rows into shared memory (16-byte vectors)
  {
    const int vpr = D / 8;  // vectors per row
    const long long* gs = a.gs[which];
    const long long* hs = a.hs[which];
    const __nv_bfloat16* gb = a.gh[which] + (long long)b * gs[0] + (long long)hloc * gs[1];
    const __nv_bfloat16* hb = a.h[which] + (long long)b * hs[0] + (long long)hloc * hs[1];
    const __nv_bfloat16* ib = a.inits + ((long long)b * a.H + h) * D;
    uint4* Gv = reinterpret_cast<uint4*>(G_s);
    uint4* Hv = reinterpret_cast<uint4*>(H_s);
    for (int i = tid; i < kFastTT * vpr; i += blockDim.x) {
      const int t = i / vpr, ch = i % vpr;
      uint4 gv = make_uint4(0, 0, 0, 0), hv = make_uint4(0, 0, 0, 0);
      if (t < tlen) {
        gv = __ldg(reinterpret_cast<const uint4*>(gb + (long long)(t0 + t) * gs[2]) + ch);
        const int tp = t0 + t - 1;
        hv = tp >= 0 ? __ldg(reinterpret_cast<const uint4*>(hb + (long long)tp * hs[2]) + ch)
                     : __ldg(reinterpret_cast<const uint4*>(ib) + ch);
      }
      Gv[i] = gv;
      Hv[i] = hv;
    }
  }
  const __nv_bfloat16* urow = cb + (long long)(head_col + c) * a.sc_e + t0 + s * kFastSeg;
  auto load_u = [&](int k) {  // the value row's 8 tokens of block k of this thread's segment
    return (s * kFastSeg + 8 * k < tlen) ? __ldg(reinterpret_cast<const uint4*>(urow + 8 * k))
                                         : make_uint4(0, 0, 0, 0);
  };
  uint4 uv_next = load_u(3);  // in flight during the local scan and the look-back
  __syncthreads();

  const int gi = c / a.r;
  const float* al_row = alpha_s + gi * ld_a + s * kFastSeg;  // al_row[t] = alpha at local token s*32 + t
  // reverse local scan of the segment (zero carry from the right)
  float sa = 1.f, sx = 0.f;
#pragma unroll
  for (int t = kFastSeg - 1; t >= 0; --t) {
    const float an = 1.0f - al_row[t + 1];
    sx = an * sx + __bfloat162float(G_s[(s * kFastSeg + t) * D + c]);
    sa *= an;
  }
  // segment 1 (odd lane) lies to the right of segment 0
  const float a1 = __shfl_sync(0xffffffffu, sa, lane | 1);
  const float x1 = __shfl_sync(0xffffffffu, sx, lane | 1);
  const float tileA = sa * a1, tileX = sa * x1 + sx;  // meaningful on s == 0

  const long long tile_idx = (long long)j * BH + bh;
  const int rj = a.nchunks - 1 - j;
  const bool is_anchor = (rj % kAnchorStride) == 0;
  if (rj == 0) {
    if (s == 0) shE[c] = 0.f;
  } else {
    if (!is_anchor) {
      if (s == 0) {
        a.aggX[tile_idx * D + c] = tileX;
        if (c % a.r == 0) a.aggA[tile_idx * Da + gi] = tileA;
      }
      __syncthreads();  // thread 0's release store of the flag publishes the block's payload
      if (tid == 0) st_release_u32(&a.flags[tile_idx], (epoch << 2) | kFlagAgg);
    }
    const int mr = (rj - 1) / kAnchorStride * kAnchorStride;
    if (tid < 32) {
      const bool to = warp_wait_flags(a.flags, BH, bh, a.nchunks, mr, rj, true, epoch, a.ws, lane);
      if (tid == 0) sh_timeout = to;
    }
    __syncthreads();
    if (s == 0)
      shE[c] = sh_timeout ? 0.f
                          : compose_carry(a.inclX, a.aggA, a.aggX, BH, bh, a.nchunks, mr, rj, true, D, Da, c, gi);
  }
  if (is_anchor) {
    if (s == 0) a.inclX[tile_idx * D + c] = tileA * shE[c] + tileX;
    __syncthreads();  // thread 0's release store of the flag publishes the block's payload
    if (tid == 0) st_release_u32(&a.flags[tile_idx], (epoch << 2) | kFlagIncl);
  }
  __syncthreads();

  // final reverse walk fused with the elementwise part: g^_t, du (t-contiguous row of
  // grad_combined) and the dlogit terms, one 8-token block at a time from the end of the segment
  {
    __nv_bfloat16* grow =
        a.grad_combined + (long long)b * a.gc_b + (long long)(head_col + c) * a.gc_e + t0 + s * kFastSeg;
    float carry = (s == 1) ? shE[c] : a1 * shE[c] + x1;
    const int wq = tid >> 5;  // this warp's 16 channels
    // after the butterfly, lane l holds the warp's sum of token (l >> 2) & 7 of the block
    const int tloc = ((lane & 16) ? 4 : 0) + ((lane & 8) ? 2 : 0) + ((lane & 4) ? 1 : 0);
#pragma unroll 1
    for (int k = 3; k >= 0; --k) {
      float f[8], du[8], ds[8];
      unpack8(uv_next, f);
      if (k > 0) uv_next = load_u(k - 1);  // the next block's row, in flight during this block
#pragma unroll
      for (int e = 7; e >= 0; --e) {
        const int t = 8 * k + e;
        const int tl = s * kFastSeg + t;
        carry = (1.0f - al_row[t + 1]) * carry + __bfloat162float(G_s[tl * D + c]);
        const float al = al_row[t];
        du[e] = al * carry;
        const float hp = __bfloat162float(H_s[tl * D + c]);
        const float dalpha = (f[e] - hp) * carry;
        ds[e] = a.use_sigmoid ? dalpha * (al * (1.0f - al)) : dalpha;
      }
      if (s * kFastSeg + 8 * k < tlen) *reinterpret_cast<uint4*>(grow + 8 * k) = pack8(du);
      // the block's 8 dlogit terms summed over the warp's 16 channels of this segment (lanes of
      // equal bit 0): halving rounds over lane bits 4, 3, 2 keep the upper half of the values in
      // the lanes with the bit set, then a plain round over bit 1
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const bool up = (lane & 16) != 0;
        const float send = up ? ds[jj] : ds[jj + 4];
        const float keep = up ? ds[jj + 4] : ds[jj];
        ds[jj] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
      }
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const bool up = (lane & 8) != 0;
        const float send = up ? ds[jj] : ds[jj + 2];
        const float keep = up ? ds[jj + 2] : ds[jj];
        ds[jj] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
      }
      {
        const bool up = (lane & 4) != 0;
        const float send = up ? ds[0] : ds[1];
        const float keep = up ? ds[1] : ds[0];
        ds[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
      }
      ds[0] += __shfl_xor_sync(0xffffffffu, ds[0], 2);
      if ((lane & 2) == 0) part[wq * kFastTT + s * kFastSeg + 8 * k + tloc] = ds[0];
    }
    if (t0 == 0 && s == 0)
      a.grad_inits[((long long)b * a.H + h) * D + c] = __float2bfloat16_rn(carry * (1.0f - al_row[0]));
  }
  __syncthreads();

  // dlogit of each (group, token): the group's r / 16 warp sums in a fixed order
  for (int q = tid; q < Da * kFastTT; q += blockDim.x) {
    const int g = q / kFastTT, t = q % kFastTT;
    const int wpg = a.r / 16;
    float sum = 0.f;
    for (int w = 0; w < wpg; ++w) sum += part[(g * wpg + w) * kFastTT + t];
    dlog_s[g * kFastTT + t] = sum;
    if (t < tlen)
      a.grad_combined[(long long)b * a.gc_b + (long long)(head_col + D + g) * a.gc_e + t0 + t] = __float2bfloat16_rn(sum);
  }
  __syncthreads();
  // per-tile bias partial: warp g sums the tile's dlogit of group g in a fixed tree order
  {
    const int warp = tid >> 5;
    for (int g = warp; g < Da; g += blockDim.x / 32) {
      float v = 0.f;
      for (int t = lane; t < kFastTT; t += 32) v += (t < tlen) ? dlog_s[g * kFastTT + t] : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) a.bias_part[(((long long)b * a.nchunks + j) * a.H + h) * Da + g] = v;
    }
  }

  if (tid == 0) finish_launch(a.ws, gridDim.x);
}

inline size_t fast_fwd_smem_bytes(int D, int Da) {
  return (size_t)kFastTT * D * 2 + sizeof(float) * (size_t)Da * kFastTT;
}
inline size_t fast_bwd_smem_bytes(int D, int Da) {
  return (size_t)kFastTT * D * 2 * 2 + sizeof(float) * ((size_t)(D / 16) * kFastTT + (size_t)Da * (kFastTT + 1) +
                                                         (size_t)Da * kFastTT + D);
}

inline ScanGeometry fast_geometry(int B, int T, int NH, int NKVH, int Da, int r) {
  ScanGeometry g;
  g.B = B; g.T = T; g.NH = NH; g.NKVH = NKVH; g.Da = Da; g.r = r;
  g.D = Da * r; g.H = NH + 2 * NKVH; g.F = g.H * (g.D + Da);
  g.P = 2; g.L = kFastSeg; g.TT = kFastTT; g.nthreads = 2 * g.D;
  g.nchunks = T > 0 ? (T + kFastTT - 1) / kFastTT : 0;
  return g;
}

inline bool aligned16p(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Shape conditions shared by the fast kernels.
inline bool fast_shape_ok(int T, int Da, int r) {
  const int D = Da * r;
  return T % 8 == 0 && D % 32 == 0 && D >= 32 && D <= 256 && Da <= kFastMaxDa;
}

}  // namespace ltvqkv
