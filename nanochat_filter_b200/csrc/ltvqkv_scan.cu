// Filter scan (EWMA with time-varying gain), forward and backward, for sm_100a.
//
// Semantics follow the reference's sequential oracle
// (nanochat/ops/ltv_reference_ops.py:7-34 QuantizedStateUpdate, :37-124 the scan loop):
//   alpha_t = sigmoid(logit_t + bias)            (or logit_t + bias without sigmoid)
//   h_t     = (1 - alpha_t) * h_{t-1} + alpha_t * u_t     fp32 carry, output rounded to dtype
// backward:
//   g^_t    = g_t + (1 - alpha_{t+1}) * g^_{t+1}
//   du_t    = alpha_t * g^_t
//   dalpha  = g^_t * (u_t - h_{t-1})  with h_{t-1} the SAVED (dtype-rounded) output, inits at t=0
//   dlogit  = sum over the r channels of the group of dalpha * alpha*(1-alpha)
//   dinits  = g^_0 * (1 - alpha_0);  dbias = sum over b, t of dlogit.
//
// Design (B200): one CTA per (batch, head, T-chunk) tile holding all D channels of the head, so
// the per-group dlogit reduction stays inside the CTA (no atomics). Inside a tile, each channel
// is split into P segments of L steps; a thread scans its segment sequentially in registers,
// segments are composed as affine maps (a, x): carry_out = a * carry_in + x. Across T-chunks,
// carries propagate by look-back over a flag/payload array in the workspace: every 8th chunk is
// an anchor publishing its inclusive carry, the others publish aggregates; a tile composes its
// anchor's carry with the aggregates in between in chunk order (a fixed association, so results
// do not depend on timing). Tiles are drawn from a ticket counter in chunk-major order, so every
// tile waited on was scheduled earlier (no deadlock); each spin is bounded.
#include <algorithm>
#include <cstddef>
#include <mutex>

#include "ltvqkv_common.cuh"

namespace ltvqkv {

enum : unsigned int { kFlagNone = 0, kFlagAgg = 1, kFlagIncl = 2 };
constexpr int kAnchorStride = 8;  // chunks between look-back anchors

struct ScanGeometry {
  int B, T, NH, NKVH, Da, r, D, H, F;
  int TT;        // tokens per tile
  int nchunks;   // ceil(T / TT)
  int P;         // threads per channel
  int L;         // tokens per thread segment (TT = P * L)
  int nthreads;  // D * P
};

__host__ __device__ inline int pow2_floor(int v) {
  int p = 1;
  while (p * 2 <= v) p *= 2;
  return p;
}

// Tile geometry shared by host sizing and kernels. `budget` = target channel*token elements.
inline ScanGeometry make_geometry(int B, int T, int NH, int NKVH, int Da, int r, int budget) {
  ScanGeometry g;
  g.B = B; g.T = T; g.NH = NH; g.NKVH = NKVH; g.Da = Da; g.r = r;
  g.D = Da * r; g.H = NH + 2 * NKVH; g.F = g.H * (g.D + Da);
  int P = pow2_floor(std::max(1, 256 / std::max(1, g.D)));
  P = std::min(P, 32);
  g.P = P;
  g.nthreads = g.D * P;
  int L = budget / std::max(1, g.D * P);
  L = std::max(1, std::min(L, 64));
  g.L = L;
  g.TT = P * L;
  g.nchunks = T > 0 ? (T + g.TT - 1) / g.TT : 0;
  return g;
}

constexpr int kFwdBudget = 8192;
constexpr int kBwdBudget = 4096;

struct ScanWorkspaceLayout {
  size_t flags, aggA, aggX, inclX, bias_part, init_part, init_cnt, total;
};

inline ScanWorkspaceLayout scan_ws_layout(const ScanGeometry& g) {
  using ltvqkv_host::align_up;
  ScanWorkspaceLayout L;
  size_t tiles = (size_t)g.B * g.H * g.nchunks;
  size_t off = sizeof(WorkspaceHeader);
  L.flags = off; off = align_up(off + tiles * 4, 256);
  L.aggA = off;  off = align_up(off + tiles * g.Da * 4, 256);
  L.aggX = off;  off = align_up(off + tiles * g.D * 4, 256);
  L.inclX = off; off = align_up(off + tiles * g.D * 4, 256);
  L.bias_part = off; off = align_up(off + (size_t)g.B * g.nchunks * g.H * g.Da * 4, 256);
  L.init_part = off; off = align_up(off + (size_t)g.B * g.H * g.D * 4, 256);  // shared initial state
  L.init_cnt = off;  off = align_up(off + (size_t)g.H * 4, 256);
  L.total = off;
  return L;
}

struct ScanFwdArgs {
  const void* combined;
  long long sc_b, sc_t, sc_e;
  const void* inits;
  const float* logit_bias;
  void* out[3];
  ScanGeometry g;
  int use_sigmoid;
  WorkspaceHeader* ws;
  unsigned int* flags;
  float* aggA;
  float* aggX;
  float* inclX;
};

struct ScanBwdArgs {
  const void* combined;
  long long sc_b, sc_t, sc_e;
  const void* inits;
  const float* logit_bias;
  const void* h[3];
  long long hs[3][4];
  const void* gh[3];
  long long gs[3][4];
  void* grad_combined;
  long long gc_b, gc_t, gc_e;
  void* grad_inits;
  ScanGeometry g;
  int use_sigmoid;
  WorkspaceHeader* ws;
  unsigned int* flags;
  float* aggA;
  float* aggX;
  float* inclX;
  float* bias_part;
};


// Spin (one thread) until the flag of a predecessor tile carries the current epoch and a
// state; returns the state, or kFlagIncl with *timed_out set when the wait gave up.
LTVQKV_DEVICE unsigned int wait_flag(const unsigned int* flag, unsigned int epoch_tag, WorkspaceHeader* ws,
                                     bool* timed_out) {
  unsigned long long t0 = 0;
  for (unsigned int it = 0;; ++it) {
    unsigned int f = ld_acquire_u32(flag);
    if ((f >> 2) == epoch_tag && (f & 3u) != kFlagNone) return f & 3u;
    if (it == 64) t0 = global_timer_ns();
    if (it > 64) {
      __nanosleep(64);
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        record_timeout(ws, 0x5CA0u);
        *timed_out = true;
        return kFlagIncl;
      }
    }
  }
}

}  // namespace ltvqkv

#include "ltvqkv_scan_fast.cuh"
#include "ltvqkv_scan_tma.cuh"

namespace ltvqkv {

// ------------------------------------------------------------------------------------------
// Forward
// ------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(1024) scan_fwd_kernel(ScanFwdArgs args) {
  extern __shared__ float smem[];
  const ScanGeometry& g = args.g;
  const int D = g.D, TT = g.TT, P = g.P, L = g.L, Da = g.Da, r = g.r;
  const int ldu = TT + 1;
  float* U = smem;                       // [D][TT+1]
  float* alpha = U + D * ldu;            // [Da][TT]
  float* segA = alpha + Da * TT;         // [D*P]
  float* segX = segA + D * P;            // [D*P]
  float* shE = segX + D * P;             // [D]
  __shared__ unsigned int sh_tile, sh_state, sh_epoch;

  const int tid = threadIdx.x;
  if (tid == 0) {
    sh_tile = draw_ticket(args.ws);
    sh_epoch = *((volatile unsigned int*)&args.ws->epoch) & 0x3FFFFFFFu;
  }
  __syncthreads();
  const unsigned int tile = sh_tile;
  const unsigned int epoch = sh_epoch;
  const int BH = g.B * g.H;
  const int j = (int)(tile / BH);  // chunk index (chunk-major ticket order)
  const int bh = (int)(tile % BH);
  const int b = bh / g.H, h = bh % g.H;
  const int t0 = j * TT;
  const int tlen = min(TT, g.T - t0);

  const T* cb = reinterpret_cast<const T*>(args.combined) + (long long)b * args.sc_b;
  const int head_col = h * (D + Da);

  // Gate values for this tile.
  for (int i = tid; i < Da * TT; i += blockDim.x) {
    int gi = i / TT, t = i - gi * TT;
    if (t < tlen) {
      float l = Elem<T>::load(cb + (long long)(t0 + t) * args.sc_t + (long long)(head_col + D + gi) * args.sc_e) +
                args.logit_bias[h * Da + gi];
      alpha[gi * TT + t] = args.use_sigmoid ? sigmoid_f32(l) : l;
    }
  }
  // Value tile, coalesced along whichever of (t, channel) is unit-stride.
  if (args.sc_t == 1) {
    for (int i = tid; i < D * TT; i += blockDim.x) {
      int c = i / TT, t = i - c * TT;
      if (t < tlen) U[c * ldu + t] = Elem<T>::load(cb + (long long)(t0 + t) + (long long)(head_col + c) * args.sc_e);
    }
  } else {
    for (int i = tid; i < D * TT; i += blockDim.x) {
      int t = i / D, c = i - t * D;
      if (t < tlen)
        U[c * ldu + t] = Elem<T>::load(cb + (long long)(t0 + t) * args.sc_t + (long long)(head_col + c) * args.sc_e);
    }
  }
  __syncthreads();

  const int c = tid / P, s = tid - (tid / P) * P;
  const int gi = c / r;
  const int seg0 = s * L, seg1 = min(seg0 + L, tlen);
  {
    float a = 1.f, x = 0.f;
    for (int t = seg0; t < seg1; ++t) {
      float al = alpha[gi * TT + t];
      x = (1.0f - al) * x + al * U[c * ldu + t];
      a *= (1.0f - al);
    }
    segA[c * P + s] = a;
    segX[c * P + s] = x;
  }
  __syncthreads();
  float ea = 1.f, ex = 0.f;  // composition of segments 0..s-1 of this channel
  for (int sp = 0; sp < s; ++sp) {
    ex = segA[c * P + sp] * ex + segX[c * P + sp];
    ea *= segA[c * P + sp];
  }
  const bool is_last_seg = (s == P - 1);
  float tileA = 0.f, tileX = 0.f;
  if (is_last_seg) {
    float a = segA[c * P + s], x = segX[c * P + s];
    tileA = ea * a;
    tileX = a * ex + x;
  }

  const long long tile_idx = (long long)j * BH + bh;  // payload slot of this tile
  // Deterministic look-back: every kAnchorStride-th chunk is an anchor that publishes its
  // inclusive carry; any other chunk publishes its aggregate and derives its carry-in from its
  // anchor's inclusive carry composed with the aggregates in between, in chunk order — the
  // same association whatever the timing, so results are identical run to run.
  const bool is_anchor = (j % kAnchorStride) == 0;
  if (j == 0) {
    if (is_last_seg) shE[c] = Elem<T>::load(reinterpret_cast<const T*>(args.inits) + ((long long)b * g.H + h) * D + c);
  } else {
    if (!is_anchor) {
      if (is_last_seg) {
        args.aggX[tile_idx * D + c] = tileX;
        if (c % r == 0) args.aggA[tile_idx * Da + gi] = tileA;
        __threadfence();
      }
      __syncthreads();
      if (tid == 0) st_release_u32(&args.flags[tile_idx], (epoch << 2) | kFlagAgg);
    }
    const int m = (j - 1) / kAnchorStride * kAnchorStride;
    bool timed_out = false;
    float E = 0.f;
    for (int k = m; k < j; ++k) {
      const long long pidx = (long long)k * BH + bh;
      if (tid == 0) sh_state = wait_flag(&args.flags[pidx], epoch, args.ws, &timed_out);
      __syncthreads();
      if (is_last_seg && !timed_out) {
        if (k == m) {
          E = ld_cg_f32(&args.inclX[pidx * D + c]);
        } else {
          E = ld_cg_f32(&args.aggA[pidx * Da + gi]) * E + ld_cg_f32(&args.aggX[pidx * D + c]);
        }
      }
      __syncthreads();
    }
    if (is_last_seg) shE[c] = E;
  }
  if (is_anchor) {
    if (is_last_seg) {
      args.inclX[tile_idx * D + c] = tileA * shE[c] + tileX;
      __threadfence();
    }
    __syncthreads();
    if (tid == 0) st_release_u32(&args.flags[tile_idx], (epoch << 2) | kFlagIncl);
  }
  __syncthreads();

  // Final pass: walk the segment from its exact carry, overwriting U with h.
  {
    float carry = ea * shE[c] + ex;
    for (int t = seg0; t < seg1; ++t) {
      float al = alpha[gi * TT + t];
      carry = (1.0f - al) * carry + al * U[c * ldu + t];
      U[c * ldu + t] = carry;
    }
  }
  __syncthreads();

  int which, hloc, nheads;
  split_head(h, g.NH, g.NKVH, which, hloc, nheads);
  T* out = reinterpret_cast<T*>(args.out[which]) + (((long long)b * nheads + hloc) * g.T + t0) * D;
  for (int i = tid; i < D * tlen; i += blockDim.x) {
    int t = i / D, cc = i - t * D;
    Elem<T>::store(out + (long long)t * D + cc, U[cc * ldu + t]);
  }

  if (tid == 0) finish_launch(args.ws, gridDim.x);
}

// ------------------------------------------------------------------------------------------
// Backward
// ------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(1024) scan_bwd_kernel(ScanBwdArgs args) {
  extern __shared__ float smem[];
  const ScanGeometry& g = args.g;
  const int D = g.D, TT = g.TT, P = g.P, L = g.L, Da = g.Da, r = g.r;
  const int ld = TT + 1;
  float* G = smem;                 // [D][TT+1]: upstream grad, then g^
  float* Hs = G + D * ld;          // [D][TT+1]: h_{t-1}, then dlogit contributions
  float* alpha = Hs + D * ld;      // [Da][TT+1]: alpha_{t0+t}, t = 0..tlen (alpha_T := 0)
  float* segA = alpha + Da * ld;   // [D*P]
  float* segX = segA + D * P;      // [D*P]
  float* shE = segX + D * P;       // [D]
  float* red = shE + D;            // [Da][TT]
  __shared__ unsigned int sh_tile, sh_state, sh_epoch;

  const int tid = threadIdx.x;
  if (tid == 0) {
    sh_tile = draw_ticket(args.ws);
    sh_epoch = *((volatile unsigned int*)&args.ws->epoch) & 0x3FFFFFFFu;
  }
  __syncthreads();
  const unsigned int tile = sh_tile;
  const unsigned int epoch = sh_epoch;
  const int BH = g.B * g.H;
  const int j = g.nchunks - 1 - (int)(tile / BH);  // reverse chunk order
  const int bh = (int)(tile % BH);
  const int b = bh / g.H, h = bh % g.H;
  const int t0 = j * TT;
  const int tlen = min(TT, g.T - t0);
  int which, hloc, nheads;
  split_head(h, g.NH, g.NKVH, which, hloc, nheads);

  const T* cb = reinterpret_cast<const T*>(args.combined) + (long long)b * args.sc_b;
  const int head_col = h * (D + Da);

  for (int i = tid; i < Da * ld; i += blockDim.x) {
    int gi = i / ld, t = i - gi * ld;
    if (t <= tlen) {
      float al = 0.f;
      if (t0 + t < g.T) {
        float l = Elem<T>::load(cb + (long long)(t0 + t) * args.sc_t + (long long)(head_col + D + gi) * args.sc_e) +
                  args.logit_bias[h * Da + gi];
        al = args.use_sigmoid ? sigmoid_f32(l) : l;
      }
      alpha[gi * ld + t] = al;
    }
  }
  {
    const T* gp = reinterpret_cast<const T*>(args.gh[which]);
    const long long* st = args.gs[which];
    const T* base = gp + (long long)b * st[0] + (long long)hloc * st[1];
    if (st[3] == 1 || st[2] != 1) {
      for (int i = tid; i < D * TT; i += blockDim.x) {
        int t = i / D, c = i - t * D;
        if (t < tlen) G[c * ld + t] = Elem<T>::load(base + (long long)(t0 + t) * st[2] + (long long)c * st[3]);
      }
    } else {
      for (int i = tid; i < D * TT; i += blockDim.x) {
        int c = i / TT, t = i - c * TT;
        if (t < tlen) G[c * ld + t] = Elem<T>::load(base + (long long)(t0 + t) + (long long)c * st[3]);
      }
    }
  }
  __syncthreads();

  const int c = tid / P, s = tid - (tid / P) * P;
  const int gi = c / r;
  const int seg0 = min(s * L, tlen), seg1 = min(s * L + L, tlen);
  {
    float a = 1.f, x = 0.f;
    for (int t = seg1 - 1; t >= seg0; --t) {
      float an = 1.0f - alpha[gi * ld + t + 1];
      x = an * x + G[c * ld + t];
      a *= an;
    }
    segA[c * P + s] = a;
    segX[c * P + s] = x;
  }
  __syncthreads();
  float ea = 1.f, ex = 0.f;  // composition of segments s+1..P-1 (to the right)
  for (int sp = P - 1; sp > s; --sp) {
    ex = segA[c * P + sp] * ex + segX[c * P + sp];
    ea *= segA[c * P + sp];
  }
  const bool is_first_seg = (s == 0);
  float tileA = 0.f, tileX = 0.f;
  if (is_first_seg) {
    float a = segA[c * P], x = segX[c * P];
    tileA = ea * a;
    tileX = a * ex + x;
  }

  const long long tile_idx = (long long)j * BH + bh;
  // Deterministic look-back in reverse chunk order (see the forward kernel): rj counts chunks
  // from the end; anchors publish inclusive carries, the others aggregates.
  const int rj = g.nchunks - 1 - j;
  const bool is_anchor = (rj % kAnchorStride) == 0;
  if (rj == 0) {
    if (is_first_seg) shE[c] = 0.f;
  } else {
    if (!is_anchor) {
      if (is_first_seg) {
        args.aggX[tile_idx * D + c] = tileX;
        if (c % r == 0) args.aggA[tile_idx * Da + gi] = tileA;
        __threadfence();
      }
      __syncthreads();
      if (tid == 0) st_release_u32(&args.flags[tile_idx], (epoch << 2) | kFlagAgg);
    }
    const int mr = (rj - 1) / kAnchorStride * kAnchorStride;
    bool timed_out = false;
    float E = 0.f;
    for (int rk = mr; rk < rj; ++rk) {
      const long long pidx = (long long)(g.nchunks - 1 - rk) * BH + bh;
      if (tid == 0) sh_state = wait_flag(&args.flags[pidx], epoch, args.ws, &timed_out);
      __syncthreads();
      if (is_first_seg && !timed_out) {
        if (rk == mr) {
          E = ld_cg_f32(&args.inclX[pidx * D + c]);
        } else {
          E = ld_cg_f32(&args.aggA[pidx * Da + gi]) * E + ld_cg_f32(&args.aggX[pidx * D + c]);
        }
      }
      __syncthreads();
    }
    if (is_first_seg) shE[c] = E;
  }
  if (is_anchor) {
    if (is_first_seg) {
      args.inclX[tile_idx * D + c] = tileA * shE[c] + tileX;
      __threadfence();
    }
    __syncthreads();
    if (tid == 0) st_release_u32(&args.flags[tile_idx], (epoch << 2) | kFlagIncl);
  }
  __syncthreads();

  {
    float carry = ea * shE[c] + ex;  // g^ at the token right after this segment
    for (int t = seg1 - 1; t >= seg0; --t) {
      carry = (1.0f - alpha[gi * ld + t + 1]) * carry + G[c * ld + t];
      G[c * ld + t] = carry;
    }
  }
  // h_{t-1} for the tile (saved forward output, or inits at t = 0).
  {
    const T* hp = reinterpret_cast<const T*>(args.h[which]);
    const long long* st = args.hs[which];
    const T* base = hp + (long long)b * st[0] + (long long)hloc * st[1];
    const T* ini = reinterpret_cast<const T*>(args.inits) + ((long long)b * g.H + h) * D;
    for (int i = tid; i < D * TT; i += blockDim.x) {
      int t = i / D, cc = i - t * D;
      if (t < tlen) {
        int tt = t0 + t - 1;
        Hs[cc * ld + t] = tt < 0 ? Elem<T>::load(ini + cc) : Elem<T>::load(base + (long long)tt * st[2] + (long long)cc * st[3]);
      }
    }
  }
  __syncthreads();

  // Elementwise part: du, dalpha -> dlogit contributions, dinits.
  T* gcb = reinterpret_cast<T*>(args.grad_combined) + (long long)b * args.gc_b;
  const bool t_fast = (args.sc_t == 1 || args.gc_t == 1);
  for (int i = tid; i < D * TT; i += blockDim.x) {
    int cc, t;
    if (t_fast) { cc = i / TT; t = i - cc * TT; }
    else { t = i / D; cc = i - t * D; }
    if (t >= tlen) continue;
    const int gg = cc / r;
    const float al = alpha[gg * ld + t];
    const float ghat = G[cc * ld + t];
    const float u = Elem<T>::load(cb + (long long)(t0 + t) * args.sc_t + (long long)(head_col + cc) * args.sc_e);
    Elem<T>::store(gcb + (long long)(t0 + t) * args.gc_t + (long long)(head_col + cc) * args.gc_e, al * ghat);
    const float dalpha = (u - Hs[cc * ld + t]) * ghat;
    Hs[cc * ld + t] = args.use_sigmoid ? dalpha * (al * (1.0f - al)) : dalpha;
    if (t0 + t == 0)
      Elem<T>::store(reinterpret_cast<T*>(args.grad_inits) + ((long long)b * g.H + h) * D + cc, ghat * (1.0f - al));
  }
  __syncthreads();
  for (int i = tid; i < Da * TT; i += blockDim.x) {
    int gg = i / TT, t = i - gg * TT;
    if (t < tlen) {
      float sum = 0.f;
      for (int k = 0; k < r; ++k) sum += Hs[(gg * r + k) * ld + t];
      Elem<T>::store(gcb + (long long)(t0 + t) * args.gc_t + (long long)(head_col + D + gg) * args.gc_e, sum);
      red[gg * TT + t] = sum;
    }
  }
  __syncthreads();
  for (int gg = tid; gg < Da; gg += blockDim.x) {
    float sum = 0.f;
    for (int t = 0; t < tlen; ++t) sum += red[gg * TT + t];
    args.bias_part[(((long long)b * g.nchunks + j) * g.H + h) * Da + gg] = sum;
  }

  if (tid == 0) finish_launch(args.ws, gridDim.x);
}

// ------------------------------------------------------------------------------------------
// fp32 exact-order path. One CTA per (batch, head), one thread per channel, sequential in t,
// with every multiply and add separately rounded (no FMA contraction): the operation order of
// the reference's sequential oracle (ltv_reference_ops.py:103-122 and the autograd backward of
// QuantizedStateUpdate, :20-34), so fp32 results match it to the last bit up to the library
// expf. Used for dtype fp32, where the tolerance is 1e-5; bf16 takes the chunked kernels.
// ------------------------------------------------------------------------------------------
struct ExactArgs {
  const float* combined;
  long long sc_b, sc_t, sc_e;
  const float* inits;
  const float* logit_bias;
  float* out[3];
  const float* h[3];
  long long hs[3][4];
  const float* gh[3];
  long long gs[3][4];
  float* grad_combined;
  long long gc_b, gc_t, gc_e;
  float* grad_inits;
  float* bias_part;  // [B][H][Da]
  int B, T, NH, NKVH, Da, r, D, H, use_sigmoid;
};

LTVQKV_DEVICE float exact_alpha(const ExactArgs& a, const float* cb, int t, int head_col, int h, int g) {
  float raw = __fadd_rn(cb[(long long)t * a.sc_t + (long long)(head_col + a.D + g) * a.sc_e], a.logit_bias[h * a.Da + g]);
  return a.use_sigmoid ? sigmoid_f32_exact(raw) : raw;
}

__global__ void __launch_bounds__(1024) scan_fwd_exact_kernel(ExactArgs a) {
  const int bh = blockIdx.x;
  const int b = bh / a.H, h = bh % a.H;
  const int c = threadIdx.x;
  if (c >= a.D) return;
  int which, hloc, nheads;
  split_head(h, a.NH, a.NKVH, which, hloc, nheads);
  const float* cb = a.combined + (long long)b * a.sc_b;
  const int head_col = h * (a.D + a.Da);
  const int g = c / a.r;
  float st = a.inits[((long long)b * a.H + h) * a.D + c];
  float* out = a.out[which] + ((long long)b * nheads + hloc) * (long long)a.T * a.D + c;
  for (int t = 0; t < a.T; ++t) {
    const float al = exact_alpha(a, cb, t, head_col, h, g);
    const float u = cb[(long long)t * a.sc_t + (long long)(head_col + c) * a.sc_e];
    const float t1 = __fmul_rn(__fsub_rn(1.0f, al), st);
    const float t2 = __fmul_rn(al, u);
    st = __fadd_rn(t1, t2);
    out[(long long)t * a.D] = st;
  }
}

__global__ void __launch_bounds__(1024) scan_bwd_exact_kernel(ExactArgs a) {
  extern __shared__ float red[];  // [D] per-channel terms of the group sums
  const int bh = blockIdx.x;
  const int b = bh / a.H, h = bh % a.H;
  const int c = threadIdx.x;
  const bool active = c < a.D;
  int which, hloc, nheads;
  split_head(h, a.NH, a.NKVH, which, hloc, nheads);
  const float* cb = a.combined + (long long)b * a.sc_b;
  float* gcb = a.grad_combined + (long long)b * a.gc_b;
  const int head_col = h * (a.D + a.Da);
  const int g = active ? c / a.r : 0;
  const long long* hs = a.hs[which];
  const long long* gs = a.gs[which];
  const float* hp = a.h[which] + (long long)b * hs[0] + (long long)hloc * hs[1] + (long long)c * hs[3];
  const float* gp = a.gh[which] + (long long)b * gs[0] + (long long)hloc * gs[1] + (long long)c * gs[3];
  const float init = active ? a.inits[((long long)b * a.H + h) * a.D + c] : 0.f;
  float gacc = 0.f;
  float bias_acc = 0.f;  // threads c < Da accumulate their group's bias gradient
  for (int t = a.T - 1; t >= 0; --t) {
    float al = 0.f, term = 0.f;
    if (active) {
      gacc = __fadd_rn(gacc, gp[(long long)t * gs[2]]);
      al = exact_alpha(a, cb, t, head_col, h, g);
      const float u = cb[(long long)t * a.sc_t + (long long)(head_col + c) * a.sc_e];
      const float sprev = t > 0 ? hp[(long long)(t - 1) * hs[2]] : init;
      gcb[(long long)t * a.gc_t + (long long)(head_col + c) * a.gc_e] = __fmul_rn(gacc, al);
      term = __fmul_rn(gacc, __fsub_rn(u, sprev));
      red[c] = term;
    }
    __syncthreads();
    if (c < a.Da) {
      float ga = 0.f;
      for (int k = 0; k < a.r; ++k) ga = __fadd_rn(ga, red[c * a.r + k]);
      const float ag = exact_alpha(a, cb, t, head_col, h, c);
      const float graw = a.use_sigmoid ? __fmul_rn(__fmul_rn(ga, __fsub_rn(1.0f, ag)), ag) : ga;
      gcb[(long long)t * a.gc_t + (long long)(head_col + a.D + c) * a.gc_e] = graw;
      bias_acc = __fadd_rn(bias_acc, graw);
    }
    __syncthreads();
    if (active) gacc = __fmul_rn(gacc, __fsub_rn(1.0f, al));
  }
  if (active) a.grad_inits[((long long)b * a.H + h) * a.D + c] = gacc;
  if (c < a.Da) a.bias_part[((long long)b * a.H + h) * a.Da + c] = bias_acc;
}

// grad_logit_bias[h, g] += sum over b (descending, the oracle's order) of per-(b, h) partials.
__global__ void bias_reduce_exact_kernel(const float* part, float* grad_bias, int B, int H, int Da) {
  int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= H * Da) return;
  float sum = 0.f;
  for (int b = B - 1; b >= 0; --b) sum = __fadd_rn(sum, part[(long long)b * H * Da + idx]);
  grad_bias[idx] = __fadd_rn(grad_bias[idx], sum);
}

// grad_logit_bias[h, g] += sum over (b, chunk) of the per-tile partials: one CTA per (h, g),
// each thread sums a fixed strided subset, then a fixed shared-memory tree (deterministic).
constexpr int kBiasReduceThreads = 256;
__global__ void __launch_bounds__(kBiasReduceThreads) bias_reduce_kernel(const float* part, float* grad_bias, int B,
                                                                         int nchunks, int H, int Da) {
  __shared__ float sm[kBiasReduceThreads];
  const int idx = blockIdx.x;  // h * Da + g
  const int n = B * nchunks;
  float sum = 0.f;
  for (int bj = threadIdx.x; bj < n; bj += kBiasReduceThreads) sum += part[(long long)bj * H * Da + idx];
  sm[threadIdx.x] = sum;
  __syncthreads();
  for (int o = kBiasReduceThreads / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) sm[threadIdx.x] += sm[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) grad_bias[idx] += sm[0];
}

__global__ void zero_grad_inits_kernel(void* p, long long n, int bf16) {
  long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (bf16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(0.f);
  else reinterpret_cast<float*>(p)[i] = 0.f;
}

inline size_t fwd_smem_bytes(const ScanGeometry& g) {
  return sizeof(float) * ((size_t)g.D * (g.TT + 1) + (size_t)g.Da * g.TT + 2 * (size_t)g.D * g.P + g.D);
}
inline size_t bwd_smem_bytes(const ScanGeometry& g) {
  return sizeof(float) * (2 * (size_t)g.D * (g.TT + 1) + (size_t)g.Da * (g.TT + 1) + 2 * (size_t)g.D * g.P + g.D +
                          (size_t)g.Da * g.TT);
}

}  // namespace ltvqkv

using namespace ltvqkv;

static int validate_scan_shape(int B, int T, int NH, int NKVH, int Da, int r) {
  if (B < 0 || T < 0 || NH < 0 || NKVH < 0 || Da <= 0 || r <= 0) return LTVQKV_ERR_SHAPE;
  if (NH + 2 * NKVH <= 0) return LTVQKV_ERR_SHAPE;
  long long D = (long long)Da * r;
  if (D > 1024) return LTVQKV_ERR_SHAPE;
  return LTVQKV_OK;
}

namespace {
constexpr size_t kMaxDynSmem = 227 * 1024;  // per-CTA dynamic shared memory limit of sm_100

// Exact [B, F, T]-contiguous view of combined / grad_combined (what the projection produces).
bool production_layout(const void* p, int64_t sb, int64_t st, int64_t se, int T, int F) {
  return p != nullptr && aligned16p(p) && st == 1 && se == T && sb == (int64_t)F * T && T % 8 == 0;
}

bool bf16_map_2d(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swizzle) {
  const uint64_t dims[2] = {cols, rows};
  const uint64_t strides[1] = {cols * 2};
  const uint32_t box[2] = {box_cols, box_rows};
  return ltvqkv_host::encode_tiled_map(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, swizzle);
}

// [B, heads, T, D] tensor with d unit stride as a 4-D map (d, t, head, b), box (D, tt, 1, 1).
bool bf16_map_rows(CUtensorMap* m, const void* base, const int64_t* st, int B, int heads, int T, int D, int tt) {
  const uint64_t dims[4] = {(uint64_t)D, (uint64_t)T, (uint64_t)heads, (uint64_t)B};
  const uint64_t strides[3] = {(uint64_t)st[2] * 2, (uint64_t)st[1] * 2, (uint64_t)st[0] * 2};
  const uint32_t box[4] = {(uint32_t)D, (uint32_t)tt, 1, 1};
  return ltvqkv_host::encode_tiled_map(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box,
                                       CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Row kernels by head dim (64, 128 or 256) and chunk length (32 or 64 tokens).
template <int kTT>
decltype(&scan_fwd_rows_kernel<128, 32>) row_fwd_kernel(int D) {
  return D == 64 ? scan_fwd_rows_kernel<64, kTT> : (D == 128 ? scan_fwd_rows_kernel<128, kTT> : scan_fwd_rows_kernel<256, kTT>);
}
decltype(&scan_bwd_rows_kernel<128, 32, false>) row_bwd_kernel(int D, bool ckpt) {
  if (ckpt) return scan_bwd_rows_kernel<128, 32, true>;  // checkpoints come from the D = 128 fused forward
  return D == 64 ? scan_bwd_rows_kernel<64, 32, false>
                 : (D == 128 ? scan_bwd_rows_kernel<128, 32, false> : scan_bwd_rows_kernel<256, 32, false>);
}
// Chunk lengths and ring depths of the row kernels, measured on B200 at config 2 (576 rows, head
// dim 128). Forward: 64-token chunks (128-byte value-tile rows; 32 when a decay group is narrower
// than 64 channels) in a 3-stage ring, 4 CTAs per SM, so all rows are resident in one wave.
// Backward: 32-token chunks in a 2-stage ring, 4 CTAs per SM; 64-token chunks fit only 2 CTAs per
// SM (two waves of rows) and measured slower.
int row_fwd_chunk_tokens(int r) { return r >= 64 ? 64 : 32; }
int row_bwd_chunk_tokens(int /*r*/) { return 32; }
constexpr int kRowFwdStages = 3;
constexpr int kRowBwdStages = 2;

int persistent_grid(const void* kernel, int threads, size_t smem, int ntiles) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  return std::max(1, std::min(ntiles, per_sm * ltvqkv_host::num_sms()));
}
// Whether the forward takes the row-streaming kernel (bf16, production layout, enough rows).
bool row_fwd_applies(int dtype, const void* combined, int64_t sc_b, int64_t sc_t, int64_t sc_e, const void* inits,
                     const void* out_q, const void* out_k, const void* out_v, int B, int T, int NH, int NKVH, int Da,
                     int r) {
  const int D = Da * r, H = NH + 2 * NKVH, F = H * (D + Da);
  const int rtt = row_fwd_chunk_tokens(r);
  return dtype == LTVQKV_DTYPE_BF16 && fast_shape_ok(T, Da, r) && r >= rtt && r % 32 == 0 &&
         (D == 64 || D == 128 || D == 256) && H * Da <= kRowMaxBias &&
         (long long)B * H >= 2LL * ltvqkv_host::num_sms() &&
         row_fwd_smem_bytes(D, Da, H, rtt, kRowFwdStages) <= kMaxDynSmem &&
         production_layout(combined, sc_b, sc_t, sc_e, T, F) && aligned16p(inits) &&
         (NH == 0 || aligned16p(out_q)) && (NKVH == 0 || (aligned16p(out_k) && aligned16p(out_v)));
}

// Row-streaming forward when its conditions hold; `used` reports whether it ran.
int try_row_fwd(bool& used, int dtype, const void* combined, int64_t sc_b, int64_t sc_t, int64_t sc_e,
                const void* inits, const float* logit_bias, void* out_q, void* out_k, void* out_v, int B, int T, int NH,
                int NKVH, int Da, int r, int use_sigmoid, char* ws, cudaStream_t s) {
  used = false;
  const int D = Da * r, H = NH + 2 * NKVH, F = H * (D + Da);
  const int rtt = row_fwd_chunk_tokens(r);
  const int rst = kRowFwdStages;
  if (!row_fwd_applies(dtype, combined, sc_b, sc_t, sc_e, inits, out_q, out_k, out_v, B, T, NH, NKVH, Da, r)) return LTVQKV_OK;
  used = true;
  CUtensorMap tm_u, tm_l;
  const uint64_t rows = (uint64_t)B * F;
  if (!bf16_map_2d(&tm_u, combined, T, rows, rtt, D, rtt == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B) ||
      !bf16_map_2d(&tm_l, combined, T, rows, rtt, Da, CU_TENSOR_MAP_SWIZZLE_NONE))
    return LTVQKV_ERR_LAUNCH;
  TmaFwdArgs f;
  f.inits = reinterpret_cast<const __nv_bfloat16*>(inits); f.logit_bias = logit_bias;
  f.out[0] = reinterpret_cast<__nv_bfloat16*>(out_q); f.out[1] = reinterpret_cast<__nv_bfloat16*>(out_k);
  f.out[2] = reinterpret_cast<__nv_bfloat16*>(out_v);
  f.B = B; f.T = T; f.NH = NH; f.NKVH = NKVH; f.Da = Da; f.r = r; f.D = D; f.H = H; f.F = F;
  f.nchunks = (T + rtt - 1) / rtt; f.nrows = B * H; f.use_sigmoid = use_sigmoid; f.stages = rst;
  f.ws = reinterpret_cast<WorkspaceHeader*>(ws);
  const size_t tsm = row_fwd_smem_bytes(D, Da, H, rtt, rst);
  const int threads = D + 32;
  auto kern = rtt == 64 ? row_fwd_kernel<64>(D) : row_fwd_kernel<32>(D);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tsm) != cudaSuccess)
    return ltvqkv_host::check_launch();
  const int grid = persistent_grid((const void*)kern, threads, tsm, f.nrows);
  kern<<<grid, threads, tsm, s>>>(tm_u, tm_l, f);
  return ltvqkv_host::check_launch();
}

// Row-streaming backward when its conditions hold; `used` reports whether it ran.
int try_row_bwd(bool& used, int dtype, const void* combined, int64_t sc_b, int64_t sc_t, int64_t sc_e,
                const void* inits, const float* logit_bias, const void* hq, const int64_t* hq_strides, const void* hk,
                const int64_t* hk_strides, const void* hv, const int64_t* hv_strides, const void* grad_hq,
                const int64_t* gq_strides, const void* grad_hk, const int64_t* gk_strides, const void* grad_hv,
                const int64_t* gv_strides, void* grad_combined, int64_t gc_b, int64_t gc_t, int64_t gc_e,
                void* grad_inits, float* grad_logit_bias, int B, int T, int NH, int NKVH, int Da, int r,
                int use_sigmoid, char* ws, size_t workspace_bytes, cudaStream_t s, const float* ckpt = nullptr,
                bool shared_init = false, float* grad_init_sum = nullptr, bool bias_overwrite = false) {
  used = false;
  auto rows_ok = [&](const void* p, const int64_t* st) {
    return p == nullptr || (aligned16p(p) && st[3] == 1 && st[0] % 8 == 0 && st[1] % 8 == 0 && st[2] % 8 == 0);
  };
  // with checkpoints the outputs are not read (their maps are never used)
  auto h_ok = [&](const void* p, const int64_t* st) { return ckpt != nullptr || rows_ok(p, st); };
  const int H = NH + 2 * NKVH, D = Da * r;
  const int tpg = r / 32;
  const bool r_ok = r % 32 == 0 && tpg >= 1 && (tpg & (tpg - 1)) == 0;
  const int Fh = H * (D + Da);
  const int rtt = row_bwd_chunk_tokens(r);
  const int rst = kRowBwdStages;
  const size_t tsm = row_bwd_smem_bytes(D, Da, H, rtt, rst);
  if (!(dtype == LTVQKV_DTYPE_BF16 && r_ok && r >= rtt && (D == 64 || D == 128 || D == 256) &&
        H * Da <= kRowMaxBias && fast_shape_ok(T, Da, r) && tsm <= kMaxDynSmem &&
        (long long)B * H >= 2LL * ltvqkv_host::num_sms() && production_layout(combined, sc_b, sc_t, sc_e, T, Fh) &&
        production_layout(grad_combined, gc_b, gc_t, gc_e, T, Fh) && aligned16p(inits) &&
        h_ok(hq, hq_strides) && rows_ok(grad_hq, gq_strides) &&
        (NKVH == 0 || (h_ok(hk, hk_strides) && h_ok(hv, hv_strides) && rows_ok(grad_hk, gk_strides) &&
                       rows_ok(grad_hv, gv_strides))) &&
        (ckpt == nullptr || (D == 128 && T % rtt == 0 && aligned16p(ckpt)))))
    return LTVQKV_OK;
  used = true;
  CUtensorMap tm_u, tm_du, tm_l, tm_g[3], tm_h[3];
  const uint64_t rows = (uint64_t)B * Fh;
  const CUtensorMapSwizzle tile_swz = rtt == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  bool ok = bf16_map_2d(&tm_u, combined, T, rows, rtt, D, tile_swz) &&
            bf16_map_2d(&tm_du, grad_combined, T, rows, rtt, D, tile_swz) &&
            bf16_map_2d(&tm_l, combined, T, rows, row_bwd_logit_box(rtt), Da, CU_TENSOR_MAP_SWIZZLE_NONE);
  const void* hh[3] = {hq, hk, hv};
  const void* gg[3] = {grad_hq, grad_hk, grad_hv};
  const int64_t* hst[3] = {hq_strides, hk_strides, hv_strides};
  const int64_t* gst[3] = {gq_strides, gk_strides, gv_strides};
  const int heads[3] = {NH, NKVH, NKVH};
  for (int i = 0; i < 3 && ok; ++i) {
    const int src = heads[i] > 0 ? i : 0;  // unused groups reuse the q maps
    ok = bf16_map_rows(&tm_g[i], gg[src], gst[src], B, heads[src], T, D, rtt);
    if (ckpt == nullptr) ok = ok && bf16_map_rows(&tm_h[i], hh[src], hst[src], B, heads[src], T, D, rtt);
    else tm_h[i] = tm_g[i];  // not read
  }
  if (!ok) return LTVQKV_ERR_LAUNCH;
  const ScanWorkspaceLayout wx = scan_ws_layout(fast_geometry(B, T, NH, NKVH, Da, r));
  if (workspace_bytes < wx.total) return LTVQKV_ERR_WORKSPACE;
  TmaBwdArgs f;
  f.inits = reinterpret_cast<const __nv_bfloat16*>(inits); f.logit_bias = logit_bias;
  f.grad_combined = reinterpret_cast<__nv_bfloat16*>(grad_combined);
  f.grad_inits = reinterpret_cast<__nv_bfloat16*>(grad_inits);
  f.bias_part = reinterpret_cast<float*>(ws + wx.bias_part);
  f.grad_bias = grad_logit_bias;
  f.ckpt = ckpt;
  f.inits_bs = shared_init ? 0 : (long long)H * D;
  f.init_part = shared_init ? reinterpret_cast<float*>(ws + wx.init_part) : nullptr;
  f.init_cnt = reinterpret_cast<unsigned int*>(ws + wx.init_cnt);
  f.grad_init_sum = grad_init_sum;
  f.bias_overwrite = bias_overwrite ? 1 : 0;
  if (shared_init && cudaMemsetAsync(f.init_cnt, 0, (size_t)H * 4, s) != cudaSuccess)
    return ltvqkv_host::check_launch();
  f.B = B; f.T = T; f.NH = NH; f.NKVH = NKVH; f.Da = Da; f.r = r; f.D = D; f.H = H; f.F = Fh;
  f.nchunks = (T + rtt - 1) / rtt; f.nrows = B * H; f.use_sigmoid = use_sigmoid; f.stages = rst;
  f.ws = reinterpret_cast<WorkspaceHeader*>(ws);
  const int threads = D / 2 + (ckpt != nullptr ? 64 : 32);  // consumers own channel pairs, producer (+ replay) warp
  auto kern = row_bwd_kernel(D, ckpt != nullptr);  // 32-token chunks
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tsm) != cudaSuccess)
    return ltvqkv_host::check_launch();
  const int grid = persistent_grid((const void*)kern, threads, tsm, f.nrows);
  kern<<<grid, threads, tsm, s>>>(tm_u, tm_l, tm_du, tm_g[0], tm_g[1], tm_g[2], tm_h[0], tm_h[1], tm_h[2], f);
  return ltvqkv_host::check_launch();  // the kernel's last CTA also reduces the bias partials
}

}  // namespace

extern "C" size_t ltvqkv_scan_workspace_bytes(int B, int T, int NH, int NKVH, int Da, int r) {
  if (validate_scan_shape(B, T, NH, NKVH, Da, r) != LTVQKV_OK) return 0;
  ScanGeometry gf = make_geometry(B, T, NH, NKVH, Da, r, kFwdBudget);
  ScanGeometry gb = make_geometry(B, T, NH, NKVH, Da, r, kBwdBudget);
  ScanGeometry gx = fast_geometry(B, T, NH, NKVH, Da, r);
  return std::max({scan_ws_layout(gf).total, scan_ws_layout(gb).total, scan_ws_layout(gx).total});
}

extern "C" int ltvqkv_scan_fwd(int dtype, const void* combined, int64_t sc_b, int64_t sc_t, int64_t sc_e,
                               const void* inits, const float* logit_bias, void* out_q, void* out_k, void* out_v,
                               int B, int T, int NH, int NKVH, int Da, int r, int use_sigmoid, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (!ltvqkv_host::valid_dtype(dtype)) return LTVQKV_ERR_DTYPE;
  int st = validate_scan_shape(B, T, NH, NKVH, Da, r);
  if (st != LTVQKV_OK) return st;
  if (B == 0 || T == 0) return LTVQKV_OK;
  if (!combined || !inits || !logit_bias || (NH > 0 && !out_q) || (NKVH > 0 && (!out_k || !out_v)))
    return LTVQKV_ERR_INVALID_ARG;
  ScanGeometry g = make_geometry(B, T, NH, NKVH, Da, r, kFwdBudget);
  ScanWorkspaceLayout wl = scan_ws_layout(g);
  if (!workspace || workspace_bytes < wl.total) return LTVQKV_ERR_WORKSPACE;
  char* ws = reinterpret_cast<char*>(workspace);
  ScanFwdArgs a;
  a.combined = combined; a.sc_b = sc_b; a.sc_t = sc_t; a.sc_e = sc_e;
  a.inits = inits; a.logit_bias = logit_bias;
  a.out[0] = out_q; a.out[1] = out_k; a.out[2] = out_v;
  a.g = g; a.use_sigmoid = use_sigmoid;
  a.ws = reinterpret_cast<WorkspaceHeader*>(ws);
  a.flags = reinterpret_cast<unsigned int*>(ws + wl.flags);
  a.aggA = reinterpret_cast<float*>(ws + wl.aggA);
  a.aggX = reinterpret_cast<float*>(ws + wl.aggX);
  a.inclX = reinterpret_cast<float*>(ws + wl.inclX);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == LTVQKV_DTYPE_F32) {
    ExactArgs e = {};
    e.combined = reinterpret_cast<const float*>(combined); e.sc_b = sc_b; e.sc_t = sc_t; e.sc_e = sc_e;
    e.inits = reinterpret_cast<const float*>(inits); e.logit_bias = logit_bias;
    e.out[0] = reinterpret_cast<float*>(out_q); e.out[1] = reinterpret_cast<float*>(out_k);
    e.out[2] = reinterpret_cast<float*>(out_v);
    e.B = B; e.T = T; e.NH = NH; e.NKVH = NKVH; e.Da = Da; e.r = r; e.D = g.D; e.H = g.H; e.use_sigmoid = use_sigmoid;
    int threads = (g.D + 31) / 32 * 32;
    scan_fwd_exact_kernel<<<(unsigned int)(B * g.H), threads, 0, s>>>(e);
    return ltvqkv_host::check_launch();
  }
  {
    bool used = false;
    const int rc = try_row_fwd(used, dtype, combined, sc_b, sc_t, sc_e, inits, logit_bias, out_q, out_k, out_v, B, T,
                               NH, NKVH, Da, r, use_sigmoid, ws, s);
    if (used) return rc;
  }
  if (dtype == LTVQKV_DTYPE_BF16 && sc_t == 1 && sc_e % 8 == 0 && sc_b % 8 == 0 && fast_shape_ok(T, Da, r) &&
      aligned16p(combined) && aligned16p(inits) && (NH == 0 || aligned16p(out_q)) &&
      (NKVH == 0 || (aligned16p(out_k) && aligned16p(out_v)))) {
    const ScanGeometry gx = fast_geometry(B, T, NH, NKVH, Da, r);
    const ScanWorkspaceLayout wx = scan_ws_layout(gx);
    if (workspace_bytes < wx.total) return LTVQKV_ERR_WORKSPACE;
    FastFwdArgs f;
    f.combined = reinterpret_cast<const __nv_bfloat16*>(combined); f.sc_b = sc_b; f.sc_e = sc_e;
    f.inits = reinterpret_cast<const __nv_bfloat16*>(inits); f.logit_bias = logit_bias;
    f.out[0] = reinterpret_cast<__nv_bfloat16*>(out_q); f.out[1] = reinterpret_cast<__nv_bfloat16*>(out_k);
    f.out[2] = reinterpret_cast<__nv_bfloat16*>(out_v);
    f.B = B; f.T = T; f.NH = NH; f.NKVH = NKVH; f.Da = Da; f.r = r; f.D = gx.D; f.H = gx.H;
    f.nchunks = gx.nchunks; f.use_sigmoid = use_sigmoid;
    f.aggA = reinterpret_cast<float*>(ws + wx.aggA);
    f.aggX = reinterpret_cast<float*>(ws + wx.aggX);
    f.inclX = reinterpret_cast<float*>(ws + wx.inclX);
    // three passes: tile aggregates, carries per (row, channel), tiles from their carries
    const unsigned int tiles = (unsigned int)((long long)B * gx.H * gx.nchunks);
    const bool small = gx.D <= 128;  // 256 threads: a register cap that fits more CTAs per SM
    auto agg = small ? scan_fwd_agg_kernel<256, kFastFwdAggMinBlocks256> : scan_fwd_agg_kernel<512, 2>;
    agg<<<tiles, 2 * gx.D, 0, s>>>(f);
    int rc = ltvqkv_host::check_launch();
    if (rc != LTVQKV_OK) return rc;
    const long long nthreads = (long long)B * gx.H * gx.D;
    scan_fwd_carry_kernel<<<(unsigned int)((nthreads + 255) / 256), 256, 0, s>>>(f);
    rc = ltvqkv_host::check_launch();
    if (rc != LTVQKV_OK) return rc;
    const size_t fsm = fast_fwd_smem_bytes(gx.D, Da);
    auto apply = small ? scan_fwd_apply_kernel<256, kFastFwdMinBlocks256> : scan_fwd_apply_kernel<512, 2>;
    cudaFuncSetAttribute(apply, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fsm);
    apply<<<tiles, 2 * gx.D, fsm, s>>>(f);
    return ltvqkv_host::check_launch();
  }
  size_t smem = fwd_smem_bytes(g);
  unsigned int grid = (unsigned int)((long long)B * g.H * g.nchunks);
  if (dtype == LTVQKV_DTYPE_BF16) {
    cudaFuncSetAttribute(scan_fwd_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    scan_fwd_kernel<__nv_bfloat16><<<grid, g.nthreads, smem, s>>>(a);
  } else {
    cudaFuncSetAttribute(scan_fwd_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    scan_fwd_kernel<float><<<grid, g.nthreads, smem, s>>>(a);
  }
  return ltvqkv_host::check_launch();
}

extern "C" int ltvqkv_scan_bwd(int dtype, const void* combined, int64_t sc_b, int64_t sc_t, int64_t sc_e,
                               const void* inits, const float* logit_bias, const void* hq, const int64_t* hq_strides,
                               const void* hk, const int64_t* hk_strides, const void* hv, const int64_t* hv_strides,
                               const void* grad_hq, const int64_t* gq_strides, const void* grad_hk,
                               const int64_t* gk_strides, const void* grad_hv, const int64_t* gv_strides,
                               void* grad_combined, int64_t gc_b, int64_t gc_t, int64_t gc_e, void* grad_inits,
                               float* grad_logit_bias, int B, int T, int NH, int NKVH, int Da, int r, int use_sigmoid,
                               void* workspace, size_t workspace_bytes, void* stream) {
  if (!ltvqkv_host::valid_dtype(dtype)) return LTVQKV_ERR_DTYPE;
  int st = validate_scan_shape(B, T, NH, NKVH, Da, r);
  if (st != LTVQKV_OK) return st;
  if (B == 0) return LTVQKV_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int H = NH + 2 * NKVH;
  const int D = Da * r;
  if (T == 0) {
    // No outputs: d inits is zero, d bias unchanged.
    if (!grad_inits) return LTVQKV_ERR_INVALID_ARG;
    long long n = (long long)B * H * D;
    zero_grad_inits_kernel<<<(unsigned int)((n + 255) / 256), 256, 0, s>>>(grad_inits, n, dtype == LTVQKV_DTYPE_BF16);
    return ltvqkv_host::check_launch();
  }
  if (!combined || !inits || !logit_bias || !grad_combined || !grad_inits || !grad_logit_bias)
    return LTVQKV_ERR_INVALID_ARG;
  if ((NH > 0 && (!hq || !grad_hq || !hq_strides || !gq_strides)) ||
      (NKVH > 0 && (!hk || !hv || !grad_hk || !grad_hv || !hk_strides || !hv_strides || !gk_strides || !gv_strides)))
    return LTVQKV_ERR_INVALID_ARG;
  ScanGeometry g = make_geometry(B, T, NH, NKVH, Da, r, kBwdBudget);
  ScanWorkspaceLayout wl = scan_ws_layout(g);
  if (!workspace || workspace_bytes < wl.total) return LTVQKV_ERR_WORKSPACE;
  char* ws = reinterpret_cast<char*>(workspace);
  ScanBwdArgs a;
  a.combined = combined; a.sc_b = sc_b; a.sc_t = sc_t; a.sc_e = sc_e;
  a.inits = inits; a.logit_bias = logit_bias;
  a.h[0] = hq; a.h[1] = hk; a.h[2] = hv;
  a.gh[0] = grad_hq; a.gh[1] = grad_hk; a.gh[2] = grad_hv;
  const int64_t* hs[3] = {hq_strides, hk_strides, hv_strides};
  const int64_t* gs[3] = {gq_strides, gk_strides, gv_strides};
  for (int i = 0; i < 3; ++i)
    for (int k = 0; k < 4; ++k) {
      a.hs[i][k] = hs[i] ? hs[i][k] : 0;
      a.gs[i][k] = gs[i] ? gs[i][k] : 0;
    }
  a.grad_combined = grad_combined; a.gc_b = gc_b; a.gc_t = gc_t; a.gc_e = gc_e;
  a.grad_inits = grad_inits;
  a.g = g; a.use_sigmoid = use_sigmoid;
  a.ws = reinterpret_cast<WorkspaceHeader*>(ws);
  a.flags = reinterpret_cast<unsigned int*>(ws + wl.flags);
  a.aggA = reinterpret_cast<float*>(ws + wl.aggA);
  a.aggX = reinterpret_cast<float*>(ws + wl.aggX);
  a.inclX = reinterpret_cast<float*>(ws + wl.inclX);
  a.bias_part = reinterpret_cast<float*>(ws + wl.bias_part);
  if (dtype == LTVQKV_DTYPE_F32) {
    ExactArgs e = {};
    e.combined = reinterpret_cast<const float*>(combined); e.sc_b = sc_b; e.sc_t = sc_t; e.sc_e = sc_e;
    e.inits = reinterpret_cast<const float*>(inits); e.logit_bias = logit_bias;
    const void* hh[3] = {hq, hk, hv};
    const void* gg[3] = {grad_hq, grad_hk, grad_hv};
    for (int i = 0; i < 3; ++i) {
      e.h[i] = reinterpret_cast<const float*>(hh[i]);
      e.gh[i] = reinterpret_cast<const float*>(gg[i]);
      for (int k = 0; k < 4; ++k) { e.hs[i][k] = a.hs[i][k]; e.gs[i][k] = a.gs[i][k]; }
    }
    e.grad_combined = reinterpret_cast<float*>(grad_combined); e.gc_b = gc_b; e.gc_t = gc_t; e.gc_e = gc_e;
    e.grad_inits = reinterpret_cast<float*>(grad_inits);
    e.bias_part = a.bias_part;
    e.B = B; e.T = T; e.NH = NH; e.NKVH = NKVH; e.Da = Da; e.r = r; e.D = D; e.H = H; e.use_sigmoid = use_sigmoid;
    int threads = (D + 31) / 32 * 32;
    scan_bwd_exact_kernel<<<(unsigned int)(B * H), threads, sizeof(float) * threads, s>>>(e);
    int rc = ltvqkv_host::check_launch();
    if (rc != LTVQKV_OK) return rc;
    bias_reduce_exact_kernel<<<(H * Da + 127) / 128, 128, 0, s>>>(a.bias_part, grad_logit_bias, B, H, Da);
    return ltvqkv_host::check_launch();
  }
  {
    auto rows_ok = [&](const void* p, const int64_t* st) {
      return p == nullptr || (aligned16p(p) && st[3] == 1 && st[0] % 8 == 0 && st[1] % 8 == 0 && st[2] % 8 == 0);
    };
    const int tpg = r / 32;
    const bool r_ok = r % 32 == 0 && tpg >= 1 && (tpg & (tpg - 1)) == 0;
    {
      bool used = false;
      const int rc = try_row_bwd(used, dtype, combined, sc_b, sc_t, sc_e, inits, logit_bias, hq, hq_strides, hk,
                                 hk_strides, hv, hv_strides, grad_hq, gq_strides, grad_hk, gk_strides, grad_hv,
                                 gv_strides, grad_combined, gc_b, gc_t, gc_e, grad_inits, grad_logit_bias, B, T, NH,
                                 NKVH, Da, r, use_sigmoid, ws, workspace_bytes, s);
      if (used) return rc;
    }
    if (dtype == LTVQKV_DTYPE_BF16 && r_ok && fast_shape_ok(T, Da, r) && sc_t == 1 && sc_e % 8 == 0 &&
        sc_b % 8 == 0 && gc_t == 1 && gc_e % 8 == 0 && gc_b % 8 == 0 && aligned16p(combined) &&
        aligned16p(grad_combined) && aligned16p(inits) && rows_ok(hq, hq_strides) && rows_ok(grad_hq, gq_strides) &&
        (NKVH == 0 || (rows_ok(hk, hk_strides) && rows_ok(hv, hv_strides) && rows_ok(grad_hk, gk_strides) &&
                       rows_ok(grad_hv, gv_strides)))) {
      const ScanGeometry gx = fast_geometry(B, T, NH, NKVH, Da, r);
      const ScanWorkspaceLayout wx = scan_ws_layout(gx);
      if (workspace_bytes < wx.total) return LTVQKV_ERR_WORKSPACE;
      FastBwdArgs f;
      f.combined = reinterpret_cast<const __nv_bfloat16*>(combined); f.sc_b = sc_b; f.sc_e = sc_e;
      f.inits = reinterpret_cast<const __nv_bfloat16*>(inits); f.logit_bias = logit_bias;
      const void* hh[3] = {hq, hk, hv};
      const void* gg[3] = {grad_hq, grad_hk, grad_hv};
      for (int i = 0; i < 3; ++i) {
        f.h[i] = reinterpret_cast<const __nv_bfloat16*>(hh[i]);
        f.gh[i] = reinterpret_cast<const __nv_bfloat16*>(gg[i]);
        for (int k = 0; k < 3; ++k) { f.hs[i][k] = a.hs[i][k]; f.gs[i][k] = a.gs[i][k]; }
      }
      f.grad_combined = reinterpret_cast<__nv_bfloat16*>(grad_combined); f.gc_b = gc_b; f.gc_e = gc_e;
      f.grad_inits = reinterpret_cast<__nv_bfloat16*>(grad_inits);
      f.bias_part = reinterpret_cast<float*>(ws + wx.bias_part);
      f.B = B; f.T = T; f.NH = NH; f.NKVH = NKVH; f.Da = Da; f.r = r; f.D = gx.D; f.H = gx.H;
      f.nchunks = gx.nchunks; f.use_sigmoid = use_sigmoid;
      f.ws = reinterpret_cast<WorkspaceHeader*>(ws);
      f.flags = reinterpret_cast<unsigned int*>(ws + wx.flags);
      f.aggA = reinterpret_cast<float*>(ws + wx.aggA);
      f.aggX = reinterpret_cast<float*>(ws + wx.aggX);
      f.inclX = reinterpret_cast<float*>(ws + wx.inclX);
      const size_t fsm = fast_bwd_smem_bytes(gx.D, Da);
      auto kern = gx.D <= 128 ? scan_bwd_fast_kernel<256, kFastBwdMinBlocks256> : scan_bwd_fast_kernel<512, 2>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fsm);
      kern<<<(unsigned int)((long long)B * gx.H * gx.nchunks), 2 * gx.D, fsm, s>>>(f);
      int rc = ltvqkv_host::check_launch();
      if (rc != LTVQKV_OK) return rc;
      bias_reduce_kernel<<<H * Da, kBiasReduceThreads, 0, s>>>(f.bias_part, grad_logit_bias, B, gx.nchunks, H, Da);
      return ltvqkv_host::check_launch();
    }
  }
  size_t smem = bwd_smem_bytes(g);
  unsigned int grid = (unsigned int)((long long)B * g.H * g.nchunks);
  if (dtype == LTVQKV_DTYPE_BF16) {
    cudaFuncSetAttribute(scan_bwd_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    scan_bwd_kernel<__nv_bfloat16><<<grid, g.nthreads, smem, s>>>(a);
  } else {
    cudaFuncSetAttribute(scan_bwd_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    scan_bwd_kernel<float><<<grid, g.nthreads, smem, s>>>(a);
  }
  int rc = ltvqkv_host::check_launch();
  if (rc != LTVQKV_OK) return rc;
  bias_reduce_kernel<<<H * Da, kBiasReduceThreads, 0, s>>>(a.bias_part, grad_logit_bias, B, g.nchunks, H, Da);
  return ltvqkv_host::check_launch();
}

// Scan backward from the forward's state checkpoints (ltvqkv_proj_scan_fwd_ckpt) instead of its
// outputs: the row-streaming kernel replays each 32-token chunk's outputs from the stored fp32 state.
// Results equal ltvqkv_scan_bwd's bit for bit (grad_logit_bias overwritten, not added to; with a
// shared initial state the per-sequence initial-state gradients summed in batch order); shapes or
// layouts that kernel does not take return LTVQKV_ERR_UNSUPPORTED before anything is launched.
extern "C" int ltvqkv_scan_bwd_ckpt(int dtype, const void* combined, int64_t sc_b, int64_t sc_t, int64_t sc_e,
                                    const void* inits, int64_t inits_bs, const float* logit_bias, const float* ckpt,
                                    const void* grad_hq, const int64_t* gq_strides, const void* grad_hk,
                                    const int64_t* gk_strides, const void* grad_hv, const int64_t* gv_strides,
                                    void* grad_combined, int64_t gc_b, int64_t gc_t, int64_t gc_e, void* grad_inits,
                                    float* grad_logit_bias, int B, int T, int NH, int NKVH, int Da, int r,
                                    int use_sigmoid, void* workspace, size_t workspace_bytes, void* stream) {
  if (!ltvqkv_host::valid_dtype(dtype)) return LTVQKV_ERR_DTYPE;
  int st = validate_scan_shape(B, T, NH, NKVH, Da, r);
  if (st != LTVQKV_OK) return st;
  if (!combined || !inits || !logit_bias || !ckpt || !grad_combined || !grad_inits || !grad_logit_bias)
    return LTVQKV_ERR_INVALID_ARG;
  if ((NH > 0 && (!grad_hq || !gq_strides)) || (NKVH > 0 && (!grad_hk || !grad_hv || !gk_strides || !gv_strides)))
    return LTVQKV_ERR_INVALID_ARG;
  if (B == 0 || T == 0) return LTVQKV_ERR_UNSUPPORTED;
  if (!workspace) return LTVQKV_ERR_WORKSPACE;
  const int64_t HD = (int64_t)(NH + 2 * NKVH) * Da * r;
  if (inits_bs != 0 && inits_bs != HD) return LTVQKV_ERR_STRIDE;
  const bool shared = inits_bs == 0;
  static const int64_t kNone[4] = {0, 0, 0, 1};
  bool used = false;
  const int rc = try_row_bwd(used, dtype, combined, sc_b, sc_t, sc_e, inits, logit_bias, nullptr, kNone, nullptr,
                             kNone, nullptr, kNone, grad_hq, gq_strides, grad_hk, gk_strides, grad_hv, gv_strides,
                             grad_combined, gc_b, gc_t, gc_e, shared ? nullptr : grad_inits, grad_logit_bias, B, T,
                             NH, NKVH, Da, r, use_sigmoid, reinterpret_cast<char*>(workspace), workspace_bytes,
                             reinterpret_cast<cudaStream_t>(stream), ckpt, shared,
                             shared ? reinterpret_cast<float*>(grad_inits) : nullptr, true);
  return used ? rc : LTVQKV_ERR_UNSUPPORTED;
}

// ------------------------------------------------------------------------------------------
// Allocation-free forward scan.
//
// For callers that cannot allocate device memory on the call path: plugin hosts and serving
// runtimes that own every byte of device memory under a fixed plan, or foreign-language callers
// without access to an allocator. The look-back scratch of the forward scan lives in the
// file-scope array below instead of a caller workspace. Its size is fixed at
// kNoAllocScratchBytes (32 MiB); every GPU that loads this library holds it until the process
// exits. Problems whose forward-scan scratch would exceed it are rejected with
// LTVQKV_ERR_TOO_LARGE before anything is launched.
//
// Host code must not pass the array's name to a kernel (on the host it is only a stand-in for
// the device symbol); the first call on each device looks up the array's device address with
// cudaGetSymbolAddress while that device is current, checks the result and caches it. That
// first call may cause the driver to load this library's device code on that device, so it
// should come before any stream capture. Every call clears the part of the array that must
// start at zero (header counters and epoch, look-back flags) with cudaMemsetAsync on the
// caller's stream; all calls share the array, so calls that overlap on the GPU race with each
// other and must be serialised by the caller (one stream, or events).
// ------------------------------------------------------------------------------------------
namespace {
constexpr size_t kNoAllocScratchBytes = (size_t)32 << 20;
__device__ __align__(256) unsigned char g_scan_noalloc_scratch[kNoAllocScratchBytes];
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};
}  // namespace

namespace ltvqkv_host {
// Device address of the allocation-free array on the current device, looked up once per device with
// cudaGetSymbolAddress (the host-side name of a __device__ array is not a device address).
int noalloc_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return LTVQKV_ERR_LAUNCH;
  }
  if (dev < 0 || dev >= kNoAllocMaxDevices) return LTVQKV_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  void* ptr = g_noalloc_ptr[dev];
  if (ptr == nullptr) {
    e = cudaGetSymbolAddress(&ptr, g_scan_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr) {
      set_last_cuda_error(e);
      return LTVQKV_ERR_LAUNCH;
    }
    g_noalloc_ptr[dev] = ptr;
  }
  *out = ptr;
  return LTVQKV_OK;
}
}  // namespace ltvqkv_host

extern "C" int ltvqkv_scan_fwd_noalloc(int dtype, const void* combined, int64_t sc_b, int64_t sc_t, int64_t sc_e,
                                       const void* inits, const float* logit_bias, void* out_q, void* out_k,
                                       void* out_v, int B, int T, int NH, int NKVH, int Da, int r, int use_sigmoid,
                                       void* stream) {
  if (!ltvqkv_host::valid_dtype(dtype)) return LTVQKV_ERR_DTYPE;
  int st = validate_scan_shape(B, T, NH, NKVH, Da, r);
  if (st != LTVQKV_OK) return st;
  if (B == 0 || T == 0) return LTVQKV_OK;
  const ScanWorkspaceLayout wl = scan_ws_layout(make_geometry(B, T, NH, NKVH, Da, r, kFwdBudget));
  const ScanWorkspaceLayout wx = scan_ws_layout(fast_geometry(B, T, NH, NKVH, Da, r));
  if (std::max(wl.total, wx.total) > kNoAllocScratchBytes) return LTVQKV_ERR_TOO_LARGE;
  void* ptr = nullptr;
  st = ltvqkv_host::noalloc_scratch(&ptr);
  if (st != LTVQKV_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // The ticket/exit counters and the epoch (the header's first 12 bytes) and the look-back flags must
  // start at zero. The header's error words are left alone: a timed-out wait of an earlier call stays
  // recorded until ltvqkv_scan_noalloc_error reads it.
  static_assert(offsetof(WorkspaceHeader, error) == 12, "counters and epoch precede the error word");
  cudaError_t e = cudaMemsetAsync(ptr, 0, offsetof(WorkspaceHeader, error), s);
  const size_t flags_end = std::max(wl.aggA, wx.aggA);
  if (e == cudaSuccess)
    e = cudaMemsetAsync(static_cast<char*>(ptr) + sizeof(WorkspaceHeader), 0, flags_end - sizeof(WorkspaceHeader), s);
  if (e != cudaSuccess) {
    ltvqkv_host::set_last_cuda_error(e);
    return LTVQKV_ERR_LAUNCH;
  }
  return ltvqkv_scan_fwd(dtype, combined, sc_b, sc_t, sc_e, inits, logit_bias, out_q, out_k, out_v, B, T, NH, NKVH,
                         Da, r, use_sigmoid, ptr, kNoAllocScratchBytes, stream);
}

// Error word of the allocation-free array: a bounded device-side wait inside ltvqkv_scan_fwd_noalloc
// that gave up records LTVQKV_ERR_TIMEOUT there; this reads and clears it like ltvqkv_workspace_error.
extern "C" int ltvqkv_scan_noalloc_error(void* stream, uint32_t* err_out) {
  if (!err_out) return LTVQKV_ERR_INVALID_ARG;
  void* ptr = nullptr;
  const int st = ltvqkv_host::noalloc_scratch(&ptr);
  if (st != LTVQKV_OK) return st;
  return ltvqkv_workspace_error(ptr, stream, err_out);
}
