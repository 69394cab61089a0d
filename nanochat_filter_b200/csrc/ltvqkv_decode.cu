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

#include <mutex>

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

// bf16 path: per (head, 16-channel slice) CTA, the [tokens x projection rows] block is one small
// GEMM on the tensor cores (mma.sync m16n8k16, fp32 accumulation) from shared-memory copies of the
// slice's W rows and a 64-token tile of x, instead of one warp-wide dot product per (row, token).
// The copies are 16-byte cp.async pieces issued by all threads at once (one wait for the whole
// tile). 8 warps: warp w owns tokens 16 (w / 2) .. +15 and projection rows 16 (w % 2) .. +15. Rows
// are padded to 32 (16 value rows + up to 16 logit rows of the slice's groups), tokens to 64, K to
// a multiple of 16 (zeros); shared-memory rows are padded by 16 bytes so that ldmatrix is
// conflict-free. A GEMM of 64 x 32 x C per CTA is too small for tcgen05's 128-row tiles.
constexpr int kDmTok = 64;
constexpr int kDmSlice = 16;
constexpr int kDmRows = 32;
constexpr int kDmNt = kDmRows / 8 / 2;  // n-tiles (8 rows) per warp

LTVQKV_DEVICE void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
LTVQKV_DEVICE void ldsm_x2(uint32_t addr, uint32_t (&r)[2]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}
LTVQKV_DEVICE void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__global__ void __launch_bounds__(kDecThreads) decode_step_mma_kernel(DecodeArgs a, int Cp) {
  extern __shared__ __align__(16) unsigned char dm_smem[];
  const int ld = Cp + 8;  // elements per shared row
  __nv_bfloat16* sW = reinterpret_cast<__nv_bfloat16*>(dm_smem);
  __nv_bfloat16* sX = sW + (size_t)kDmRows * ld;
  float* res = reinterpret_cast<float*>(sX + (size_t)kDmTok * ld);  // [kDmTok][kDmRows]
  const int h = blockIdx.x;
  const int c0 = blockIdx.y * kDmSlice;
  const int c1 = min(c0 + kDmSlice, a.D);
  const int nv = c1 - c0;
  const int g0 = c0 / a.r, g1 = (c1 - 1) / a.r;
  const int rows = nv + g1 - g0 + 1;  // <= kDmRows (callers with r < 2 take the other kernel)
  const int head_row = h * (a.D + a.Da);
  const __nv_bfloat16* X = reinterpret_cast<const __nv_bfloat16*>(a.x);
  const __nv_bfloat16* W = reinterpret_cast<const __nv_bfloat16*>(a.w);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const bool vec = (a.C % 8) == 0 && ((reinterpret_cast<uintptr_t>(X) | reinterpret_cast<uintptr_t>(W)) & 15) == 0;
  int which, hloc;
  dec_split_head(h, a.NH, a.NKVH, which, hloc);
  // one warp per shared row, lanes along the row in 16-byte pieces (no index divisions)
  auto stage_row = [&](__nv_bfloat16* dst, const __nv_bfloat16* src, bool live) {
    for (int k = lane * 8; k < Cp; k += 256) {
      if (live && k < a.C) {
        if (vec) cp_async16(dst + k, src + k);
        else
          for (int e = 0; e < 8; ++e) dst[k + e] = k + e < a.C ? src[k + e] : __float2bfloat16_rn(0.f);
      } else {
        *reinterpret_cast<uint4*>(dst + k) = make_uint4(0, 0, 0, 0);
      }
    }
  };
  // the slice's projection rows: value rows c0 .. c1-1, then the logit rows of groups g0 .. g1
  for (int row = warp; row < kDmRows; row += kDecThreads / 32) {
    const int wrow = row < nv ? head_row + c0 + row : head_row + a.D + g0 + (row - nv);
    stage_row(sW + (size_t)row * ld, W + (long long)(row < rows ? wrow : 0) * a.C, row < rows);
  }
  const int mt = warp / 2, nb0 = (warp % 2) * kDmNt;  // this warp's 16 tokens, kDmNt x 8 rows
  const uint32_t sX_u = smem_u32(sX), sW_u = smem_u32(sW);
  for (int b0 = 0; b0 < a.B; b0 += kDmTok) {
    const int nb = min(kDmTok, a.B - b0);
    for (int tk = warp; tk < kDmTok; tk += kDecThreads / 32)
      stage_row(sX + (size_t)tk * ld, X + (long long)(b0 + min(tk, nb - 1)) * a.C, tk < nb);
    cp_async_wait_all();
    __syncthreads();
    float acc[kDmNt][4] = {};
    const uint32_t a_addr = sX_u + (uint32_t)(((16 * mt + (lane % 16)) * ld + (lane / 16) * 8) * 2);
    uint32_t b_addr[kDmNt];
#pragma unroll
    for (int j = 0; j < kDmNt; ++j)
      b_addr[j] = sW_u + (uint32_t)(((8 * (nb0 + j) + (lane % 8)) * ld + ((lane / 8) % 2) * 8) * 2);
    for (int k = 0; k < Cp; k += 16) {
      uint32_t af[4], bf[kDmNt][2];
      ldsm_x4(a_addr + (uint32_t)(k * 2), af);
#pragma unroll
      for (int j = 0; j < kDmNt; ++j) ldsm_x2(b_addr[j] + (uint32_t)(k * 2), bf[j]);
#pragma unroll
      for (int j = 0; j < kDmNt; ++j) mma_bf16_16816(acc[j], af, bf[j]);
    }
    // fragment (token 16 mt + lane/4 (+8), row 8 n + 2 (lane % 4) (+1)) -> res[token][row]
#pragma unroll
    for (int j = 0; j < kDmNt; ++j) {
      const int rr = 8 * (nb0 + j) + 2 * (lane % 4), tt = 16 * mt + lane / 4;
      *reinterpret_cast<float2*>(&res[tt * kDmRows + rr]) = make_float2(acc[j][0], acc[j][1]);
      *reinterpret_cast<float2*>(&res[(tt + 8) * kDmRows + rr]) = make_float2(acc[j][2], acc[j][3]);
    }
    __syncthreads();
    // consecutive threads take consecutive channels of one token: the state reads and writes of
    // a token's slice are one contiguous 32-byte piece
    for (int i = threadIdx.x; i < nv * nb; i += kDecThreads) {
      const int bb = i / nv, cc = i - (i / nv) * nv;
      const int c = c0 + cc, b = b0 + bb;
      const int g = c / a.r;
      // projection values rounded to bf16, as the reference's projection buffer stores them
      const float u = __bfloat162float(__float2bfloat16_rn(res[bb * kDmRows + cc]));
      const float l = __fadd_rn(__bfloat162float(__float2bfloat16_rn(res[bb * kDmRows + nv + g - g0])),
                                a.logit_bias[h * a.Da + g]);
      const float al = a.use_sigmoid ? sigmoid_f32(l) : l;
      float hp;
      if (a.prev[0] != nullptr) {
        const long long* ps = a.ps[which];
        hp = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.prev[which])[b * ps[0] + hloc * ps[1] + c * ps[2]]);
      } else {
        hp = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.init_param)[(long long)h * a.D + c]);
      }
      const float hn = __fadd_rn(__fmul_rn(__fsub_rn(1.0f, al), hp), __fmul_rn(al, u));
      const long long* os = a.os[which];
      reinterpret_cast<__nv_bfloat16*>(a.out[which])[b * os[0] + hloc * os[1] + c * os[2]] = __float2bfloat16_rn(hn);
    }
    __syncthreads();
  }
}

size_t decode_mma_smem(int Cp) { return (size_t)(kDmRows + kDmTok) * (Cp + 8) * 2 + (size_t)kDmRows * kDmTok * 4; }

// bf16 path for C % 64 == 0 (the model widths): the same (head, 16-channel slice) CTAs, with
//   * K cut into nq parts (4 when C/64 divides by 4, else 2 or 1), each part staged by bulk tensor
//     copies issued from its own warp onto its own mbarrier: the part's k-blocks of the 64-token
//     tile of x (one 128-byte-swizzled box [C/64/nq][64 tokens][64]), of the slice's value rows and
//     of its logit rows; copies from several warps run side by side (one thread issues about one copy
//     per few hundred cycles whatever its size), and the warps of a part start multiplying as soon as
//     that part has landed;
//   * the previous state of the thread's outputs loaded into registers while the copies land;
//   * 16 warps: warp w < 4 nq multiplies tokens 16 (w % 4) .. +15 by all 24 rows (3 independent
//     accumulator chains) over K part w / 4, and the parts are added in fixed order (part 0 + part 1
//     + ...), so a warp's chain is 48 / nq k-steps and results do not depend on timing;
//   * programmatic dependent launch: the next kernel on the stream may be scheduled while this one
//     runs; this grid's global reads wait for the previous kernel's completion (griddepcontrol.wait).
// The projection values and logits are rounded to bf16 exactly as the reference's projection
// buffer stores them, then the gate and the recurrence step as in the other paths.
constexpr int kDtTok = 64;      // tokens per tile (one box)
constexpr int kDtRows = 24;     // 16 value rows + up to 8 logit rows (r >= 2)
constexpr int kDtRegion = 1024; // swizzle atoms start on 1 KB boundaries
constexpr int kDtMaxParts = 4;

struct DecodeTmaLayout {
  size_t x, wv, wl, wl_part, red, bar, total;
};
// Every box lands on a 1 KB boundary (the 128-byte swizzle's atom): x and the value rows per part
// are whole multiples of it; the logit rows of each part get their own 1 KB-rounded slot.
__host__ __device__ inline DecodeTmaLayout decode_tma_layout(int nkb, int nq) {
  DecodeTmaLayout L;
  size_t off = 0;
  L.x = off; off += (size_t)nkb * kDtTok * 128;
  L.wv = off; off += (size_t)nkb * 16 * 128;
  L.wl_part = ((size_t)(nkb / nq) * 8 * 128 + kDtRegion - 1) / kDtRegion * kDtRegion;
  L.wl = off; off += (size_t)nq * L.wl_part;
  L.red = off; off += (size_t)(nq > 1 ? nq - 1 : 1) * kDtTok * kDtRows * 4;
  L.bar = off; off += 8 * kDtMaxParts;
  L.total = off + kDtRegion;  // alignment slack of the dynamic shared memory base
  return L;
}
inline int decode_tma_parts(int nkb) { return nkb % 4 == 0 ? 4 : (nkb % 2 == 0 ? 2 : 1); }

// Byte offset of the 16-byte piece `chunk` of 128-byte row `row` in a 128B-swizzled region.
LTVQKV_DEVICE uint32_t swz128(int row, int chunk) { return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4)); }

__global__ void __launch_bounds__(32 * 4 * kDtMaxParts, 1)
    decode_step_tma_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                           const __grid_constant__ CUtensorMap tmWl, DecodeArgs a, int nkb, int ngb, int nq) {
  extern __shared__ __align__(16) unsigned char dt_raw[];
  unsigned char* smem = smem_align<unsigned char>(dt_raw, kDtRegion);
  const DecodeTmaLayout L = decode_tma_layout(nkb, nq);
  unsigned char* sX = smem + L.x;
  unsigned char* sWv = smem + L.wv;
  unsigned char* sWl = smem + L.wl;
  float* red = reinterpret_cast<float*>(smem + L.red);  // [nq - 1][kDtTok][kDtRows]
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);  // [nq]
  __shared__ volatile int abort_flag;
  const int h = blockIdx.x;
  const int c0 = blockIdx.y * kDmSlice;
  const int nv = min(kDmSlice, a.D - c0);
  const int g0 = c0 / a.r;
  const int head_row = h * (a.D + a.Da);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nthr = blockDim.x;
  const int kpq = nkb / nq;  // k-blocks per part
  int which, hloc;
  dec_split_head(h, a.NH, a.NKVH, which, hloc);
  // Launched with programmatic stream serialisation: the next kernel on the stream may be scheduled
  // now (its CTAs set up while this grid runs), and this grid's own global reads wait below until
  // the previous kernel on the stream has completed and its writes are visible — every global read
  // of this kernel (weights included: a cast kernel may have just written them) comes after that.
  griddep_launch_dependents();
  if (threadIdx.x == 0) {
    for (int q = 0; q < nq; ++q) mbar_init(&bar[q], 1);
    abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmWl);
  }
  __syncthreads();
  griddep_wait();
  const int mt = warp % 4, kq = warp / 4;
  const uint32_t sX_u = smem_u32(sX), sWv_u = smem_u32(sWv), sWl_u = smem_u32(sWl);
  uint32_t phase = 0;
  for (int b0 = 0; b0 < a.B; b0 += kDtTok, phase ^= 1u) {
    const int nb = min(kDtTok, a.B - b0);
    const bool first = b0 == 0;
    // part q's copies: x from lane 0 of warp q (every tile, with the part's byte count), the W rows
    // from lane 0 of warp 4 + q (first tile only), so that eight threads issue side by side
    if (lane == 0 && warp < nq) {
      const int z = warp * kpq;
      const uint32_t bytes = (uint32_t)kpq * 128u * (kDtTok + (first ? 16u + (uint32_t)ngb : 0u));
      mbar_arrive_expect_tx(&bar[warp], bytes);
      tma_load_3d(sX + (size_t)z * kDtTok * 128, &tmX, &bar[warp], 0, b0, z);
    } else if (lane == 0 && first && warp >= 4 && warp < 4 + nq) {
      const int q = warp - 4, z = q * kpq;
      tma_load_3d(sWv + (size_t)z * 16 * 128, &tmW, &bar[q], 0, head_row + c0, z);
      tma_load_3d(sWl + (size_t)q * L.wl_part, &tmWl, &bar[q], 0, head_row + a.D + g0, z);
    }
    // this thread's previous states and logit biases, while the copies land
    float hp[2], lbj[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = threadIdx.x + j * nthr;
      hp[j] = 0.f;
      lbj[j] = 0.f;
      if (i < nv * nb) {
        lbj[j] = a.logit_bias[h * a.Da + (c0 + (i - (i / nv) * nv)) / a.r];
        const int bb = i / nv, c = c0 + (i - bb * nv), b = b0 + bb;
        if (a.prev[0] != nullptr) {
          const long long* ps = a.ps[which];
          hp[j] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.prev[which])[b * ps[0] + hloc * ps[1] + c * ps[2]]);
        } else {
          hp[j] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.init_param)[(long long)h * a.D + c]);
        }
      }
    }
    // tokens 16 mt .. +15 x rows 0..23 over the k-blocks of part kq, once they have landed (warps
    // beyond 4 nq only help with the epilogue)
    const bool got = kq < nq ? mbar_wait(&bar[kq], phase, &abort_flag, nullptr, 0x7e01) : true;
    if (__syncthreads_or(got ? 0 : 1)) break;  // every warp leaves together
    float acc[3][4] = {};
    const int arow = 16 * mt + (lane % 16);
    const int brow = lane % 8;
    const int lrow = brow < ngb ? brow : 0;  // logit rows beyond the slice's groups: any row (unused columns)
    const uint32_t sWlq = sWl_u + (uint32_t)(kq * L.wl_part);
    for (int kb = kq * kpq; kq < nq && kb < (kq + 1) * kpq; ++kb) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t af[4], b0f[2], b1f[2], blf[2];
        ldsm_x4(sX_u + (uint32_t)kb * (kDtTok * 128) + swz128(arow, kk * 2 + lane / 16), af);
        const int bc = kk * 2 + (lane / 8) % 2;
        ldsm_x2(sWv_u + (uint32_t)kb * (16 * 128) + swz128(brow, bc), b0f);
        ldsm_x2(sWv_u + (uint32_t)kb * (16 * 128) + swz128(8 + brow, bc), b1f);
        ldsm_x2(sWlq + swz128((kb - kq * kpq) * ngb + lrow, bc), blf);
        mma_bf16_16816(acc[0], af, b0f);
        mma_bf16_16816(acc[1], af, b1f);
        mma_bf16_16816(acc[2], af, blf);
      }
    }
    // the parts, added in fixed order: part 0 + part 1 + ... (parts 1.. through red)
    const int tt = 16 * mt + lane / 4, rr = 2 * (lane % 4);
    if (kq > 0 && kq < nq) {
      float* rq = red + (size_t)(kq - 1) * kDtTok * kDtRows;
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        *reinterpret_cast<float2*>(&rq[tt * kDtRows + 8 * j + rr]) = make_float2(acc[j][0], acc[j][1]);
        *reinterpret_cast<float2*>(&rq[(tt + 8) * kDtRows + 8 * j + rr]) = make_float2(acc[j][2], acc[j][3]);
      }
    }
    __syncthreads();
    if (kq == 0) {
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        float s0 = acc[j][0], s1 = acc[j][1], s2 = acc[j][2], s3 = acc[j][3];
        for (int q = 1; q < nq; ++q) {
          const float* rq = red + (size_t)(q - 1) * kDtTok * kDtRows;
          const float2 q0 = *reinterpret_cast<const float2*>(&rq[tt * kDtRows + 8 * j + rr]);
          const float2 q1 = *reinterpret_cast<const float2*>(&rq[(tt + 8) * kDtRows + 8 * j + rr]);
          s0 += q0.x; s1 += q0.y; s2 += q1.x; s3 += q1.y;
        }
        // the sum lands in part 1's slot (or in red itself with one part)
        *reinterpret_cast<float2*>(&red[tt * kDtRows + 8 * j + rr]) = make_float2(s0, s1);
        *reinterpret_cast<float2*>(&red[(tt + 8) * kDtRows + 8 * j + rr]) = make_float2(s2, s3);
      }
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = threadIdx.x + j * nthr;
      if (i < nv * nb) {
        const int bb = i / nv, cc = i - bb * nv;
        const int c = c0 + cc, b = b0 + bb;
        const int g = c / a.r;
        // projection values rounded to bf16, as the reference's projection buffer stores them
        const float u = __bfloat162float(__float2bfloat16_rn(red[bb * kDtRows + cc]));
        const float l = __fadd_rn(__bfloat162float(__float2bfloat16_rn(red[bb * kDtRows + 16 + g - g0])), lbj[j]);
        const float al = a.use_sigmoid ? sigmoid_f32(l) : l;
        const float hn = __fadd_rn(__fmul_rn(__fsub_rn(1.0f, al), hp[j]), __fmul_rn(al, u));
        const long long* os = a.os[which];
        reinterpret_cast<__nv_bfloat16*>(a.out[which])[b * os[0] + hloc * os[1] + c * os[2]] = __float2bfloat16_rn(hn);
      }
    }
    __syncthreads();  // red and sX are free for the next token tile
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
  const int Cp = (C + 15) / 16 * 16;
  const size_t smem = decode_mma_smem(Cp);
  // the tensor-core paths hold a slice's logit rows next to its value rows: r >= 2 keeps them <= 16
  const bool rows_fit = (kDmSlice + kDmSlice / r + 1) <= kDmRows;
  const int nkb = C / 64;
  // a 16-channel slice (starting at a multiple of 16) covers one decay group when 16 divides r, and
  // 16 / r whole groups when r divides 16; other r take the paths below
  const bool slice_groups = (r % kDmSlice == 0) || (kDmSlice % r == 0 && r >= 2);
  const int ngb = r >= kDmSlice ? 1 : kDmSlice / r;  // logit rows of a slice (<= 8)
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(weight)) & 15) == 0;
  const int nq = decode_tma_parts(nkb > 0 ? nkb : 1);
  if (dtype == LTVQKV_DTYPE_BF16 && slice_groups && C % 64 == 0 && nkb >= 1 && nkb <= 256 && aligned &&
      decode_tma_layout(nkb, nq).total <= 220 * 1024) {
    const int F = a.H * (a.D + Da);
    const uint64_t dx[3] = {64, (uint64_t)B, (uint64_t)nkb}, sx[2] = {(uint64_t)C * 2, 128};
    const uint64_t dw[3] = {64, (uint64_t)F, (uint64_t)nkb}, sw[2] = {(uint64_t)C * 2, 128};
    // boxes of one K part (nkb / nq k-blocks)
    const uint32_t kp = (uint32_t)(nkb / nq);
    const uint32_t bx[3] = {64, (uint32_t)kDtTok, kp}, bw[3] = {64, 16, kp}, bl[3] = {64, (uint32_t)ngb, kp};
    CUtensorMap tmX, tmW, tmWl;
    if (!ltvqkv_host::encode_tiled_map(&tmX, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, x, dx, sx, bx, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !ltvqkv_host::encode_tiled_map(&tmW, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, weight, dw, sw, bw,
                                       CU_TENSOR_MAP_SWIZZLE_128B) ||
        !ltvqkv_host::encode_tiled_map(&tmWl, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, weight, dw, sw, bl,
                                       CU_TENSOR_MAP_SWIZZLE_128B))
      return LTVQKV_ERR_LAUNCH;
    const size_t tsm = decode_tma_layout(nkb, nq).total;
    static std::mutex mu3;
    static size_t opted3[64] = {};  // dynamic shared memory this kernel is opted into, per device
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ltvqkv_host::check_launch();
    {
      std::lock_guard<std::mutex> lock(mu3);
      if (opted3[dev] < tsm) {
        if (cudaFuncSetAttribute(decode_step_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tsm) !=
            cudaSuccess)
          return ltvqkv_host::check_launch();
        opted3[dev] = tsm;
      }
    }
    // programmatic stream serialisation (see the kernel): consecutive decode steps of a graph or a
    // stream overlap one kernel's launch and set-up with the previous one's tail
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(a.H, (a.D + kDmSlice - 1) / kDmSlice);
    lc.blockDim = dim3(32 * 4 * kDtMaxParts);
    lc.dynamicSmemBytes = tsm;
    lc.stream = s;
    cudaLaunchAttribute la[1];
    la[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    la[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = la;
    lc.numAttrs = 1;
    const cudaError_t le = cudaLaunchKernelEx(&lc, decode_step_tma_kernel, tmX, tmW, tmWl, a, nkb, ngb, nq);
    if (le != cudaSuccess) {
      ltvqkv_host::set_last_cuda_error(le);
      return LTVQKV_ERR_LAUNCH;
    }
  } else if (dtype == LTVQKV_DTYPE_BF16 && smem <= 200 * 1024 && rows_fit) {
    static std::mutex mu;
    static bool done[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ltvqkv_host::check_launch();
    {
      std::lock_guard<std::mutex> lock(mu);
      if (!done[dev]) {
        if (cudaFuncSetAttribute(decode_step_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) !=
            cudaSuccess)
          return ltvqkv_host::check_launch();
        done[dev] = true;
      }
    }
    dim3 grid_mma(a.H, (a.D + kDmSlice - 1) / kDmSlice);
    decode_step_mma_kernel<<<grid_mma, kDecThreads, smem, s>>>(a, Cp);
  } else if (dtype == LTVQKV_DTYPE_BF16) {
    decode_step_kernel<__nv_bfloat16><<<grid, kDecThreads, 0, s>>>(a);
  } else {
    decode_step_kernel<float><<<grid, kDecThreads, 0, s>>>(a);
  }
  return ltvqkv_host::check_launch();
}
