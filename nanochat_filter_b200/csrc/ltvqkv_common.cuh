// Shared device/host helpers for libltvqkv (sm_100a only).
//
// Contents: bf16/fp32 load-store helpers, the workspace header used by every kernel that
// needs scratch, bounded spin-waits (every wait gives up after a wall-clock limit, records
// LTVQKV_ERR_TIMEOUT in the workspace and lets the kernel return), and thin inline-PTX
// wrappers for mbarriers, TMA (cp.async.bulk.tensor, no cluster multicast anywhere) and
// tcgen05 (TMEM alloc, MMA, commit, ld).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ltvqkv.h"  // include/ (on the -I path)

#define LTVQKV_DEVICE __device__ __forceinline__

namespace ltvqkv {

// ------------------------------------------------------------------------------------------
// Workspace header. Lives at the start of every workspace; zero-filled once by the caller.
// tile_counter / exit_counter drive dynamic tile scheduling and are reset by the last CTA of
// each launch, so the next launch on the same stream starts from zero again. `epoch` tags
// the look-back flags of the scan kernels: the last CTA bumps it, so flags written by older
// launches never match the current one and the flag array needs no clearing between calls.
// ------------------------------------------------------------------------------------------
struct WorkspaceHeader {
  unsigned int tile_counter;
  unsigned int exit_counter;
  unsigned int epoch;
  unsigned int error;
  unsigned int error_where;
  unsigned int pad[59];  // header is 256 bytes
};
static_assert(sizeof(WorkspaceHeader) == 256, "workspace header must be 256 bytes");

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s per wait

LTVQKV_DEVICE unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

LTVQKV_DEVICE void record_timeout(WorkspaceHeader* ws, unsigned int where) {
  if (ws != nullptr) {
    atomicExch(&ws->error, (unsigned int)LTVQKV_ERR_TIMEOUT);
    atomicExch(&ws->error_where, where);
  }
}

// Dynamic tile ticket: each CTA draws tiles in order; the draw that exceeds `total` returns
// total (callers stop). Launch finalisation resets the counters (see finish_launch).
LTVQKV_DEVICE unsigned int draw_ticket(WorkspaceHeader* ws) { return atomicAdd(&ws->tile_counter, 1u); }

// Called once per CTA by one thread after the CTA has drawn its last ticket and finished
// every global write whose ordering matters. The last CTA resets the counters and bumps the
// epoch for the next launch on this workspace.
// As finish_launch; returns true in the CTA that finished last (whose thread then sees every other
// CTA's writes that preceded their finish_launch, through L2).
LTVQKV_DEVICE bool finish_launch_last(WorkspaceHeader* ws, unsigned int num_ctas) {
  __threadfence();
  unsigned int done = atomicAdd(&ws->exit_counter, 1u);
  if (done == num_ctas - 1) {
    atomicExch(&ws->tile_counter, 0u);
    atomicExch(&ws->exit_counter, 0u);
    atomicAdd(&ws->epoch, 1u);
    __threadfence();
    return true;
  }
  return false;
}

// No fence before the count: nothing in the launch reads what a CTA wrote because of it (the next
// launch on the workspace is ordered after this one by the stream), so the CTA need not wait for
// its stores to be acknowledged before it exits.
LTVQKV_DEVICE void finish_launch(WorkspaceHeader* ws, unsigned int num_ctas) {
  unsigned int done = atomicAdd(&ws->exit_counter, 1u);
  if (done == num_ctas - 1) {
    atomicExch(&ws->tile_counter, 0u);
    atomicExch(&ws->exit_counter, 0u);
    atomicAdd(&ws->epoch, 1u);
    __threadfence();
  }
}

// ------------------------------------------------------------------------------------------
// Element conversion
// ------------------------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static LTVQKV_DEVICE float load(const float* p) { return *p; }
  static LTVQKV_DEVICE void store(float* p, float v) { *p = v; }
  static LTVQKV_DEVICE float to_f(float v) { return v; }
  static LTVQKV_DEVICE float from_f(float v) { return v; }
};
template <> struct Elem<__nv_bfloat16> {
  static LTVQKV_DEVICE float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static LTVQKV_DEVICE void store(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
  static LTVQKV_DEVICE float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static LTVQKV_DEVICE __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

// Logistic function evaluated with the CUDA math library's expf (the reference evaluates
// 1 / (1 + expf(-x)) in fp32, cpp_ewma/src/ltv_fused_concat_head_major_register_cast_scan_cuda_common.cuh:114-117).
LTVQKV_DEVICE float sigmoid_f32(float x) { return 1.0f / (1.0f + expf(-x)); }

// Logistic function for the fp32 exact-order path: exp evaluated in double and rounded to float
// (within half an ulp of the float result of the host's correctly-rounding expf in all but
// rare boundary cases), then the add and the divide each rounded once.
LTVQKV_DEVICE float sigmoid_f32_exact(float x) {
  const float e = (float)exp(-(double)x);
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
}

// ------------------------------------------------------------------------------------------
// Rotary embedding + RMS norm of a head row (the reference attention's prologue on the filter's q
// and k, nanochat/gpt.py:96-111, 224-230): y1 = x1 c + x2 s, y2 = x1 (-s) + x2 c on the element
// pairs (j, j + D/2), then z = y r with r = (mean(y^2) + eps)^(-1/2). Shared by the standalone
// kernels and the fused projection + scan forward / checkpoint backward, so that all of them
// compute the same values bit for bit; every step is an explicit round-to-nearest operation.
// ------------------------------------------------------------------------------------------
LTVQKV_DEVICE float rq_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
// Two floats rounded to bf16 and packed (lo in the low half), as one 32-bit word.
LTVQKV_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&p);
}
// The rotation of one pair with every product and sum rounded to bf16, as torch's bf16
// elementwise ops round them (x1, x2, c, s hold bf16 values, so -s is exact).
LTVQKV_DEVICE void rope_rotate_bf16(float x1, float x2, float c, float s, float& y1, float& y2) {
  y1 = rq_bf16(__fadd_rn(rq_bf16(__fmul_rn(x1, c)), rq_bf16(__fmul_rn(x2, s))));
  y2 = rq_bf16(__fadd_rn(rq_bf16(__fmul_rn(x1, -s)), rq_bf16(__fmul_rn(x2, c))));
}
// The same rotation for two adjacent elements at once on packed bf16 pairs (x1 = elements j, j + 1
// of the first half, x2 = j + D/2, j + D/2 + 1): the bf16x2 multiply and add round once to bf16,
// and since the product of two bf16 values and the sum of two bf16 values round to bf16 the same
// whether or not they pass through an fp32 rounding first, the results equal rope_rotate_bf16's.
LTVQKV_DEVICE void rope_rotate_bf16x2(uint32_t x1, uint32_t x2, uint32_t c, uint32_t s, uint32_t& y1,
                                      uint32_t& y2) {
  const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&x1);
  const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&x2);
  const __nv_bfloat162 cc = *reinterpret_cast<const __nv_bfloat162*>(&c);
  const __nv_bfloat162 ss = *reinterpret_cast<const __nv_bfloat162*>(&s);
  // the _rn forms: each product and sum rounds on its own (never contracted into a bf16 fma)
  const __nv_bfloat162 r1 = __hadd2_rn(__hmul2_rn(a, cc), __hmul2_rn(b, ss));
  const __nv_bfloat162 r2 = __hadd2_rn(__hmul2_rn(a, __hneg2(ss)), __hmul2_rn(b, cc));
  y1 = *reinterpret_cast<const uint32_t*>(&r1);
  y2 = *reinterpret_cast<const uint32_t*>(&r2);
}
LTVQKV_DEVICE float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
LTVQKV_DEVICE float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
LTVQKV_DEVICE float bf16_lane(uint32_t w, int i) { return i ? bf16_hi(w) : bf16_lo(w); }
// x / D rounded to nearest: for a power-of-two D the product with 1 / D (exact) is the same value
LTVQKV_DEVICE float rope_div_d(float x, int D) {
  return (D & (D - 1)) == 0 ? __fmul_rn(x, __fdiv_rn(1.0f, (float)D)) : __fdiv_rn(x, (float)D);
}
// r from the row's sum of squares
LTVQKV_DEVICE float rope_inv_rms(float ss, int D, float eps) { return rsqrtf(__fadd_rn(rope_div_d(ss, D), eps)); }
// r^3 (sum_j g_j y_j) / D, the norm backward's common term
LTVQKV_DEVICE float rope_k3(float r, float gy, int D) {
  return rope_div_d(__fmul_rn(__fmul_rn(__fmul_rn(r, r), r), gy), D);
}
// Gradient of the pair (x1, x2) from the gradient (g1, g2) of the normalised pair: through the norm,
// dy = r g - y k3, then the transposed rotation dx1 = dy1 c - dy2 s, dx2 = dy1 s + dy2 c.
LTVQKV_DEVICE void rope_norm_bwd(float r, float k3, float g1, float g2, float y1, float y2, float c, float s,
                                 float& dx1, float& dx2) {
  const float dy1 = __fmaf_rn(r, g1, -__fmul_rn(y1, k3));
  const float dy2 = __fmaf_rn(r, g2, -__fmul_rn(y2, k3));
  dx1 = __fmaf_rn(dy1, c, -__fmul_rn(dy2, s));
  dx2 = __fmaf_rn(dy1, s, __fmul_rn(dy2, c));
}

// ------------------------------------------------------------------------------------------
// Release/acquire flag helpers (gpu scope)
// ------------------------------------------------------------------------------------------
LTVQKV_DEVICE void st_release_u32(unsigned int* p, unsigned int v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
LTVQKV_DEVICE unsigned int ld_acquire_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
LTVQKV_DEVICE float ld_cg_f32(const float* p) { return __ldcg(p); }
// Programmatic dependent launch: let the next kernel on the stream be scheduled now; wait until the
// previous kernel on the stream has completed and its memory is visible (returns at once when this
// grid was not launched with programmatic stream serialisation).
LTVQKV_DEVICE void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
LTVQKV_DEVICE void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------------------------------------------
// Shared-memory address helpers
// ------------------------------------------------------------------------------------------
LTVQKV_DEVICE uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// 16-byte global -> shared copy that bypasses registers (cp.async, L2 only); commit of this thread's
// copies issued since the last commit as one group; waits for all / all but the newest N groups.
LTVQKV_DEVICE void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
LTVQKV_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
LTVQKV_DEVICE void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
template <int N>
LTVQKV_DEVICE void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ------------------------------------------------------------------------------------------
// mbarrier
// ------------------------------------------------------------------------------------------
// Which output tensor and local head a global head index maps to (Q heads, K heads, V heads).
LTVQKV_DEVICE void split_head(int h, int NH, int NKVH, int& which, int& hloc, int& nheads) {
  if (h < NH) { which = 0; hloc = h; nheads = NH; }
  else if (h < NH + NKVH) { which = 1; hloc = h - NH; nheads = NKVH; }
  else { which = 2; hloc = h - NH - NKVH; nheads = NKVH; }
}

// `p` advanced to the next multiple of `align` bytes (a power of two) of the shared window, by
// pointer arithmetic: an integer round trip would hide from the compiler that the result points
// into shared memory, turning every access through it into a generic one.
template <typename T>
LTVQKV_DEVICE T* smem_align(void* p, uint32_t align) {
  unsigned char* c = reinterpret_cast<unsigned char*>(p);
  return reinterpret_cast<T*>(c + ((align - (smem_u32(c) & (align - 1))) & (align - 1)));
}
LTVQKV_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
LTVQKV_DEVICE void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
LTVQKV_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
LTVQKV_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
LTVQKV_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait on an mbarrier phase. Returns false (after recording a timeout) when the
// phase did not complete within kWaitLimitNs or another role already gave up (*abort != 0).
LTVQKV_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, WorkspaceHeader* ws,
                             unsigned int where) {
  if (mbar_try_wait(bar, parity)) return true;
  unsigned long long t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      *abort = 1;
      record_timeout(ws, where);
      return false;
    }
  }
}

// ------------------------------------------------------------------------------------------
// TMA (tiled bulk tensor copies; plain CTA-local destinations)
// ------------------------------------------------------------------------------------------
LTVQKV_DEVICE void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(m) : "memory");
}
LTVQKV_DEVICE void tma_load_3d(void* smem_dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(m), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
LTVQKV_DEVICE void tma_load_2d(void* smem_dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(m), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
LTVQKV_DEVICE void tma_load_4d(void* smem_dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(m), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
// Contiguous shared -> global bulk copy (16-byte aligned addresses, size a multiple of 16).
LTVQKV_DEVICE void bulk_store(void* gdst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(smem_src)),
               "r"(bytes)
               : "memory");
}
// Barrier among `count` threads (a multiple of 32) of the CTA, id 1..15 (0 is __syncthreads).
// Plain (untiled) bulk copy global -> this CTA's shared memory, completing on `bar`; both
// addresses 16-byte aligned, size a multiple of 16.
LTVQKV_DEVICE void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
LTVQKV_DEVICE void named_barrier(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
// Named barrier that also ORs a predicate over the participating threads: every thread gets the
// same answer, so a group can leave a loop together when any of its threads saw a wait time out.
LTVQKV_DEVICE bool named_barrier_or(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}
LTVQKV_DEVICE void tma_store_2d(const CUtensorMap* m, const void* smem_src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(m),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}
LTVQKV_DEVICE void tma_store_3d(const CUtensorMap* m, const void* smem_src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(m),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
LTVQKV_DEVICE void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
LTVQKV_DEVICE void tma_store_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
LTVQKV_DEVICE void tma_store_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
LTVQKV_DEVICE void tma_store_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
LTVQKV_DEVICE void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------------------------------------
// tcgen05
// ------------------------------------------------------------------------------------------
LTVQKV_DEVICE void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
LTVQKV_DEVICE void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
LTVQKV_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
LTVQKV_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
LTVQKV_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, bf16 inputs, fp32 accumulation (kind::f16).
LTVQKV_DEVICE void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
LTVQKV_DEVICE void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
LTVQKV_DEVICE void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 columns of 32-bit values: thread i of the warp receives row (lane base + i),
// columns [col, col+32).
LTVQKV_DEVICE void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// ---- CTA pairs (cluster of 2, tcgen05 cta_group::2) ----
LTVQKV_DEVICE uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The same shared-memory variable in cluster CTA `rank`, as a shared::cluster address.
LTVQKV_DEVICE uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
LTVQKV_DEVICE void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
LTVQKV_DEVICE void st_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}
LTVQKV_DEVICE void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Relaxed remote arrive, for barriers that only hand back tensor memory: the arriving warp's TMEM
// reads are complete (tcgen05.wait::ld, then tcgen05.fence::before_thread_sync) and it publishes no
// memory writes through the barrier, so the release ordering of its preceding global stores (which
// waits for them to be acknowledged) is not needed.
LTVQKV_DEVICE void mbar_arrive_cluster_relaxed(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Wait on a local mbarrier whose phase completes through arrivals from the peer CTA (acquire at
// cluster scope, so the peer's writes made before its arrive are visible).
LTVQKV_DEVICE bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
LTVQKV_DEVICE bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort, WorkspaceHeader* ws,
                                     unsigned int where) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      *abort = 1;
      record_timeout(ws, where);
      return false;
    }
  }
}
// 3-D tiled load into this CTA's shared memory whose completion is counted on the pair leader's
// mbarrier (`bar_cluster` is a shared::cluster address). No multicast.
LTVQKV_DEVICE void tma_load_3d_pair(void* smem_dst, const CUtensorMap* m, uint32_t bar_cluster, int c0, int c1,
                                    int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(m), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
LTVQKV_DEVICE void tma_load_4d_pair(void* smem_dst, const CUtensorMap* m, uint32_t bar_cluster, int c0, int c1,
                                    int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(m), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
// Element-wise fp32 add of a shared-memory tile into global memory (tensor-map addressed).
LTVQKV_DEVICE void tma_reduce_add_3d(const CUtensorMap* m, const void* smem_src, int c0, int c1, int c2) {
  asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   m),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
LTVQKV_DEVICE void tmem_alloc_pair(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
LTVQKV_DEVICE void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
LTVQKV_DEVICE void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem of both CTAs] (+)= A[smem of both CTAs] * B[smem of both CTAs]^T, issued by the leader:
// M = 256 rows (128 per CTA), B split by N between the CTAs, bf16 -> fp32.
LTVQKV_DEVICE void umma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the mbarrier at this smem offset in every CTA of `cta_mask` once the pair MMAs issued
// so far complete.
LTVQKV_DEVICE void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// UMMA shared-memory matrix descriptor for a 128-byte-swizzled operand tile
// (sm_100 descriptor: start>>4 in [0,14), LBO>>4 in [16,30), SBO>>4 in [32,46), version 1 at
// bit 46, base offset 0, layout type SWIZZLE_128B (2) in [61,64)).
//   K-major tile:  rows of 128 B (64 bf16 along K), 8-row atoms 1024 B apart  -> SBO = 1024.
//   MN-major tile: rows of 128 B (64 bf16 along M/N) per k, 8-k atoms 1024 B apart -> SBO = 1024,
//                  successive 64-wide M/N blocks LBO bytes apart.
LTVQKV_DEVICE uint64_t umma_desc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 D.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4)                          // D format: f32
         | (1u << 7)                        // A format: bf16
         | (1u << 10)                       // B format: bf16
         | ((uint32_t)(a_mn_major & 1) << 15)
         | ((uint32_t)(b_mn_major & 1) << 16)
         | ((uint32_t)(N >> 3) << 17)
         | ((uint32_t)(M >> 4) << 24);
}

}  // namespace ltvqkv

// ------------------------------------------------------------------------------------------
// Host-side helpers shared by the .cu files
// ------------------------------------------------------------------------------------------
namespace ltvqkv_host {
// Encodes a tiled TMA descriptor (cuTensorMapEncodeTiled through the driver entry point).
// dims[0] is the innermost extent; strides_bytes holds the byte strides of dims 1..rank-1.
bool encode_tiled_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);
int num_sms();
void set_last_cuda_error(cudaError_t e);
int check_launch();  // returns LTVQKV_OK or LTVQKV_ERR_LAUNCH (and records the CUDA error text)
// Device address of ltvqkv_scan_fwd_noalloc's fixed array on the current device (ltvqkv_scan.cu).
int noalloc_scratch(void** out);
inline bool valid_dtype(int dtype) { return dtype == LTVQKV_DTYPE_F32 || dtype == LTVQKV_DTYPE_BF16; }
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
}  // namespace ltvqkv_host
