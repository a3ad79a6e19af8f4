// Thin inline-PTX wrappers for sm_100a: mbarriers, TMA tile loads, cp.async,
// and the tcgen05 family (TMEM alloc, UMMA issue/commit, TMEM load/store).
//
// Descriptor bit layouts follow the PTX ISA "Matrix Descriptors" and
// "Instruction descriptor" sections for tcgen05 (kind::f16).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <cmath>

namespace dta {

// ---------------------------------------------------------------------------
// status codes written by kernels into the caller's error word
// ---------------------------------------------------------------------------
enum : int {
  KERR_NONE = 0,
  KERR_TIMEOUT_PRODUCER = 101,
  KERR_TIMEOUT_MMA = 102,
  KERR_TIMEOUT_SOFTMAX = 103,
  KERR_TIMEOUT_DRAIN = 104,
  KERR_BAD_ROW = 105,  // a query row or key limit outside the tensors (clamped, output not trusted)
};

// Default wait budget, ~2 s at 1.9 GHz: longer than any legitimate wait in
// these kernels (one key tile of one job is microseconds), short enough that a
// broken pipeline returns control to the host instead of hanging the GPU.  The
// caller may pass a different budget; waits that drain in-flight copies or
// tensor-core ops on the way out always use this one.
constexpr long long kWaitTimeoutCycles = 4000000000LL;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Where a bounded wait records that it gave up: the CTA's abort flag (shared
// memory, seen by every role), the kernel error word (global memory, read by
// the host) and the wait budget in clock64 cycles.
struct WaitCtx {
  volatile int* abort_flag;
  int* err;
  long long limit;
};

static __device__ __forceinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, const WaitCtx& w, int code) {
  long long t0 = clock64();
  uint32_t it = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++it & 255u) == 0u) {
      if (*w.abort_flag) return false;
      if (clock64() - t0 > w.limit) {
        *w.abort_flag = 1;
        atomicCAS(w.err, 0, code);
        return false;
      }
    }
  }
}

// Bounded wait for the phase with parity `parity` to complete.  Returns false
// (after raising the CTA abort flag and recording `code` in the error word)
// when the wait exceeds the budget, or when another role already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const WaitCtx& w, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, w, code);
}

// Polling variant for latency-critical single-thread waiters (the MMA issuer):
// mbarrier.test_wait never suspends, so the phase completion is seen within a
// few cycles instead of after try_wait's suspend interval.  Same bound and
// abort protocol as mbar_wait.
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
static __device__ __forceinline__ bool mbar_poll_slow(uint32_t bar, uint32_t parity, const WaitCtx& w, int code) {
  const long long t0 = clock64();
  uint32_t it = 0;
  while (true) {
    if (mbar_test(bar, parity)) return true;
    if ((++it & 1023u) == 0u) {
      if (*w.abort_flag) return false;
      if (clock64() - t0 > w.limit) {
        *w.abort_flag = 1;
        atomicCAS(w.err, 0, code);
        return false;
      }
    }
  }
}
__device__ __forceinline__ bool mbar_poll(uint32_t bar, uint32_t parity, const WaitCtx& w, int code) {
  if (mbar_test(bar, parity)) return true;
  return mbar_poll_slow(bar, parity, w, code);
}

// Bounded wait until a shared-memory counter reaches `target` (same abort
// protocol as mbar_wait).
__device__ __forceinline__ bool smem_wait_geq(volatile int* c, int target, const WaitCtx& w, int code) {
  if (*c >= target) return true;
  const long long t0 = clock64();
  while (*c < target) {
    if (*w.abort_flag) return false;
    if (clock64() - t0 > w.limit) {
      *w.abort_flag = 1;
      atomicCAS(w.err, 0, code);
      return false;
    }
    __nanosleep(20);
  }
  return true;
}

// Programmatic dependent launch: the dependent grid's wait for the grid it
// depends on (complete, writes visible), and the primary's early trigger.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dependents_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Thread-block clusters: the hardware cluster barrier (every thread of every
// CTA arrives; release/acquire orders shared-memory writes before it with
// distributed-shared-memory reads after it), the CTA's rank and the cluster's
// size, and loads from a peer CTA's shared memory.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
// the shared::cluster address of `addr` (a shared::cta address) in CTA `rank`
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Warp-collective variant: every lane waits, then the warp reconverges so the
// caller may issue .sync.aligned tcgen05 instructions.  The result is the
// AND over the warp (an abort seen by any lane aborts the whole warp).
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, const WaitCtx& w, int code) {
  const bool ok = mbar_wait(bar, parity, w, code);
  return __all_sync(0xffffffffu, ok);
}

// ---------------------------------------------------------------------------
// TMA (tiled, no multicast) and cp.async
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* tmap, uint32_t bar, int x, int y,
                                            int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar)
      : "memory");
}
// One lane of the (converged) warp returns true (elect.sync).  Code that issues
// tcgen05.mma this way runs warp-uniform, so descriptors and counters live in
// uniform registers instead of being moved there before every instruction.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// Tiled TMA store (shared -> global) into the bulk async-group of this thread.
__device__ __forceinline__ void tma_store_4d(const void* tmap, uint32_t src, int x, int y, int z, int w) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(tmap),
               "r"(x), "r"(y), "r"(z), "r"(w), "r"(src)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// this thread's bulk stores have finished reading shared memory
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// this thread's bulk stores are complete
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: UMMA descriptors
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor (64 bit):
//   [0,14)  start address >> 4
//   [16,30) leading-dimension byte offset >> 4
//   [32,46) stride-dimension byte offset >> 4
//   [46,48) descriptor version (1 on sm_100)
//   [49,52) base offset (0: atoms are 1024-byte aligned)
//   [52]    LBO mode (0)
//   [61,64) layout: 2 = 128-byte swizzle
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Instruction descriptor (32 bit) for kind::f16 with bf16 inputs, fp32 accumulate:
//   [4,6) D format (1 = f32); [7,10) A format (1 = bf16); [10,13) B format (1 = bf16);
//   [15] A major (0 = K); [16] B major (0 = K, 1 = MN); [17,23) N >> 3; [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, int b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)b_mn_major << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem], issued by one thread.
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when all tcgen05 ops previously issued by this thread complete.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM <-> registers (32 lanes x 32-bit, one lane per thread)
// ---------------------------------------------------------------------------
#define DTA_R8(i) "=r"(r[i + 0]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), "=r"(r[i + 5]), \
                  "=r"(r[i + 6]), "=r"(r[i + 7])
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : DTA_R8(0), DTA_R8(8), DTA_R8(16), DTA_R8(24)
      : "r"(taddr));
}
#undef DTA_R8
#define DTA_F8(i) "=f"(r[i + 0]), "=f"(r[i + 1]), "=f"(r[i + 2]), "=f"(r[i + 3]), "=f"(r[i + 4]), "=f"(r[i + 5]), \
                  "=f"(r[i + 6]), "=f"(r[i + 7])
// Same load with the 32 columns landing directly in float registers r[0..31].
__device__ __forceinline__ void tmem_ld32f(uint32_t taddr, float* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : DTA_F8(0), DTA_F8(8), DTA_F8(16), DTA_F8(24)
      : "r"(taddr));
}
#undef DTA_F8
#define DTA_W8(i) "r"(r[i + 0]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), "r"(r[i + 5]), \
                  "r"(r[i + 6]), "r"(r[i + 7])
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      DTA_W8(0), DTA_W8(8), DTA_W8(16), DTA_W8(24)
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      DTA_W8(0), DTA_W8(8)
      : "memory");
}
#undef DTA_W8
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------
// per-warpgroup register reallocation (all 4 warps of a warpgroup execute it)
// ---------------------------------------------------------------------------
template <int N>
__device__ __forceinline__ void regs_release() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_acquire() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// ---------------------------------------------------------------------------
// math helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// three-input maximum (one instruction on sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
// packed fp32 pairs (one instruction operates on both halves)
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// 2^x evaluated on the FMA pipe instead of the MUFU unit.  Range reduction
// x = n + f with n = rint(x) (the 1.5 * 2^23 shifter leaves rint(x) in the low
// mantissa bits of t) and |f| <= 1/2; 2^f from a degree-3 polynomial whose
// coefficients minimise the maximum relative error on [-1/2, 1/2] (computed
// for this kernel with the Remez exchange algorithm: 7.5e-5 in exact arithmetic,
// 1.5e-4 in fp32 over [-126, 8], against bf16 rounding of P at 2e-3); 2^n is
// applied by adding n to the exponent field.  Inputs below -126 are clamped
// (the result is then a negligible tiny number, never NaN).
__device__ __forceinline__ float exp2_poly(float x) {
  x = fmaxf(x, -126.0f);
  const float t = __fadd_rn(x, 12582912.0f);
  const float n = __fsub_rn(t, 12582912.0f);
  const float f = __fsub_rn(x, n);
  float p = __fmaf_rn(0.05517166905792616f, f, 0.2426111221932161f);
  p = __fmaf_rn(p, f, 0.6932609854606553f);
  p = __fmaf_rn(p, f, 0.9999280735394012f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// 32-byte global store (one sector per lane)
__device__ __forceinline__ void st_global_v8(void* ptr, const uint32_t (&v)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(ptr), "r"(v[0]), "r"(v[1]), "r"(v[2]),
               "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

}  // namespace dta
