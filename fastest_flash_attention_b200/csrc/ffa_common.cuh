// Shared device helpers for the sm_100a attention kernels: mbarriers with
// bounded waits, TMA tile loads, tcgen05 (TMEM allocation, MMA issue, commit,
// TMEM <-> register moves) and the shared-memory / instruction descriptors the
// tensor cores consume.  Everything here is hand-written inline PTX; no
// CUTLASS/CuTe code is included.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "ffa_b200.h"

namespace ffa {

// ---------------------------------------------------------------------------
// Error reporting shared by all kernels.  `err` points at a device word; the
// first failing wait records its site code there and the host turns it into
// an FFA_ERR_DEVICE_TIMEOUT status.  No kernel ever traps.
// ---------------------------------------------------------------------------
struct ErrCtx {
  uint32_t* err;              // device error word (may be nullptr)
  unsigned long long limit_ns;  // wall-clock limit for one wait
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t lane_id() {
  uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ------------------------------- mbarrier ----------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
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

// Non-blocking probe (test_wait never suspends the thread, unlike try_wait):
// for issuers that poll several barriers and take whichever is ready.
__device__ __forceinline__ bool mbar_poll(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  The wait is bounded
// by wall-clock time: on expiry the site code is recorded in the error word,
// `*abort` is raised so every other role of the CTA stops waiting too, and
// false is returned.  A raised `*abort` makes every later wait return false
// immediately, unless `drain` is set: draining waits (for copies or MMAs still
// in flight before the CTA releases its memory) ignore the abort flag and are
// bounded by at least kDrainFloorNs whatever the caller's limit, so a short
// user limit can never let a CTA free shared memory or TMEM under a copy or
// an MMA that is still running.
constexpr unsigned long long kDrainFloorNs = 4000000000ull;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const ErrCtx& ec,
                                          volatile int* abort, uint32_t site, bool drain = false) {
  if (mbar_test(bar, parity)) return true;
  if (!drain && *abort) return false;
  // The limit is counted in SM clock cycles (cheap to read); 2 cycles per ns
  // over-approximates every B200 clock, so the wall-clock bound still holds.
  const long long t0 = clock64();
  const unsigned long long lim_ns =
      (drain && ec.limit_ns < kDrainFloorNs) ? kDrainFloorNs : ec.limit_ns;
  const long long limit = (long long)(lim_ns * 2ull);
  uint32_t spins = 0;
  while (true) {
    if (mbar_test(bar, parity)) return true;
    if (((++spins) & 15u) == 0) {
      if (!drain && *abort) return false;
      if (clock64() - t0 > limit) {
        *abort = 1;
        if (ec.err) atomicCAS(ec.err, 0u, site);
        return false;
      }
    }
  }
}

// The MMA issuer's wait: a non-blocking probe first (cheap when the phase is
// already complete, the common case), then the bounded blocking wait.
__device__ __forceinline__ bool mbar_wait_mma(uint64_t* bar, uint32_t parity, const ErrCtx& ec, volatile int* abort,
                                              uint32_t site, bool drain = false) {
  if (mbar_poll(bar, parity)) return true;
  return mbar_wait(bar, parity, ec, abort, site, drain);
}

// ---------------------------------- TMA ------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(m) : "memory");
}

// 4-D tiled load (no multicast) completing on an mbarrier transaction count.
__device__ __forceinline__ void tma_load_4d(const CUtensorMap* m, uint64_t* bar, void* dst, int c0, int c1,
                                            int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
      "l"(m), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// 4-D tiled store smem -> global (bulk async group; out-of-bounds rows of the
// box are not written).  Wait with tma_store_wait_read before reusing `src`.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* m, const void* src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(m),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(src))
               : "memory");
}
__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ------------------------------- tcgen05 -----------------------------------
// Warp-collective TMEM allocation; the base address is written to smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
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

// D[tmem] (+)= A[smem] * B[smem]^T   (kind::f16, fp32 accumulate)
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every previously issued tcgen05 op of this thread retires.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Instruction descriptor for kind::f16 with fp32 accumulation.
//   ab_fmt: 0 = f16, 1 = bf16;  a_mn / b_mn: operand is MN-major (1) or K-major (0)
__host__ __device__ constexpr uint32_t make_idesc_f16(uint32_t M, uint32_t N, uint32_t ab_fmt, uint32_t a_mn,
                                                      uint32_t b_mn) {
  return (1u << 4) | (ab_fmt << 7) | (ab_fmt << 10) | (a_mn << 15) | (b_mn << 16) | ((N >> 3) << 17) |
         ((M >> 4) << 24);
}

// Shared-memory matrix descriptor, 128-byte swizzle, sm100 version field.
//   K-major tiles : rows of 128 B, 8-row groups `sbo` bytes apart (lbo unused -> 16 B)
//   MN-major tiles: 64-element MN chunks `lbo` bytes apart, 8-row K groups `sbo` apart
__device__ __forceinline__ uint64_t make_sdesc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;   // descriptor version for sm100
  d |= 2ull << 61;   // SWIZZLE_128B
  return d;
}

// TMEM -> registers: 32 lanes x 32 consecutive 32-bit columns (one column per
// register, lane = thread of the warp).  Values are undefined until
// tmem_ld_wait() has been executed; callers pass the registers through it.
#define FFA_R8(a, o) "=r"(a[o + 0]), "=r"(a[o + 1]), "=r"(a[o + 2]), "=r"(a[o + 3]), "=r"(a[o + 4]), \
                     "=r"(a[o + 5]), "=r"(a[o + 6]), "=r"(a[o + 7])
#define FFA_W8(a, o) "+r"(a[o + 0]), "+r"(a[o + 1]), "+r"(a[o + 2]), "+r"(a[o + 3]), "+r"(a[o + 4]), \
                     "+r"(a[o + 5]), "+r"(a[o + 6]), "+r"(a[o + 7])
#define FFA_I8(a, o) "r"(a[o + 0]), "r"(a[o + 1]), "r"(a[o + 2]), "r"(a[o + 3]), "r"(a[o + 4]), \
                     "r"(a[o + 5]), "r"(a[o + 6]), "r"(a[o + 7])

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : FFA_R8(r, 0), FFA_R8(r, 8), FFA_R8(r, 16), FFA_R8(r, 24)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : FFA_R8(r, 0), FFA_R8(r, 8)
      : "r"(taddr));
}
// Completes outstanding tcgen05.ld of this thread; the registers are threaded
// through so the compiler cannot hoist their uses above the wait.
__device__ __forceinline__ void tmem_ld_wait32(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : FFA_W8(r, 0), FFA_W8(r, 8), FFA_W8(r, 16), FFA_W8(r, 24)::"memory");
}
__device__ __forceinline__ void tmem_ld_wait16(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : FFA_W8(r, 0), FFA_W8(r, 8)::"memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      FFA_I8(r, 0), FFA_I8(r, 8), FFA_I8(r, 16), FFA_I8(r, 24)
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      FFA_I8(r, 0), FFA_I8(r, 8)
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), FFA_I8(r, 0)
               : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Generic-proxy smem writes -> visible to the async proxy (tensor core / TMA).
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Re-balance the register file between warpgroups (all warps of a
// warpgroup execute the same call).  The per-warpgroup budgets of a kernel
// must add up to at most its launch allocation.
template <uint32_t N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// ------------------------------ math ---------------------------------------
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// tanh(x) = 1 - 2 / (2^(2x*log2 e) + 1); accurate to a few ulp of 1 in fp32,
// which matters because softcap multiplies it back up by the cap.
__device__ __forceinline__ float tanh_acc(float x) {
  const float e = ex2(x * 2.8853900817779268f);  // 2*log2(e)
  return 1.0f - 2.0f * rcp(e + 1.0f);
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Packed fp32x2 arithmetic (one FMA-pipe instruction for two lanes of work).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

// Softcap for small arguments.  With k = scale / softcap and |k s| <= 1/2,
//   tanh(k s) = k y,   y = s (1 + r),   r = v (A + v (B + C v)),   v = s^2,
// where (A, B, C) = (a k^2, b k^4, c k^6) and x (1 + a x^2 + b x^4 + c x^6)
// is an odd degree-7 polynomial fitted to tanh on [-1/2, 1/2] (least squares
// on Chebyshev nodes, reweighted towards minimax: max abs error 2.0e-7, 2.2e-7
// evaluated in fp32).  softcap * log2(e) * tanh(k s) = scale * log2(e) * y, so
// callers use y with the plain score multiplier.  Two lanes per packed
// instruction: five FMA-pipe instructions per pair of scores.
constexpr double SOFTCAP_POLY_A = -0.3332648070862027;
constexpr double SOFTCAP_POLY_B = 0.13186077719149775;
constexpr double SOFTCAP_POLY_C = -0.04423483979939102;

// (A, B, C) for k = scale / softcap (host side, in double, then rounded).
inline void softcap_poly_coeffs(float k, float* abc) {
  const double k2 = (double)k * (double)k;
  abc[0] = (float)(SOFTCAP_POLY_A * k2);
  abc[1] = (float)(SOFTCAP_POLY_B * k2 * k2);
  abc[2] = (float)(SOFTCAP_POLY_C * k2 * k2 * k2);
}

__device__ __forceinline__ float2 softcap_small2(float2 s, float a, float b, float c) {
  const float2 v = fmul2(s, s);
  float2 t = ffma2(f2(c), v, f2(b));
  t = ffma2(t, v, f2(a));
  return ffma2(s, fmul2(t, v), s);
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

template <typename T>
struct DtypeFmt;
template <>
struct DtypeFmt<__nv_bfloat16> {
  static constexpr uint32_t value = 1;
};
template <>
struct DtypeFmt<__half> {
  static constexpr uint32_t value = 0;
};

}  // namespace ffa
