// Thin inline-PTX wrappers for the sm_100a features the tensor-core kernels use:
// mbarriers (with bounded waits), TMA tensor loads, tcgen05 TMEM allocation,
// MMA, commit, TMEM loads/stores and the shared-memory matrix descriptors.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace p3d {
namespace sm100 {

// Device-side failure bits, kept by each kernel file in its own __device__ word and
// read back (and cleared) through p3d_device_errors().  Bit 0 says that a bounded wait
// gave up; bits 1-4 say which role's wait it was.
enum : unsigned {
  kErrTimeout = 1u,
  kErrProducer = 2u,   // TMA producer
  kErrMma = 4u,        // MMA issuer
  kErrSoftmax = 8u,    // softmax / epilogue warps
  kErrTeardown = 16u   // a drain before TMEM is freed
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that may suspend the thread for up to `hint_ns` (it resumes as soon as the phase
// completes): a waiting warp then takes no issue slots from the warps that do the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Non-blocking test of a phase: cheaper than try_wait when the phase has already completed.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of an mbarrier, giving up after timeout_ns: then the
// timeout bit is set in *errors and false is returned, so the caller can unwind
// instead of spinning forever.
//
// Elapsed time is the sum of the forward steps of %globaltimer between consecutive
// polls, each step capped at 1 ms, so that a re-synchronised (stepped) timer can
// neither end a wait early nor extend it; the SM cycle counter, summed the same way,
// bounds the wait as well (at 4 cycles per nanosecond of the limit) in case the
// nanosecond timer stalls.  `role` is or-ed into *errors with kErrTimeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned *errors,
                                          uint64_t timeout_ns = 2000000000ull, unsigned role = 0u) {
  if (mbar_test_wait(bar, parity)) return true;
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t_last = global_timer_ns(), waited_ns = 0;
  long long c_last = clock64(), waited_cycles = 0;
  while (!mbar_try_wait_sleep(bar, parity, 20000u)) {
    const uint64_t t = global_timer_ns();
    const long long c = clock64();
    const long long dt = (long long)(t - t_last), dc = c - c_last;
    t_last = t;
    c_last = c;
    if (dt > 0) waited_ns += dt < 1000000 ? (uint64_t)dt : 1000000ull;
    if (dc > 0) waited_cycles += dc < 4000000 ? dc : 4000000;
    if (waited_ns > timeout_ns || (unsigned long long)waited_cycles > 4ull * timeout_ns) {
      atomicOr(errors, kErrTimeout | role);
      return false;
    }
  }
  return true;
}

// ------------------------------------------------------------------ TMA
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0, int c1,
                                            int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, "
      "%7}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

// Plain (non-tensor) bulk copy global -> shared, completing `bytes` on the mbarrier.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
               : "memory");
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t holder_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(holder_smem), "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
// Generic-proxy shared-memory stores made visible to later async-proxy readers (TMA,
// tcgen05.mma) after the next thread synchronisation.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T  (kind::f16: bf16 or f16 inputs, fp32 accumulate)
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once every tcgen05 operation issued so far by this thread completes.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// Warp-wide forms: every lane of a converged warp executes the call with the same (warp-
// uniform) operands, and one lane elected by elect.sync -- the same lane every time the whole
// warp takes part -- issues the instruction.  Keeping the operands warp-uniform lets them
// live in uniform registers instead of being moved there before every instruction.
__device__ __forceinline__ void mma_ss_warp(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred e, p;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_ts_warp(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred e, p;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Commit by the elected lane: it tracks the operations that lane issued (mma_*_warp).
__device__ __forceinline__ void mma_commit_warp(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 16 consecutive 32-bit columns: thread i of the warp gets lane (warp quarter)+i.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t *r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t *r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t *r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t *r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// Shared-memory matrix descriptor (sm_100 "version 1"), SWIZZLE_32B layout.
//   K-major : 8-row groups of 32-byte rows at stride sbo; lbo unused (16 bytes).
//   MN-major: 16-element (32-byte) atoms along M/N at stride lbo, 8-row K groups at stride sbo.
__device__ __forceinline__ uint64_t desc_sw32(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)6 << 61;  // layout type SWIZZLE_32B
  return d;
}

// Shared-memory matrix descriptor, SWIZZLE_128B K-major layout: 8-row groups of 128-byte rows
// (1024-byte atoms, 1024-byte aligned) at stride sbo.  A K = 16 slice of a 16-bit operand is
// 32 bytes of each row: successive slices advance the start address by 32 bytes.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t smem_addr, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;  // leading-dimension offset: unused for swizzled K-major
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)2 << 61;  // layout type SWIZZLE_128B
  return d;
}

// Instruction descriptor of kind::f16 with fp32 accumulation.
//   ab_bf16: operands are bf16 (else f16); b_mn_major: B is MN-major (else K-major).
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n, bool ab_bf16, bool b_mn_major) {
  return (1u << 4)                              // D format: f32
         | ((ab_bf16 ? 1u : 0u) << 7)           // A format
         | ((ab_bf16 ? 1u : 0u) << 10)          // B format
         | ((b_mn_major ? 1u : 0u) << 16)       // B major
         | ((uint32_t)(n >> 3) << 17)           // N / 8
         | ((uint32_t)(m >> 4) << 24);          // M / 16
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Paired f32 arithmetic (sm_100 f32x2 instructions: one issue slot for two lanes of work).
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// 2^x for a pair, on the FMA pipe instead of the MUFU: Cody-Waite reduction x = j + f with
// j = rint(x) (the 1.5 * 2^23 rounding trick) and f in [-0.5, 0.5], a degree-3 polynomial
// for 2^f (coefficients fitted here for minimax relative error on [-0.5, 0.5]: max
// relative error 7.5e-5, below the 2^-9 of the bf16 P it feeds), and j added into the
// exponent field.  Inputs below -126 are clamped (-inf -> ~2^-126, not 0); x <= 127.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kMagic = 12582912.f;  // 1.5 * 2^23
  x.x = fmaxf(x.x, -126.f);
  x.y = fmaxf(x.y, -126.f);
  const float2 jj = add2(x, make_float2(kMagic, kMagic));          // rint(x) in the low bits
  const float2 r = add2(jj, make_float2(-kMagic, -kMagic));        // rint(x)
  const float2 f = fma2(r, make_float2(-1.f, -1.f), x);            // x - rint(x)
  float2 p = fma2(make_float2(0.0551716685f, 0.0551716685f), f, make_float2(0.24261114f, 0.24261114f));
  p = fma2(p, f, make_float2(0.69326097f, 0.69326097f));
  p = fma2(p, f, make_float2(0.99992806f, 0.99992806f));
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(jj.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(jj.y) << 23)));
}

// exp2_poly2 without the lower clamp, for arguments known to lie in [-125, 127] (the
// fixed-reference softmax of the stencil forward keeps them in [-64, 0]).
__device__ __forceinline__ float2 exp2_poly2_inrange(float2 x) {
  constexpr float kMagic = 12582912.f;  // 1.5 * 2^23
  const float2 jj = add2(x, make_float2(kMagic, kMagic));
  const float2 r = add2(jj, make_float2(-kMagic, -kMagic));
  const float2 f = fma2(r, make_float2(-1.f, -1.f), x);
  float2 p = fma2(make_float2(0.0551716685f, 0.0551716685f), f, make_float2(0.24261114f, 0.24261114f));
  p = fma2(p, f, make_float2(0.69326097f, 0.69326097f));
  p = fma2(p, f, make_float2(0.99992806f, 0.99992806f));
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(jj.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(jj.y) << 23)));
}

// Maximum of three (sm_100 three-input max; NaN handling as fmaxf).
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

}  // namespace sm100
}  // namespace p3d
