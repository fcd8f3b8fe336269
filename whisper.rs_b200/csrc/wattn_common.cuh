// wattn_common.cuh -- shared device helpers for the sm_100a attention path:
// element types, bounded mbarrier waits, TMA loads, tcgen05 (TMEM + UMMA)
// wrappers, and the per-device status word.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/wattn.h"

#define WATTN_DEVINL __device__ __forceinline__

namespace wattn {

// Head dimension served by every kernel (all Whisper models use 64).
constexpr int kHeadDim = 64;

// ------------------------------------------------------------ status word
// Every kernel gets a pointer to its device's status word (a __device__ int
// of the library). A bounded wait that runs out stores WATTN_ERR_TIMEOUT
// there and the kernel winds down instead of hanging; wattn_device_status()
// reads and clears it.

// Limits of one bounded wait: wall clock (%globaltimer) and, independently,
// the number of try_wait rounds (each suspends for at most kSuspendHintNs).
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s
constexpr uint32_t kSuspendHintNs = 1000;
constexpr uint32_t kMaxWaitRounds = 4000000;  // >= 4 s of 1 us suspends

WATTN_DEVINL unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// status[0]: status word; status[1]: site of the first wait that ran out
// (kernel << 24 | role << 16 | barrier << 8 | iteration & 0xff).
WATTN_DEVINL void report_error(int *status, int code, int site) {
  if (atomicCAS(status, WATTN_OK, code) == WATTN_OK) atomicExch(status + 1, site);
}
WATTN_DEVINL void report_timeout(int *status, int site) {
  report_error(status, WATTN_ERR_TIMEOUT, site);
}

// ------------------------------------------------------------ element types
template <int DT> struct Elem;
template <> struct Elem<WATTN_F32> { using T = float; };
template <> struct Elem<WATTN_F16> { using T = __half; };
template <> struct Elem<WATTN_BF16> { using T = __nv_bfloat16; };

WATTN_DEVINL float to_f32(float x) { return x; }
WATTN_DEVINL float to_f32(__half x) { return __half2float(x); }
WATTN_DEVINL float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> WATTN_DEVINL T from_f32(float x);
template <> WATTN_DEVINL float from_f32<float>(float x) { return x; }
template <> WATTN_DEVINL __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> WATTN_DEVINL __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Packs (lo, hi) into one 32-bit word of two 16-bit values, round to nearest.
template <typename T> WATTN_DEVINL uint32_t pack2(float lo, float hi);
template <> WATTN_DEVINL uint32_t pack2<__half>(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
template <> WATTN_DEVINL uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Unpacks two 16-bit values of one 32-bit word to f32.
template <typename T> WATTN_DEVINL float2 unpack2(uint32_t w);
template <> WATTN_DEVINL float2 unpack2<__half>(uint32_t w) {
  __half2 h = *reinterpret_cast<__half2 *>(&w);
  return __half22float2(h);
}
template <> WATTN_DEVINL float2 unpack2<__nv_bfloat16>(uint32_t w) {
  // bf16 -> f32 is a 16-bit shift.
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// 2^x on the SFU (PTX ex2.approx, flush-to-zero).
WATTN_DEVINL float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction (sm_100 three-input max).
WATTN_DEVINL float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for a pair on the FMA pipe, for x <= 8 (x below -126 gives ~0).
// Range reduction x = j + f with j = rint(x) (the 1.5 * 2^23 rounding trick)
// and f in [-1/2, 1/2]; 2^f from a cubic fitted for minimum relative error on
// that interval (a discretised Chebyshev fit solved as a linear programme,
// exp2_poly.py: max relative error 7.5e-5 after f32 evaluation, below the
// bf16 / f16 rounding of P); 2^j is applied by adding j to the exponent.
WATTN_DEVINL float2 exp2_fma2(float2 x) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  x.x = fmaxf(x.x, -126.0f);
  x.y = fmaxf(x.y, -126.0f);
  const float2 t = __fadd2_rn(x, make_float2(kMagic, kMagic));
  const float2 j = __fadd2_rn(t, make_float2(-kMagic, -kMagic));
  const float2 f = __ffma2_rn(j, make_float2(-1.0f, -1.0f), x);
  float2 p = __ffma2_rn(make_float2(5.517221987e-02f, 5.517221987e-02f), f,
                        make_float2(2.426111549e-01f, 2.426111549e-01f));
  p = __ffma2_rn(p, f, make_float2(6.932608485e-01f, 6.932608485e-01f));
  p = __ffma2_rn(p, f, make_float2(9.999280572e-01f, 9.999280572e-01f));
  // The low mantissa bits of t hold j + 2^22; shifting by 23 drops the rest.
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

// ------------------------------------------------------------ dependent launch
// Programmatic dependent launch. grid_dep_wait: waits until the grids this
// launch depends on have completed and their memory is visible (a no-op when
// the launch did not ask for programmatic serialisation). grid_dep_launch:
// lets the next such launch in the stream start its CTAs (they then run up
// to their own grid_dep_wait) once every CTA of this grid has called it.
WATTN_DEVINL void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
WATTN_DEVINL void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------ shared memory
WATTN_DEVINL uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------ mbarrier
WATTN_DEVINL void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Makes barrier initialisation visible to the async proxy (TMA, tcgen05).
WATTN_DEVINL void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

WATTN_DEVINL void mbar_arrive(uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

WATTN_DEVINL void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

WATTN_DEVINL bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Non-blocking probe: whether the phase of `bar` with the given parity has
// completed (mbarrier.test_wait never suspends the thread).
WATTN_DEVINL bool mbar_test_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

#ifndef WATTN_WAIT_PROBE
#define WATTN_WAIT_PROBE 1
#endif

// Waits for the phase of `bar` with the given parity to complete. Bounded:
// if `*abort` is set (another role already gave up) it returns false at
// once; if the wait itself runs past kWaitLimitNs it reports a timeout,
// sets *abort and returns false. Callers then wind down instead of hanging.
WATTN_DEVINL bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort,
                            int *status, int site) {
  uint32_t addr = smem_u32(bar);
  if (WATTN_WAIT_PROBE && mbar_test_wait(addr, parity)) return true;
  if (mbar_try_wait(addr, parity)) return true;
  unsigned long long t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(addr, parity)) return true;
    if ((it & 15) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs || it > kMaxWaitRounds) {
        report_timeout(status, site);
        *abort = 1;
        return false;
      }
    }
  }
}

// ------------------------------------------------------------ TMA
WATTN_DEVINL void tma_prefetch_desc(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

WATTN_DEVINL void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0,
                              int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

WATTN_DEVINL void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0,
                              int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

WATTN_DEVINL void tma_load_4d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0,
                              int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory tile -> global through a tensor map (elements outside the
// map's extent are not written); completes as a bulk async-group.
WATTN_DEVINL void tma_store_4d(const CUtensorMap *map, const void *src, int c0, int c1, int c2,
                               int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
WATTN_DEVINL void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until every committed bulk store of this thread has read its source.
WATTN_DEVINL void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) accesses.
WATTN_DEVINL void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------ tcgen05
// TMEM addresses: bits 31..16 lane, bits 15..0 column.
WATTN_DEVINL void tmem_alloc(uint32_t *smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
WATTN_DEVINL void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
WATTN_DEVINL void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
WATTN_DEVINL void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
WATTN_DEVINL void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (f16 or bf16 operands, f32 accum).
WATTN_DEVINL void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem], kind::f16.
WATTN_DEVINL void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05 operation issued so far by this
// thread has completed.
WATTN_DEVINL void umma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

WATTN_DEVINL void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
WATTN_DEVINL void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 consecutive 32-bit columns of this thread's TMEM lane.
WATTN_DEVINL void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

// 16 consecutive 32-bit columns of this thread's TMEM lane.
WATTN_DEVINL void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

// tcgen05.ld results are only valid after tcgen05.wait::ld, but the compiler
// sees both as opaque asm and may move uses of the result registers above
// the wait. Passing the registers through this empty volatile asm (ordered
// after the wait like every volatile asm) pins all uses below it.
WATTN_DEVINL void reg_fence(uint32_t (&r)[32]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                 "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31]));
}

WATTN_DEVINL void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// ------------------------------------------------------------ UMMA descriptors
// Shared-memory matrix descriptor (sm_100 format): start address, leading
// and stride byte offsets (all >> 4), version 1 at bits 46-47, swizzle mode
// at bits 61-63 (2 = 128-byte swizzle).
WATTN_DEVINL uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3fff);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3fff) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3fff) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor of kind::f16 with f32 accumulation.
// ab_type: 0 = f16, 1 = bf16. a_mn / b_mn: operand is MN-major (1) or K-major (0).
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t ab_type, uint32_t m, uint32_t n,
                                                 uint32_t a_mn, uint32_t b_mn) {
  return (1u << 4)               // D format f32
         | (ab_type << 7)        // A format
         | (ab_type << 10)       // B format
         | (a_mn << 15)          // A major
         | (b_mn << 16)          // B major
         | ((n >> 3) << 17)      // N >> 3
         | ((m >> 4) << 24);     // M >> 4
}

}  // namespace wattn
