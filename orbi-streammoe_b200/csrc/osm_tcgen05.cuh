// osm_tcgen05.cuh -- tcgen05 / TMA / mbarrier helpers shared by the
// tensor-core expert kernels (osm_tc.cu: 16-bit operands; osm_tcd.cu: int8
// digit planes).  Every wait is bounded: after two seconds the status bit is
// set and a CTA-wide abort flag releases the other roles.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "osm_common.cuh"

namespace osm {
namespace {

// ---- tcgen05 / TMA helpers ----
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;            // leading offset: unused for swizzled K-major
  d |= (uint64_t)(1024 >> 4) << 32;  // 8-row groups 1024 bytes apart
  d |= (uint64_t)1 << 46;            // descriptor version
  d |= (uint64_t)2 << 61;            // 128-byte swizzle
  return d;
}
// kind::f16 instruction descriptor: fp32 D; A and B both fp16 (bf16 = false)
// or both bf16; K-major; N and M.
__device__ __forceinline__ uint32_t idesc16(int M, int N, bool bf16) {
  const uint32_t ab = bf16 ? ((1u << 7) | (1u << 10)) : 0u;
  return (1u << 4) | ab | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t bd, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a), "l"(bd), "r"(idesc), "r"(acc));
}
// the same with enable-input-d fixed: accumulate (ACC) or overwrite
template <bool ACC>
__device__ __forceinline__ void mma_tsk(uint32_t d, uint32_t a, uint64_t bd, uint32_t idesc) {
  if constexpr (ACC)
    asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, 1;" ::"r"(d), "r"(a), "l"(bd), "r"(idesc));
  else
    asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, 0;" ::"r"(d), "r"(a), "l"(bd), "r"(idesc));
}
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
      "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]),
      "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]),
      "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
      : "memory");
}
template <int N>
__device__ __forceinline__ void tst(uint32_t taddr, const uint32_t (&v)[N]) {
  if constexpr (N == 32) st32(taddr, v);
  else if constexpr (N == 16) st16(taddr, v);
  else st8(taddr, v);
}
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 3-D tiled TMA load (box: 8 words x 128 rows x 1 slot) signalled on bar.
__device__ __forceinline__ void tma3(void* dst, const void* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
// Pair p (0..3) of a Q4 word: (q_2p, q_2p+1) as 16-bit lanes (q in the low
// byte of each) in K order.
__device__ __forceinline__ uint32_t nib_pair(uint32_t lo, uint32_t hi, int p) {
  const uint32_t sel = (uint32_t)p | ((8u | p) << 4) | ((4u + p) << 8) | ((8u | p) << 12);
  return prmt(lo, hi, sel);
}
__device__ __forceinline__ uint32_t bf2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t bf2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t h2u(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __half2 u2h(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }
// fp32 pair -> bf16x2 (round to nearest even), low half = a
__device__ __forceinline__ uint32_t pack_bf2(float a, float b) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(b), "f"(a));
  return d;
}
__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// try_wait with a suspend-time hint: a thread whose phase is not complete is
// suspended until it completes (or the hint, 1 ms, runs out) instead of
// spinning, so waiting roles leave the issue slots to the working ones.
__device__ __forceinline__ bool mbar_try_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait on an mbarrier phase shared by every role of the CTA: after
// two seconds the status bit is set and the CTA-wide abort flag makes all
// later waits return at once, so no role waits on one that has stopped.
constexpr uint64_t kTcWaitNs = 2000000000ull;
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                        uint32_t* status) {
  if (mbar_try_sleep(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    if (mbar_try_sleep(bar, parity)) return true;
    if (*abort) return false;
    if (global_ns() - t0 > kTcWaitNs) break;
  }
  *abort = 1;
  atomicOr(status, kStatusCopyTimeout);
  return false;
}

// tc_wait by every lane of a warp, with one outcome for the whole warp (a
// lane that gave up stops the others too, so no lane is left at a
// warp-collective instruction).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          uint32_t* status) {
  const bool w = tc_wait(bar, parity, abort, status);
  return __all_sync(0xFFFFFFFFu, w);
}


}  // namespace
}  // namespace osm
