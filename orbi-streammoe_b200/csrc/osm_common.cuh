// osm_common.cuh -- device helpers shared by the sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace osm {

constexpr int kWarp = 32;
constexpr int kGroup = 64;          // quantisation group along the input dim
constexpr int kMaxExperts = 1024;   // router width supported by the selectors
constexpr int kMaxTopK = 32;

// Device status bits (osm_context_status).
constexpr uint32_t kStatusNonFinite = 1u << 0;
constexpr uint32_t kStatusBadMass = 1u << 1;
constexpr uint32_t kStatusNotResident = 1u << 2;
constexpr uint32_t kStatusBadSlot = 1u << 3;
constexpr uint32_t kStatusCopyTimeout = 1u << 4;  // a bounded wait on an async copy gave up
constexpr uint32_t kStatusF16Range = 1u << 5;     // prefill: a value left the fp16 range
constexpr uint32_t kStatusPrefillFallback = 1u << 6;  // host: a checked prefill call re-ran in fp32
constexpr uint32_t kStatusPeerTimeout = 1u << 7;  // expert parallel: a rank did not reach a barrier

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t bits16) {
  return __uint_as_float(bits16 << 16);
}

// Round-to-nearest-even fp32 -> bf16 bits (finite inputs).
__device__ __forceinline__ uint32_t f32_to_bf16_rne(float v) {
  uint32_t u = __float_as_uint(v);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu) != 0)
    return (u >> 16) | 0x40u;
  return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}

// x ~= hi + lo with hi = bf16(x), lo = bf16(x - hi): 16 significant bits,
// relative error <= 2^-17.  x - hi is exact in fp32.
__device__ __forceinline__ void split_bf16(float x, uint32_t& hi, uint32_t& lo) {
  hi = f32_to_bf16_rne(x);
  const float r = __fsub_rn(x, bf16_bits_to_f32(hi));
  lo = f32_to_bf16_rne(r);
}

__device__ __forceinline__ uint32_t pack2(uint32_t lo16, uint32_t hi16) {
  return (lo16 & 0xFFFFu) | (hi16 << 16);
}

// Nibble pair k (0..3) of a Q4 word as a bf16x2 register holding exactly
// (q_k, q_{k+4}): OR the nibbles into the mantissa of 128.0 (0x4300) and
// subtract 128 (exact).
__device__ __forceinline__ uint32_t nibble_pair_bf16(uint32_t w, int k) {
  uint32_t v;
  const uint32_t s = w >> (4 * k);
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(v) : "r"(s), "r"(0x000F000Fu), "r"(0x43004300u));
  uint32_t out;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(out) : "r"(v), "r"(0x43004300u));
  return out;
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + C, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float d[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

// Reference sigmoid / silu op order (reference_ops.cpp:214-220):
// sigmoid(v) = 1 / (1 + exp(-v)); silu(v) = v * sigmoid(v).
__device__ __forceinline__ float ref_sigmoid(float v) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)));
}
__device__ __forceinline__ float ref_silu(float v) { return __fmul_rn(v, ref_sigmoid(v)); }

// Programmatic dependent launch: a kernel launched with the programmatic
// stream-serialisation attribute may start before its predecessor ends;
// pdl_wait() blocks until the predecessor has completed and flushed memory
// (a no-op for ordinary launches), pdl_trigger() lets the successor start.
#ifdef OSM_PHASE_TIMING
__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t % 100000000ull;
}
// kernel timeline (debug builds): slot 4q = first CTA start, 4q+1 = last CTA
// start, 4q+2 = last return from pdl_wait, 4q+3 = last CTA end
#define OSM_TL_SLOTS 16
__device__ __forceinline__ unsigned long long gtime_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#define TL_START(q) do { if (threadIdx.x == 0) { const unsigned long long t_ = gtime_ns(); \
  atomicMin(&g_tl[4 * (q)], t_); atomicMax(&g_tl[4 * (q) + 1], t_); } } while (0)
#define TL_WAITED(q) do { if (threadIdx.x == 0) atomicMax(&g_tl[4 * (q) + 2], gtime_ns()); } while (0)
#define TL_END(q) do { if (threadIdx.x == 0) atomicMax(&g_tl[4 * (q) + 3], gtime_ns()); } while (0)
#define TL_MARK(slot) do { if (threadIdx.x == 0) atomicMax(&g_tl[(slot)], gtime_ns()); } while (0)
#else
#define TL_MARK(slot) do { } while (0)
#define TL_START(q) do { } while (0)
#define TL_WAITED(q) do { } while (0)
#define TL_END(q) do { } while (0)
#endif
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- bulk asynchronous copies (global -> shared) tracked by an mbarrier ----
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}
// Makes initialised barriers visible to the async proxy (the copy engine).
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// One arrival that also expects `bytes` of copy completions on the barrier.
__device__ __forceinline__ void mbar_arrive_expect(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
// Adds `bytes` of expected copy completions without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// Copies `bytes` (a multiple of 16; both addresses 16-byte aligned) and
// signals their arrival on `bar`.  No multicast.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// Polls at most `polls` times (each try_wait may suspend briefly); false when
// the phase did not complete.
constexpr uint32_t kCopyPolls = 1u << 21;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kCopyPolls; ++i)
    if (mbar_test(bar, parity)) return true;
  return false;
}

// The first bounded wait of a consumer on a copy polls g_first_polls times
// (kCopyPolls unless lowered through osm_test_set_copy_wait_polls); when it
// gives up the caller records kStatusCopyTimeout and waits again with the
// full bound (mbar_wait), so the copies have landed before the data is read
// or the block exits.  One variable per translation unit, set by
// set_first_wait_polls() of that unit.
static __device__ uint32_t g_first_polls = kCopyPolls;
__device__ __forceinline__ bool mbar_wait_first(uint64_t* bar, uint32_t parity) {
  // read-only while kernels run (set from the host between launches): a
  // cached load, not one to memory on every wait
  const uint32_t n = __ldg(&g_first_polls);
  for (uint32_t i = 0; i < n; ++i)
    if (mbar_test(bar, parity)) return true;
  return false;
}
static inline cudaError_t set_first_wait_polls(uint32_t n) {
  return cudaMemcpyToSymbol(g_first_polls, &n, sizeof(n));
}

// Block-floating-point int8 digits of 8 consecutive activations (physical
// inputs k0..k0+7 of one group) for the B fragments: b0 takes the even
// positions, b1 the odd ones.  s = 2^e with 127 s > max|x_group|.
struct Digits {
  uint32_t b0[3], b1[3];
};
__device__ __forceinline__ int group_exponent(float m) {
  int E = (int)((__float_as_uint(m) >> 23) & 0xFF) - 127;
  if (E < -100) E = -100;   // zero / tiny groups: digits are 0 anyway
  if (E > 120) E = 120;     // keeps 2^-e finite
  return E - 5;             // |x| < 2^(E+1) = 64 s
}
// y = rint(x 2^(14-e)) (|y| < 2^20) split into balanced base-128 digits:
// y = d0 2^14 + d1 2^7 + d2 with |d| <= 64.
__device__ __forceinline__ Digits make_digits(const float (&v)[8], int e) {
  const float sc = __uint_as_float((uint32_t)(127 + 14 - e) << 23);  // 2^(14-e)
  uint32_t p[3][8];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int y = __float2int_rn(v[m] * sc);
    const int d2 = ((y + 64) & 127) - 64;
    const int y1 = (y - d2) >> 7;
    const int d1 = ((y1 + 64) & 127) - 64;
    const int d0 = (y1 - d1) >> 7;
    p[0][m] = (uint32_t)d0 & 0xFFu;
    p[1][m] = (uint32_t)d1 & 0xFFu;
    p[2][m] = (uint32_t)d2 & 0xFFu;
  }
  Digits D;
#pragma unroll
  for (int d = 0; d < 3; ++d) {
    D.b0[d] = p[d][0] | (p[d][2] << 8) | (p[d][4] << 16) | (p[d][6] << 24);
    D.b1[d] = p[d][1] | (p[d][3] << 8) | (p[d][5] << 16) | (p[d][7] << 24);
  }
  return D;
}

// Monotone map of finite floats (and -inf) to unsigned keys.
__device__ __forceinline__ uint32_t ord_key(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Block reductions over blockDim.x threads (<= 1024); `red` holds 32 floats.
__device__ __forceinline__ float block_reduce_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.0f;
  const int nw = blockDim.x >> 5;
  for (int w = 0; w < nw; ++w) s += red[w];
  return s;
}

__device__ __forceinline__ float block_reduce_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = -INFINITY;
  const int nw = blockDim.x >> 5;
  for (int w = 0; w < nw; ++w) s = fmaxf(s, red[w]);
  return s;
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

}  // namespace osm
