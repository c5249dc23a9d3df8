// osm_prefill.cu -- prefill-sized batches on the 5th-generation tensor cores.
//
// For large token counts the expert half of run_qwen_sparse_moe_vulkan_accum
// (src/model/routed_moe.cpp:254-430: per routed expert gate/up GEMV ->
// SwiGLU -> down GEMV, weighted sum in pick order, plus the sigmoid-gated
// shared expert) runs as a token-sorted grouped GEMM.  Pairs (token, pick) are
// grouped by expert into chunks of up to 128; an item is (chunk, 128 weight
// rows).  Per 64-wide K tile, 256 worker threads (two per weight row, each
// with half of the tile's K range):
//   * copy the tile's Q4 rows (MLX affine, eight nibbles per u32, LSB first:
//     reference_ops.cpp:47-63) and the chunk's fp16 activation rows into a
//     6-stage ring (cp.async, four tiles ahead);
//   * dequantise w = s q + b (bf16 scale and bias of group k/64,
//     reference_ops.cpp:11-67) into an fp16 tile in the 128-byte-swizzled
//     K-major layout the tensor core reads;
//   * one thread issues tcgen05.mma (kind::f16: fp16 x fp16 -> fp32 in tensor
//     memory), M = 128 rows, N = the chunk's pairs rounded up to 16, K = 64,
//     and commits to the tile's mbarrier, so the dequantisation of the next
//     tile overlaps the MMAs of this one.
// After an item's last tile the workers read the accumulators back
// (tcgen05.ld, lane = row) and store fp16: h = SiLU(g) u for gate/up
// (shaders/swiglu.comp), the expert output rows for down.  A final kernel sums
// each token's rows in pick order with its routing weights, then the shared
// expert's row with its gate (routed_moe.cpp:396-404).
//
// Operands are fp16 (the 16-bit tensor-core type with 11 significand bits):
// activations, dequantised weights, h and the expert rows are each rounded to
// fp16 once, which keeps outputs within 2e-3 of the fp32 reference (bf16
// operands, with 8 bits, measured about 7e-3).  Values at or beyond 65504
// set status bit kStatusF16Range.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "osm_common.cuh"
#include "osm_kernels.cuh"

namespace osm {
namespace {

constexpr int kPfThreads = 256;            // two threads per weight row of the item
constexpr int kPfM = 128;                  // weight rows per item (MMA M)
constexpr int kPfN = 128;                  // pairs per chunk (MMA N <= 128)
constexpr int kPfStages = 6;               // copy ring depth (K tiles)
constexpr int kPfAhead = kPfStages - 2;    // K tiles whose copies run ahead
constexpr int kPfATile = kPfM * 128;       // 128 rows x 64 fp16 = 16 KB
constexpr int kPfBTile = kPfN * 128;       // 128 pairs x 64 fp16 = 16 KB
constexpr int kPfQTile = kPfM * 32;        // 128 rows x 64 nibbles = 4 KB
constexpr size_t kPfOffB = 4 * (size_t)kPfATile;  // A: [2 buffers][2 matrices]
constexpr size_t kPfOffQ = kPfOffB + (size_t)kPfStages * kPfBTile;
constexpr size_t kPfSmem = kPfOffQ + (size_t)kPfStages * 2 * kPfQTile + 1024;  // + alignment
constexpr uint32_t kPfTmemCols = 256;      // gate accumulators 0..127, up 128..255

// ---- tcgen05 helpers ----
// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (start, stride and layout fields of the sm_100 format).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;           // leading offset: unused for swizzled K-major
  d |= (uint64_t)(1024 >> 4) << 32; // stride offset
  d |= (uint64_t)1 << 46;           // descriptor version
  d |= (uint64_t)2 << 61;           // 128-byte swizzle
  return d;
}
// Instruction descriptor, kind::f16: fp16 A and B (format 0), fp32 D
// (format 1), both K-major.
__device__ __forceinline__ uint32_t umma_idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(ad), "l"(bd), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit_pf() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait_pf() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// four bf16 scales (groups g..g+3) of one row; volatile so it is issued early
__device__ __forceinline__ uint2 ld_nc_u2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
__device__ __forceinline__ uint32_t h2_bits(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __half2 bits_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }

// Eight nibbles of w (consecutive K positions, LSB first) -> fp16(s q + b),
// four packed pairs in K order.  Each pair is built as (1024 + q) in fp16
// (exact), the 1024 is removed exactly, and s q + b is rounded once.
__device__ __forceinline__ uint4 dequant8(uint32_t w, __half2 s2, __half2 b2) {
  const uint32_t lo = w & 0x0F0F0F0Fu;          // q0 q2 q4 q6 in bytes 0..3
  const uint32_t hi = (w >> 4) & 0x0F0F0F0Fu;   // q1 q3 q5 q7
  const __half2 k1024 = bits_h2(0x64006400u);
  uint32_t r[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    // byte 0 = lo[p], byte 2 = hi[p]; bytes 1 and 3 replicate lo[p]'s sign (0)
    const uint32_t sel = (uint32_t)p | ((8u | p) << 4) | ((4u + p) << 8) | ((8u | p) << 12);
    const uint32_t v = prmt(lo, hi, sel) | 0x64006400u;
    r[p] = h2_bits(__hfma2(__hsub2(bits_h2(v), k1024), s2, b2));
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}
// bf16 bits -> fp16 (the scales and biases are bf16 in the expert format)
__device__ __forceinline__ __half2 bf16_to_h2(uint32_t b16) {
  const __half h = __float2half_rn(__uint_as_float(b16 << 16));
  return __halves2half2(h, h);
}

struct PfItem {
  const uint8_t* ptr;
  int kind, pos0, ntok, r0, nrows, nk;
};

// Item (chunk, 128-row tile) -> its description; false when it has no work
// (rows beyond a smaller expert kind, or an expert without a slot).
template <bool DOWN>
__device__ bool pf_item(const PfArgs& a, int item, PfItem& it) {
  const int nmt = DOWN ? a.nmt_dn : a.nmt_gu;
  const int ch = item / nmt, mt = item - ch * nmt;
  const int2 cj = a.chunks[ch];
  const ActEntry en = a.act[cj.x];
  it.ptr = en.ptr;
  it.kind = en.kind;
  it.pos0 = en.off + cj.y;
  it.ntok = min(kPfN, en.cnt - cj.y);
  it.r0 = mt * kPfM;
  const int rows = DOWN ? a.dn.rows[en.kind] : a.gu.rows[en.kind];
  it.nrows = min(kPfM, rows - it.r0);
  it.nk = (DOWN ? a.dn.K[en.kind] : a.H) >> 6;
  return it.ntok > 0 && it.nrows > 0 && en.ptr != nullptr;
}
template <bool DOWN>
__device__ int pf_next(const PfArgs& a, int i, int i1, PfItem& it) {
  for (; i < i1; ++i)
    if (pf_item<DOWN>(a, i, it)) return i;
  return i1;
}

template <bool DOWN>
__global__ void __launch_bounds__(kPfThreads, 1) pf_gemm_kernel(PfArgs a) {
  constexpr int NMAT = DOWN ? 1 : 2;  // gate and up share the activations
  constexpr int NARR = 2 * NMAT;      // scale and bias arrays
  extern __shared__ unsigned char pfraw[];
  __shared__ __align__(8) uint64_t bar_mma[kPfStages];
  __shared__ __align__(8) uint64_t bar_acc;
  __shared__ uint32_t s_tmem;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  unsigned char* sm = pfraw + ((1024u - (smem_addr(pfraw) & 1023u)) & 1023u);
  unsigned char* Abuf = sm;
  unsigned char* Bbuf = sm + kPfOffB;
  unsigned char* Qbuf = sm + kPfOffQ;
  if (t == 0) {
    for (int s = 0; s < kPfStages; ++s) mbar_init(&bar_mma[s], 1);
    mbar_init(&bar_acc, 1);
    mbar_init_fence();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(&s_tmem)),
                 "r"(kPfTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  pdl_wait();
  const int n_items = *a.n_ch * (DOWN ? a.nmt_dn : a.nmt_gu);
  const int per = (n_items + gridDim.x - 1) / gridDim.x;
  const int i0 = min(n_items, (int)blockIdx.x * per), i1 = min(n_items, i0 + per);

  // ---- copy side: walks the same K tiles kPfAhead tiles ahead ----
  PfItem li;
  int litem = pf_next<DOWN>(a, i0, i1, li), lkt = 0;
  const int row = t & (kPfM - 1), kh = t >> 7;  // weight row, half of the K tile
  int tok[4];
  auto load_tok = [&]() {
    if (DOWN || litem >= i1) return;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = (t >> 3) + 32 * j;
      tok[j] = n < li.ntok ? a.pair_tok[li.pos0 + n] : 0;
    }
  };
  load_tok();
  auto issue_load = [&](uint32_t step) {
    if (litem < i1) {
      const int st = (int)(step % kPfStages);
      // this thread's 16 bytes (32 nibbles) of its row: it dequantises them itself
      unsigned char* qdst = Qbuf + (size_t)st * 2 * kPfQTile + row * 32 + kh * 16;
      unsigned char* bdst = Bbuf + (size_t)st * kPfBTile;
      if (row < li.nrows) {
        const size_t rowb = DOWN ? (size_t)(a.dn.K[li.kind] >> 1) : (size_t)(a.H >> 1);
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
          const uint64_t off = DOWN ? a.dn.w[li.kind] : (m ? a.gu.w2[li.kind] : a.gu.w[li.kind]);
          cp16(qdst + m * kPfQTile, li.ptr + off + (size_t)(li.r0 + row) * rowb + (size_t)lkt * 32 + kh * 16);
        }
      }
      const int c = t & 7;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = (t >> 3) + 32 * j;
        if (n < li.ntok) {
          const uint16_t* src = DOWN ? a.hb + (size_t)(li.pos0 + n) * a.Imax + lkt * 64 + c * 8
                                     : a.xb + (size_t)tok[j] * a.H + lkt * 64 + c * 8;
          cp16(bdst + n * 128 + ((c ^ (n & 7)) << 4), src);
        }
      }
      if (++lkt == li.nk) {
        litem = pf_next<DOWN>(a, litem + 1, i1, li);
        lkt = 0;
        load_tok();
      }
    }
    cp_commit_pf();  // one group per K tile, empty ones included
  };
  for (int p = 0; p < kPfAhead; ++p) issue_load((uint32_t)p);

  // ---- compute side ----
  PfItem ci;
  int citem = pf_next<DOWN>(a, i0, i1, ci);
  auto scale_ptr = [&](const PfItem& it, int arr, int kb) -> const uint8_t* {
    uint64_t off;
    int G;
    if (DOWN) {
      off = arr ? a.dn.b[it.kind] : a.dn.s[it.kind];
      G = a.dn.K[it.kind] >> 6;
    } else {
      off = arr == 0 ? a.gu.s[it.kind] : arr == 1 ? a.gu.b[it.kind] : arr == 2 ? a.gu.s2[it.kind] : a.gu.b2[it.kind];
      G = a.H >> 6;
    }
    return it.ptr + off + (size_t)(it.r0 + row) * G * 2 + (size_t)kb * 2;
  };
  uint2 sc_cur[NARR], sc_nxt[NARR];
#pragma unroll
  for (int r = 0; r < NARR; ++r) {
    sc_cur[r] = make_uint2(0u, 0u);
    sc_nxt[r] = make_uint2(0u, 0u);
  }
  if (citem < i1 && row < ci.nrows)
#pragma unroll
    for (int r = 0; r < NARR; ++r) sc_cur[r] = ld_nc_u2(scale_ptr(ci, r, 0));
  uint32_t s = 0, nacc = 0;
  while (citem < i1) {
    PfItem ni;
    const int nitem = pf_next<DOWN>(a, citem + 1, i1, ni);
    const int npad = (ci.ntok + 15) & ~15;
    const uint32_t idesc = umma_idesc_f16(kPfM, npad);
    for (int kb = 0; kb < ci.nk; kb += 4) {
      // the next four groups' scales, one block ahead
      if (kb + 4 < ci.nk) {
        if (row < ci.nrows)
#pragma unroll
          for (int r = 0; r < NARR; ++r) sc_nxt[r] = ld_nc_u2(scale_ptr(ci, r, kb + 4));
      } else if (nitem < i1 && row < ni.nrows) {
#pragma unroll
        for (int r = 0; r < NARR; ++r) sc_nxt[r] = ld_nc_u2(scale_ptr(ni, r, 0));
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk, ++s) {
        const int kt = kb + kk;
        const int st = (int)(s % kPfStages);
        // stage (s - 2) and A buffer s & 1 were last read by the MMAs of step s - 2
        if (s >= 2) {
          const uint32_t ps = s - 2;
          if (!mbar_wait_first(&bar_mma[ps % kPfStages], (ps / kPfStages) & 1)) {
            if (t == 0) atomicOr(a.status, kStatusCopyTimeout);
            mbar_wait(&bar_mma[ps % kPfStages], (ps / kPfStages) & 1);
          }
        }
        issue_load(s + kPfAhead);
        cp_wait_pf<kPfAhead>();  // this thread's copies of step s have landed
        // dequantise this thread's 32 weights of its row in each matrix (the
        // Q4 bytes it copied itself; the activation rows are covered by the
        // barrier before the MMAs)
        const unsigned char* qrow = Qbuf + (size_t)st * 2 * kPfQTile + row * 32 + kh * 16;
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
          const uint2 sv = sc_cur[2 * m], bv = sc_cur[2 * m + 1];
          const uint32_t s16 = ((kk < 2 ? sv.x : sv.y) >> ((kk & 1) * 16)) & 0xFFFFu;
          const uint32_t b16 = ((kk < 2 ? bv.x : bv.y) >> ((kk & 1) * 16)) & 0xFFFFu;
          const __half2 s2 = bf16_to_h2(s16), b2 = bf16_to_h2(b16);
          const uint4 w0 = *reinterpret_cast<const uint4*>(qrow + m * kPfQTile);
          const uint32_t wd[4] = {w0.x, w0.y, w0.z, w0.w};
          unsigned char* arow = Abuf + (size_t)((s & 1) * 2 + m) * kPfATile + row * 128;
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(arow + (((4 * kh + c) ^ (row & 7)) << 4)) = dequant8(wd[c], s2, b2);
        }
        // generic-proxy writes (cp.async, stores) -> the tensor core's async proxy
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (t == 0) {
          tc_fence_after();
#pragma unroll
          for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              const uint64_t ad = umma_desc_sw128(smem_addr(Abuf + (size_t)((s & 1) * 2 + m) * kPfATile + ks * 32));
              const uint64_t bd = umma_desc_sw128(smem_addr(Bbuf + (size_t)st * kPfBTile + ks * 32));
              tc_mma(tmem + (uint32_t)(m * 128), ad, bd, idesc, (kt | ks) != 0 ? 1u : 0u);
            }
          tc_commit(&bar_mma[st]);
          if (kt == ci.nk - 1) tc_commit(&bar_acc);
        }
      }
#pragma unroll
      for (int r = 0; r < NARR; ++r) sc_cur[r] = sc_nxt[r];
    }
    // ---- epilogue: accumulators -> fp16 rows ----
    if (!mbar_wait_first(&bar_acc, nacc & 1)) {
      if (t == 0) atomicOr(a.status, kStatusCopyTimeout);
      mbar_wait(&bar_acc, nacc & 1);
    }
    ++nacc;
    tc_fence_after();
    // warp w reads tensor-memory lanes 32 (w % 4) .. +31; warps w and w + 4
    // take alternate 16-column blocks
    const int erow = (warp & 3) * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    bool over = false;
    for (int c0 = 16 * (warp >> 2); c0 < npad; c0 += 32) {
      uint32_t g[16], u[16];
      tc_ld16(lane_base + (uint32_t)c0, g);
      if (!DOWN) tc_ld16(lane_base + 128u + (uint32_t)c0, u);
      tc_wait_ld();
      if (erow < ci.nrows) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int n = c0 + j;
          if (n < ci.ntok) {
            const float v = DOWN ? __uint_as_float(g[j])
                                 : __fmul_rn(ref_silu(__uint_as_float(g[j])), __uint_as_float(u[j]));
            over |= !(fabsf(v) < 65504.0f);
            const uint16_t hv = __half_as_ushort(__float2half_rn(v));
            if (DOWN) a.pb[(size_t)(ci.pos0 + n) * a.H + ci.r0 + erow] = hv;
            else a.hb[(size_t)(ci.pos0 + n) * a.Imax + ci.r0 + erow] = hv;
          }
        }
      }
    }
    if (over) atomicOr(a.status, kStatusF16Range);
    tc_fence_before();
    citem = nitem;
    ci = ni;
  }
  cp_wait_pf<0>();
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPfTmemCols));
}

// out[b] = sum over picks j in order of w[b][j] * row(tp_pos[b][j]), then the
// shared expert's row scaled by sg[b], then the residual; each element in
// fp32 with one rounding per operation.  Eight consecutive elements per
// thread (H % 8 == 0): 16-byte row loads.  F16OUT: out holds fp16 rows
// (values beyond the fp16 range set kStatusF16Range).
template <bool F16OUT>
__global__ void __launch_bounds__(256) combine_bf16_kernel(
    const uint16_t* __restrict__ pb, const int* __restrict__ tp_pos, const float* __restrict__ w,
    const float* __restrict__ sg, const float* __restrict__ res, void* __restrict__ out, int H, int k,
    unsigned int* status) {
  pdl_wait();
  const int b = blockIdx.x;  // rows in x: more than 65535 of them are allowed
  const int i = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (i >= H) return;
  const int kp = k + (sg != nullptr ? 1 : 0);
  const int* tp = tp_pos + (size_t)b * kp;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < kp; ++j) {
    const float wj = j < k ? w[(size_t)b * k + j] : sg[b];
    const uint4 q = *reinterpret_cast<const uint4*>(pb + (size_t)tp[j] * H + i);
    const uint32_t qq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&qq[u]));
      acc[2 * u] = __fadd_rn(acc[2 * u], __fmul_rn(wj, v.x));
      acc[2 * u + 1] = __fadd_rn(acc[2 * u + 1], __fmul_rn(wj, v.y));
    }
  }
  if (res) {
    const float4 r0 = *reinterpret_cast<const float4*>(res + (size_t)b * H + i);
    const float4 r1 = *reinterpret_cast<const float4*>(res + (size_t)b * H + i + 4);
    const float rr[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
    for (int u = 0; u < 8; ++u) acc[u] = __fadd_rn(rr[u], acc[u]);
  }
  if (F16OUT) {
    bool over = false;
    uint32_t o[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      over |= fabsf(acc[2 * u]) >= 65504.0f || fabsf(acc[2 * u + 1]) >= 65504.0f;
      const __half2 hv = __floats2half2_rn(acc[2 * u], acc[2 * u + 1]);
      o[u] = *reinterpret_cast<const uint32_t*>(&hv);
    }
    if (over) atomicOr(status, kStatusF16Range);
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + (size_t)b * H + i) =
        make_uint4(o[0], o[1], o[2], o[3]);
  } else {
    float* op = static_cast<float*>(out) + (size_t)b * H + i;
    *reinterpret_cast<float4*>(op) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    *reinterpret_cast<float4*>(op + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
}

// out[t] = sum over p < k, in order, of row(pos[t k + p]), then + extra[t]:
// fp16 rows, fp32 sums with one rounding per add; eight elements per thread.
__global__ void __launch_bounds__(256) gather_sum_rows_kernel(
    const uint16_t* __restrict__ rows, const int64_t* __restrict__ pos, const uint16_t* __restrict__ extra,
    float* __restrict__ out, int H, int k) {
  const int t = blockIdx.x;
  const int i = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (i >= H) return;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  auto add_row = [&](const uint16_t* r) {
    const uint4 q = *reinterpret_cast<const uint4*>(r + i);
    const uint32_t qq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&qq[u]));
      acc[2 * u] = __fadd_rn(acc[2 * u], v.x);
      acc[2 * u + 1] = __fadd_rn(acc[2 * u + 1], v.y);
    }
  };
  for (int p = 0; p < k; ++p) add_row(rows + (size_t)pos[(size_t)t * k + p] * H);
  if (extra) add_row(extra + (size_t)t * H);
  float* op = out + (size_t)t * H + i;
  *reinterpret_cast<float4*>(op) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  *reinterpret_cast<float4*>(op + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
}

template <typename Kern, typename... Args>
void launch_pdl_pf(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace

void init_prefill_attributes(int max_smem) {
  if ((size_t)max_smem < kPfSmem) return;
  cudaFuncSetAttribute(pf_gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPfSmem);
  cudaFuncSetAttribute(pf_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPfSmem);
}

bool prefill_configure(const PfArgs& a, int has_shared, int max_smem, size_t* smem) {
  if ((size_t)max_smem < kPfSmem) return false;
  if (a.H % 256 || a.H > 8192) return false;  // whole blocks of four K tiles
  const int nk = has_shared ? 2 : 1;
  for (int kd = 0; kd < nk; ++kd) {
    if (a.gu.K[kd] != a.H || a.dn.rows[kd] != a.H) return false;
    if (a.dn.K[kd] % 256 || a.dn.K[kd] > a.Imax) return false;
    const uint64_t w[3] = {a.gu.w[kd], a.gu.w2[kd], a.dn.w[kd]};
    for (uint64_t v : w)
      if (v % 16) return false;  // 16-byte row copies
    const uint64_t sc[6] = {a.gu.s[kd], a.gu.b[kd], a.gu.s2[kd], a.gu.b2[kd], a.dn.s[kd], a.dn.b[kd]};
    for (uint64_t v : sc)
      if (v % 8) return false;   // 8-byte scale reads
  }
  *smem = kPfSmem;
  return true;
}

void launch_prefill_gateup(const PfArgs& a, int grid, size_t smem, cudaStream_t s, uint64_t* launches) {
  launch_pdl_pf(pf_gemm_kernel<false>, dim3(grid), dim3(kPfThreads), smem, s, a);
  if (launches) *launches += 1;
}

void launch_prefill_down(const PfArgs& a, int grid, size_t smem, cudaStream_t s, uint64_t* launches) {
  launch_pdl_pf(pf_gemm_kernel<true>, dim3(grid), dim3(kPfThreads), smem, s, a);
  if (launches) *launches += 1;
}

void launch_gather_sum_rows(const uint16_t* rows, const int64_t* pos, const uint16_t* extra,
                            float* out, int T, int H, int k, cudaStream_t s, uint64_t* launches) {
  gather_sum_rows_kernel<<<dim3(T, (H / 8 + 255) / 256), 256, 0, s>>>(rows, pos, extra, out, H, k);
  if (launches) *launches += 1;
}

void launch_combine_bf16(const uint16_t* pb, const int* tp_pos, const float* weights,
                         const float* sgate, const float* residual, void* out, bool f16_out,
                         unsigned int* status, int B, int H, int k, cudaStream_t s,
                         uint64_t* launches) {
  const dim3 grid(B, (H / 8 + 255) / 256);
  if (f16_out)
    launch_pdl_pf(combine_bf16_kernel<true>, grid, dim3(256), 0, s, pb, tp_pos, weights, sgate,
                  residual, out, H, k, status);
  else
    launch_pdl_pf(combine_bf16_kernel<false>, grid, dim3(256), 0, s, pb, tp_pos, weights, sgate,
                  residual, out, H, k, status);
  if (launches) *launches += 1;
}

}  // namespace osm

namespace osm {
cudaError_t set_first_wait_polls_prefill(uint32_t polls) { return set_first_wait_polls(polls); }
}  // namespace osm
