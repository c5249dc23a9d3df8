// osm_tcd.cu -- grouped expert projections for fp32 calls of three or more
// tokens on the 5th-generation tensor cores, with int8 digit planes
// (tcgen05.mma kind::i8).
//
// The expert half of run_qwen_sparse_moe_vulkan_accum (src/model/
// routed_moe.cpp:254-430: per routed expert gate/up GEMV -> SwiGLU -> down
// GEMV, then the weighted sum in pick order and the sigmoid-gated shared
// expert) as a grouped GEMM over chunks of <= kDgChunk pairs (token, pick)
// that share an expert.
//
// Numerics -- the group identity of shaders/q4_gemv.comp:44-60 with exact
// integer group sums, the same as the mma.sync kernels of osm_gemv.cu:
//  * A = the Q4 nibbles q (0..15), exact as unsigned int8;
//  * B = the activations of each (row, 64-wide group) as block floating
//    point x = s (d0 + d1 2^-7 + d2 2^-14), s a power of two, |d| <= 64
//    (make_digits; error <= 2^-20 max|x_group|); a pair's three digit planes
//    are three consecutive rows of B (N = 3 x pairs, rounded up to 16);
//  * per group the MMA gives D_d = sum_k q d_d exactly (s32), and the
//    epilogue adds s_w (s 2^-14) (D0 2^14 + D1 2^7 + D2) + b_w sum(x) in
//    fp32 (|D0 2^14 + D1 2^7 + D2| < 2^31).
// The weight scale s_w (bf16) differs per row and group, so each K group has
// its own accumulator in tensor memory, read out by the epilogue while the
// later groups run.
//
// Data: the digit planes of the call's activations are written per pair
// (digits_kernel; pair positions of the grouping are consecutive within a
// chunk), so one TMA copy brings a chunk's B tile in the 128-byte-swizzled
// K-major layout the MMA reads.  Items are (chunk, 128 weight rows); a CTA
// per SM walks its range of items.  Warps (480 threads):
//   0       producer: per item, the descriptor (smem) and bulk copies of the
//           item's weight scale / bias rows and the pairs' activation
//           scales; per four K groups, TMA copies of the Q4 rows (the tensor
//           maps of osm_tc.cu over the expert slab) and of the B tiles; no
//           multicast anywhere;
//   1, 2    MMA issuers (gate, up; down uses warp 1): per two K groups four
//           tcgen05.mma kind::i8 of K = 32 per matrix (A: int8 nibbles in
//           tensor memory, B: shared memory) into two group accumulators;
//   3-6     converters: Q4 words -> int8 A (tcgen05.st; per 8 nibbles the
//           even positions then the odd ones, the digit planes' order);
//   7-14    epilogue (TMEM lanes = weight rows, warp % 4 picks the lane
//           quarter): gate/up -- warps 7-10 the gate sums, 11-14 the up
//           sums; down -- 7-10 the even K groups, 11-14 the odd ones.  Per
//           group tcgen05.ld of the s32 sums, scale and add in fp32
//           registers; at the item's end one half's sums go through shared
//           memory to the other, then SwiGLU -> h rows (gate/up) or the
//           expert output rows (down).
// Every wait is bounded (tc_wait: two seconds, then the status bit and a
// CTA-wide abort flag; the epilogue warps take their exit decisions together
// so that none is left at a named barrier).
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "osm_common.cuh"
#include "osm_kernels.cuh"
#include "osm_tcgen05.cuh"

namespace osm {
namespace {

constexpr int kDgConv = 4;                          // converter warps
constexpr int kDgEpi = 8;                           // epilogue warps
constexpr int kDgConv0 = 3;                         // first converter warp
constexpr int kDgEpi0 = kDgConv0 + kDgConv;         // first epilogue warp
constexpr int kDgWarps = kDgEpi0 + kDgEpi;
constexpr int kDgThreads = kDgWarps * 32;
constexpr int kDgM = 128;                           // weight rows per item (MMA M)
constexpr int kDgN = 3 * kDgChunk;                  // B rows (digit rows) per chunk
constexpr int kDgGMax = 32;                         // K groups per row at most (K <= 2048)
constexpr uint32_t kBTile = (uint32_t)kDgN * 128;   // one B tile: 2 K groups of int8

template <bool DOWN>
struct DgCfg {
  static constexpr int NMAT = DOWN ? 1 : 2;         // gate and up share the activations
  static constexpr int RQ = DOWN ? 5 : 3;           // raw stages (four K groups each)
  static constexpr int RO = DOWN ? 4 : 2;           // A operand stages (two K groups each)
  // accumulators: two slots of two K groups; column (slot, group, matrix) * kDgN
  static constexpr uint32_t SLOT_COLS = 2 * NMAT * kDgN;
  static constexpr uint32_t A_COLS = NMAT * 32;     // 2 groups x 64 int8 per row
  static constexpr uint32_t TMEM_A = 2 * SLOT_COLS;
  static constexpr uint32_t TMEM_USED = TMEM_A + RO * A_COLS;
  static constexpr uint32_t TMEM_ALLOC = TMEM_USED <= 256 ? 256 : 512;
  static_assert(TMEM_USED <= 512, "tensor memory budget");
  static constexpr size_t QMAT = (size_t)kDgM * 128;       // 128 rows x 4 groups of Q4
  static constexpr size_t QSTAGE = (size_t)NMAT * QMAT;
  static constexpr size_t OFF_Q = 0;
  static constexpr size_t OFF_B = OFF_Q + (size_t)RQ * QSTAGE;          // two B tiles per raw stage
  static constexpr size_t WBUF = (size_t)NMAT * 2 * kDgM * kDgGMax * 2;  // scale, bias rows (bf16)
  static constexpr size_t OFF_W = OFF_B + (size_t)RQ * 2 * kBTile;
  static constexpr size_t XSBUF = (size_t)kDgChunk * kDgGMax * 8;       // pairs' {s 2^-14, sum}
  static constexpr size_t OFF_XS = OFF_W + 2 * WBUF;
  static constexpr size_t OFF_XT = OFF_XS + 2 * XSBUF;                   // the same, [group][pair]
  static constexpr size_t OFF_X = OFF_XT + XSBUF;                        // one half's sums
  static constexpr size_t XCH = (size_t)kDgM * kDgChunk * 4;
  static constexpr size_t OFF_DESC = OFF_X + XCH;
  static constexpr size_t OFF_BAR = OFF_DESC + 2 * 256;
  static constexpr int NBAR = 2 * RQ + 2 * RO + 2 * 2 + 2 * 2 + 2;
  static constexpr size_t OFF_MISC = OFF_BAR + (size_t)NBAR * 8;
  static constexpr size_t BYTES = OFF_MISC + 64 + 1024;  // + base alignment slack
  static_assert(OFF_B % 1024 == 0 && kBTile % 1024 == 0, "swizzle atoms");
  static_assert(BYTES <= 227 * 1024, "shared memory");
};

// kind::i8 instruction descriptor: s32 D, A unsigned 8-bit (nibbles), B
// signed 8-bit (digits), both K-major; N and M.
__device__ __forceinline__ uint32_t idesc8(int M, int N) {
  return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}
template <bool ACC>
__device__ __forceinline__ void mma_i8(uint32_t d, uint32_t a, uint64_t bd, uint32_t idesc) {
  if constexpr (ACC)
    asm volatile("tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, 1;" ::"r"(d), "r"(a), "l"(bd), "r"(idesc));
  else
    asm volatile("tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, 0;" ::"r"(d), "r"(a), "l"(bd), "r"(idesc));
}
__device__ __forceinline__ void epi_sync() {
  asm volatile("bar.sync 3, %0;" ::"n"(kDgEpi * 32) : "memory");
}
// Barrier of the epilogue warps that also ORs a flag across them.
__device__ __forceinline__ bool epi_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 4, %2, p;\n"
      " selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(kDgEpi * 32)
      : "memory");
  return r != 0;
}
// 2-D TMA copy (box 128 bytes x kDgN rows) signalled on bar; no multicast.
__device__ __forceinline__ void tma2(void* dst, const void* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(smem_addr(bar)), "r"(x), "r"(y)
      : "memory");
}

#ifdef OSM_DG_TRACE
// debug builds: event times (ns) of CTA 0 of the last launch of each kernel
__device__ unsigned long long g_dgt[2][16][512];
#define DGT(kind, idx)                                                                   \
  do {                                                                                   \
    if (blockIdx.x == 0 && (unsigned)(idx) < 512u) g_dgt[DOWN][kind][idx] = global_ns(); \
  } while (0)
#else
#define DGT(kind, idx) \
  do {                 \
  } while (0)
#endif

// One item as the producer decodes it (shared memory, two slots by item
// parity); end = 1 after the CTA's last item.
struct DgDesc {
  const uint8_t* ptr;
  int kind, pos0, ntok, r0, nrows, nk, slot, end;
  int orow[kDgChunk];  // down: output row (token * (k + 1) + pick) of each pair
};
static_assert(sizeof(DgDesc) <= 256, "descriptor slot");

template <bool DOWN>
__device__ __forceinline__ bool dg_item(const TcArgs& a, int item, DgDesc& it) {
  const int nmt = DOWN ? a.nmt_dn : a.nmt_gu;
  const int ch = item / nmt, mt = item - ch * nmt;
  const int2 cj = a.chunks[ch];
  const ActEntry en = a.act[cj.x];
  it.ptr = en.ptr;
  it.kind = en.kind;
  it.pos0 = en.off + cj.y;
  it.ntok = min(kDgChunk, en.cnt - cj.y);
  it.r0 = mt * kDgM;
  const int rows = DOWN ? a.dn.rows[en.kind] : a.gu.rows[en.kind];
  it.nrows = min(kDgM, rows - it.r0);
  it.nk = (DOWN ? a.dn.K[en.kind] : a.H) >> 6;
  it.slot = 0;
  it.end = 0;
  if (en.kind == 0 && en.ptr != nullptr && a.slab_stride)
    it.slot = (int)((uint64_t)(en.ptr - a.slab) / a.slab_stride);
  return it.ntok > 0 && it.nrows > 0 && en.ptr != nullptr;
}

template <bool DOWN>
__global__ void __launch_bounds__(kDgThreads, 1) dg_kernel(const DgArgs d, const __grid_constant__ DgMaps maps) {
  using C = DgCfg<DOWN>;
  const TcArgs& a = d.t;
  extern __shared__ unsigned char dgraw[];
  unsigned char* sm = dgraw + ((1024u - (smem_addr(dgraw) & 1023u)) & 1023u);
  uint64_t* qfull = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
  uint64_t* qempty = qfull + C::RQ;
  uint64_t* opfull = qempty + C::RQ;
  uint64_t* opempty = opfull + C::RO;
  uint64_t* accfull = opempty + C::RO;
  uint64_t* accempty = accfull + 2;
  uint64_t* scfull = accempty + 2;
  uint64_t* scempty = scfull + 2;
  uint64_t* drain = scempty + 2;
  DgDesc* desc = reinterpret_cast<DgDesc*>(sm + C::OFF_DESC);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + C::OFF_MISC);
  volatile int* abort = reinterpret_cast<volatile int*>(sm + C::OFF_MISC + 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < C::RQ; ++i) {
      mbar_init(&qfull[i], 1);
      mbar_init(&qempty[i], C::NMAT);  // one commit per MMA issuer
    }
    for (int i = 0; i < C::RO; ++i) {
      mbar_init(&opfull[i], kDgConv);
      mbar_init(&opempty[i], C::NMAT);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accfull[i], C::NMAT);  // one commit per MMA issuer
      mbar_init(&accempty[i], kDgEpi);  // every epilogue warp reads each slot
      mbar_init(&scfull[i], 1);
      mbar_init(&scempty[i], kDgEpi);
      mbar_init(&drain[i], 1);
    }
    *abort = 0;
    mbar_init_fence();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(s_tmem)),
                 "r"(C::TMEM_ALLOC));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *s_tmem;
  pdl_wait();
  const int nmt = DOWN ? a.nmt_dn : a.nmt_gu;
  const int n_items = *a.n_ch * nmt;
  const int per = (n_items + gridDim.x - 1) / gridDim.x;
  const int i0 = min(n_items, (int)blockIdx.x * per), i1 = min(n_items, i0 + per);
  const int sec0 = DOWN ? 2 : 0;        // tensor-map section of matrix 0
  // B maps by box height (16, 32, 48 digit rows = the item's npad)
  const unsigned char(*bmaps)[128] = DOWN ? maps.hd : maps.xd;
  const float2* qsrc = DOWN ? d.hq : d.xq;
  const int qstride = (DOWN ? a.Imax : a.H) >> 6;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      uint32_t qs = 0, jj = 0;
      bool ok = true;
      for (int item = i0; item <= i1 && ok; ++item) {
        DgDesc it;
        if (item < i1) {
          if (!dg_item<DOWN>(a, item, it)) continue;
          if (DOWN)
            for (int t = 0; t < it.ntok; ++t)
              it.orow[t] = a.pair_tok[it.pos0 + t] * a.kp1 + a.pair_pick[it.pos0 + t];
        } else {
          it.end = 1;  // after the last item
        }
        const int b = (int)(jj & 1);
        if (jj >= 2 && !tc_wait(&scempty[b], ((jj >> 1) - 1) & 1, abort, a.status)) break;
        desc[b] = it;
        if (it.end) {
          mbar_arrive(&scfull[b]);
          break;
        }
        // the item's scale / bias rows and its pairs' activation scales
        const int G = it.nk;
        const uint32_t wbytes = (uint32_t)(it.nrows * G * 2), xbytes = (uint32_t)(it.ntok * qstride * 8);
        mbar_arrive_expect(&scfull[b], (uint32_t)(C::NMAT * 2) * wbytes + xbytes);
        unsigned char* wb = sm + C::OFF_W + (size_t)b * C::WBUF;
#pragma unroll
        for (int m = 0; m < C::NMAT; ++m) {
          const uint64_t so = DOWN ? a.dn.s[it.kind] : (m ? a.gu.s2[it.kind] : a.gu.s[it.kind]);
          const uint64_t bo = DOWN ? a.dn.b[it.kind] : (m ? a.gu.b2[it.kind] : a.gu.b[it.kind]);
          const size_t roff = (size_t)it.r0 * G * 2;
          bulk_load(wb + (size_t)(2 * m) * kDgM * kDgGMax * 2, it.ptr + so + roff, wbytes, &scfull[b]);
          bulk_load(wb + (size_t)(2 * m + 1) * kDgM * kDgGMax * 2, it.ptr + bo + roff, wbytes, &scfull[b]);
        }
        bulk_load(sm + C::OFF_XS + (size_t)b * C::XSBUF, qsrc + (size_t)it.pos0 * qstride, xbytes,
                  &scfull[b]);
        ++jj;
        // Q4 rows and B tiles, four K groups per raw stage
        for (int kb = 0; kb < (G >> 2); ++kb, ++qs) {
          const int st = (int)(qs % C::RQ);
          if (qs >= (uint32_t)C::RQ && !tc_wait(&qempty[st], ((qs / C::RQ) - 1) & 1, abort, a.status)) {
            ok = false;
            break;
          }
          unsigned char* q = sm + C::OFF_Q + (size_t)st * C::QSTAGE;
          unsigned char* bt = sm + C::OFF_B + (size_t)st * 2 * kBTile;
          const int nb = (3 * it.ntok + 15) >> 4;      // box of 16 nb rows
          const void* bmap = &bmaps[nb - 1][0];
          DGT(0, qs);
          mbar_arrive_expect(&qfull[st], (uint32_t)(C::NMAT * C::QMAT + 2 * 16 * 128 * nb));
#pragma unroll
          for (int m = 0; m < C::NMAT; ++m)
            tma3(q + m * C::QMAT, &maps.q.m[it.kind][sec0 + m][0], kb * 32, it.r0, it.slot, &qfull[st]);
          tma2(bt, bmap, kb * 256, 3 * it.pos0, &qfull[st]);
          tma2(bt + kBTile, bmap, kb * 256 + 128, 3 * it.pos0, &qfull[st]);
        }
      }
      // no copy may still be landing when the CTA ends
      for (uint32_t q = qs > (uint32_t)C::RQ ? qs - C::RQ : 0; q < qs; ++q)
        tc_wait(&qfull[q % C::RQ], (q / C::RQ) & 1, abort, a.status);
      if (jj > 0) tc_wait(&scfull[(jj - 1) & 1], ((jj - 1) >> 1) & 1, abort, a.status);
    }
    __syncwarp();
  } else if (warp == 1 || warp == 2) {
    // ---------------- MMA issuers: warp 1 matrix 0, warp 2 matrix 1 ----------------
    const int m = warp - 1;
    if (lane == 0 && m < C::NMAT) {
      const uint64_t bdesc0 = desc_sw128(smem_addr(sm + C::OFF_B));
      uint32_t os = 0;
      for (uint32_t jj = 0;; ++jj) {
        const int b = (int)(jj & 1);
        if (!tc_wait(&scfull[b], (jj >> 1) & 1, abort, a.status)) break;
        const DgDesc it = desc[b];
        if (it.end) break;
        const int npad = (3 * it.ntok + 15) & ~15;
        const uint32_t idesc = idesc8(kDgM, npad);
        bool ok = true;
        for (int s = 0; s < (it.nk >> 1); ++s, ++os) {
          const int st = (int)(os % C::RO);
          const uint32_t qs = os >> 1;
          const int qst = (int)(qs % C::RQ);
          const int slot = (int)(os & 1);
          if ((os & 1) == 0 && !tc_wait(&qfull[qst], (qs / C::RQ) & 1, abort, a.status)) {
            ok = false;
            break;
          }
          if (!tc_wait(&opfull[st], (os / C::RO) & 1, abort, a.status)) {
            ok = false;
            break;
          }
          if (os >= 2 && !tc_wait(&accempty[slot], ((os >> 1) - 1) & 1, abort, a.status)) {
            ok = false;
            break;
          }
          fence_after();
          if (m == 0) DGT(3, os);
          // B: tile (os & 1) of raw stage qst; K steps of 32 bytes
          const uint64_t bd = bdesc0 + ((uint64_t)(qst * 2 + (int)(os & 1)) * kBTile >> 4);
          const uint32_t am = tmem + C::TMEM_A + (uint32_t)st * C::A_COLS + (uint32_t)(m * 32);
#pragma unroll
          for (int gi = 0; gi < 2; ++gi) {
            const uint32_t dm = tmem + (uint32_t)slot * C::SLOT_COLS + (uint32_t)((gi * C::NMAT + m) * kDgN);
            mma_i8<false>(dm, am + (uint32_t)(2 * gi) * 8u, bd + (uint64_t)(2 * gi * 2), idesc);
            mma_i8<true>(dm, am + (uint32_t)(2 * gi + 1) * 8u, bd + (uint64_t)((2 * gi + 1) * 2), idesc);
          }
          commit(&accfull[slot]);
          commit(&opempty[st]);
          if (os & 1) commit(&qempty[qst]);
        }
        if (!ok) break;
      }
      // no MMA may still be writing tensor memory when it is released (the
      // epilogue has waited for every one unless the CTA gave up early)
      commit(&drain[m]);
      for (int i = 0; i < 100 && !mbar_try_sleep(&drain[m], 0); ++i) {
      }
    }
    __syncwarp();
  } else if (warp < kDgEpi0) {
    // ---------------- converters: Q4 -> int8 A ----------------
    const int row = (warp & 3) * 32 + lane;            // tensor-memory lane = weight row
    const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
    uint32_t os = 0;
    for (uint32_t jj = 0;; ++jj) {
      const int b = (int)(jj & 1);
      if (!warp_wait(&scfull[b], (jj >> 1) & 1, abort, a.status)) break;
      const int nst = desc[b].nk >> 1;
      if (desc[b].end) break;
      bool ok = true;
      for (int s = 0; s < nst; ++s, ++os) {
        const int ost = (int)(os % C::RO);
        const uint32_t qs = os >> 1;
        const int qst = (int)(qs % C::RQ);
        if (os >= (uint32_t)C::RO && !warp_wait(&opempty[ost], ((os / C::RO) - 1) & 1, abort, a.status)) {
          ok = false;
          break;
        }
        if ((os & 1) == 0 && !warp_wait(&qfull[qst], (qs / C::RQ) & 1, abort, a.status)) {
          ok = false;
          break;
        }
        fence_after();  // the MMAs that read this operand stage have completed
        if (warp == kDgConv0 && lane == 0) DGT(1, os);
        const unsigned char* q = sm + C::OFF_Q + (size_t)qst * C::QSTAGE;
        const int sw = row & 7, c0 = 4 * (int)(os & 1);
#pragma unroll
        for (int m = 0; m < C::NMAT; ++m) {
          // the stage is 128-byte swizzled by the TMA copy: 16-byte chunk c
          // of row r sits at chunk c ^ (r & 7)
          const unsigned char* qrow = q + (size_t)m * C::QMAT + row * 128;
          uint32_t av[32];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 w = *reinterpret_cast<const uint4*>(qrow + (((c0 + c) ^ sw) << 4));
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              av[8 * c + 2 * e] = ww[e] & 0x0F0F0F0Fu;
              av[8 * c + 2 * e + 1] = (ww[e] >> 4) & 0x0F0F0F0Fu;
            }
          }
          st32(tmem + lane_addr + C::TMEM_A + (uint32_t)ost * C::A_COLS + (uint32_t)(m * 32), av);
        }
        wait_st();
        fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&opfull[ost]);
          if (warp == kDgConv0) DGT(2, os);
        }
      }
      if (!ok) break;
    }
  } else {
    // ---------------- epilogue ----------------
    const int half = (warp - kDgEpi0) >> 2;
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
    float* xch = reinterpret_cast<float*>(sm + C::OFF_X);
    const float2* xt = reinterpret_cast<const float2*>(sm + C::OFF_XT);
    uint32_t os = 0;  // operand stages (two K groups) so far
    for (uint32_t jj = 0;; ++jj) {
      const int b = (int)(jj & 1);
      const bool got = warp_wait(&scfull[b], (jj >> 1) & 1, abort, a.status);
      // one decision for all epilogue warps: they meet at named barriers
      if (epi_or(!got || desc[b].end)) break;
      const DgDesc& it = desc[b];
      const int G = it.nk, ntok = it.ntok;
      // pairs are processed in blocks of four (the last block's extra pairs
      // compute values nobody stores); their digit columns in 16-column loads
      const int nblk = (ntok + 3) >> 2;
      const int npieces = (12 * nblk + 15) >> 4;
      const uint16_t* wsb = reinterpret_cast<const uint16_t*>(sm + C::OFF_W + (size_t)b * C::WBUF);
      {
        // the pairs' activation scales, transposed to [group][pair] so that
        // a group's sixteen pairs are eight 16-byte loads
        const float2* xs = reinterpret_cast<const float2*>(sm + C::OFF_XS + (size_t)b * C::XSBUF);
        float2* xw = reinterpret_cast<float2*>(sm + C::OFF_XT);
        for (int i = (warp - kDgEpi0) * 32 + lane; i < G * kDgChunk; i += kDgEpi * 32)
          xw[i] = xs[(i & (kDgChunk - 1)) * qstride + (i >> 4)];
        epi_sync();
      }
      // gate/up: this half's matrix; down: the matrix (halves split the groups)
      const int m = DOWN ? 0 : half;
      const uint16_t* srow = wsb + (size_t)(2 * m) * kDgM * kDgGMax + (size_t)row * G;
      const uint16_t* brow = srow + (size_t)kDgM * kDgGMax;
      float acc[kDgChunk];
#pragma unroll
      for (int t = 0; t < kDgChunk; ++t) acc[t] = 0.0f;
      int wg = -1;
      uint2 swv = make_uint2(0u, 0u), bwv = swv;
      // the group's scale and bias (a window of four groups is read at a
      // time), then acc[t] += s_w (s_t 2^-14) V_t + b_w X_t for the pairs;
      // with all sixteen pairs live the pairs run without branches
      auto accum = [&](const uint32_t (&v)[kDgN], int g) {
        if ((g >> 2) != wg) {
          wg = g >> 2;
          swv = *reinterpret_cast<const uint2*>(srow + 4 * wg);
          bwv = *reinterpret_cast<const uint2*>(brow + 4 * wg);
        }
        const int j = g & 3;
        const uint32_t sbits = ((j & 2) ? swv.y : swv.x) >> ((j & 1) * 16);
        const uint32_t bbits = ((j & 2) ? bwv.y : bwv.x) >> ((j & 1) * 16);
        const float sw = __uint_as_float(sbits << 16), bw = __uint_as_float(bbits << 16);
        const float4* xg = reinterpret_cast<const float4*>(xt + g * kDgChunk);
        if (nblk == kDgChunk / 4) {
          float4 q[kDgChunk / 2];
#pragma unroll
          for (int i = 0; i < kDgChunk / 2; ++i) q[i] = xg[i];
#pragma unroll
          for (int t = 0; t < kDgChunk; ++t) {
            const float qx = (t & 1) ? q[t >> 1].z : q[t >> 1].x;
            const float qy = (t & 1) ? q[t >> 1].w : q[t >> 1].y;
            const int V = (int)v[3 * t] * 16384 + (int)v[3 * t + 1] * 128 + (int)v[3 * t + 2];
            acc[t] = fmaf(bw, qy, fmaf(sw * qx, (float)V, acc[t]));
          }
        } else {
#pragma unroll
          for (int tb = 0; tb < kDgChunk / 4; ++tb) {
            if (tb < nblk) {
              const float4 q01 = xg[2 * tb], q23 = xg[2 * tb + 1];
              const float qx[4] = {q01.x, q01.z, q23.x, q23.z}, qy[4] = {q01.y, q01.w, q23.y, q23.w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int t = 4 * tb + u;
                const int V = (int)v[3 * t] * 16384 + (int)v[3 * t + 1] * 128 + (int)v[3 * t + 2];
                acc[t] = fmaf(bw, qy[u], fmaf(sw * qx[u], (float)V, acc[t]));
              }
            }
          }
        }
      };
      for (int s = 0; s < (G >> 1); ++s, ++os) {
        const int slot = (int)(os & 1);
        // a wait that gives up sets the abort flag; this warp then skips to
        // the item's barriers below
        if (!warp_wait(&accfull[slot], (os >> 1) & 1, abort, a.status)) break;
        fence_after();
        if ((warp & 3) == 3 && lane == 0) DGT(4 + half, os);
        const uint32_t sbase = tmem + lane_addr + (uint32_t)slot * C::SLOT_COLS;
        if (!DOWN && nblk == 1) {
          // at most four pairs: both groups' sums in one round of loads
          uint32_t v0[kDgN], v1[kDgN];
          ld16(sbase + (uint32_t)(m * kDgN), *reinterpret_cast<uint32_t(*)[16]>(&v0[0]));
          ld16(sbase + (uint32_t)((C::NMAT + m) * kDgN), *reinterpret_cast<uint32_t(*)[16]>(&v1[0]));
          wait_ld();
          fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&accempty[slot]);
          accum(v0, 2 * s);
          accum(v1, 2 * s + 1);
        } else {
#pragma unroll
          for (int gi = 0; gi < 2; ++gi) {
            if (DOWN && gi != half) continue;
            uint32_t v[kDgN];
            const uint32_t base = sbase + (uint32_t)((gi * C::NMAT + m) * kDgN);
#pragma unroll
            for (int p = 0; p < 3; ++p) {
              if (p < npieces) {
                uint32_t (&vp)[16] = *reinterpret_cast<uint32_t(*)[16]>(&v[16 * p]);
                ld16(base + (uint32_t)(16 * p), vp);
              }
            }
            wait_ld();
            if (DOWN || gi == 1) {
              // this warp has read its columns of the slot
              fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&accempty[slot]);
            }
            accum(v, 2 * s + gi);
          }
        }
        if ((warp & 3) == 3 && lane == 0) DGT(6, os);
      }
      // ---- half 1's sums to shared memory, half 0 finishes the rows ----
      if (half == 1) {
#pragma unroll
        for (int t = 0; t < kDgChunk; ++t)
          if (t < ntok) xch[t * kDgM + row] = acc[t];
      }
      epi_sync();
      if (half == 0 && row < it.nrows && !*abort) {
#pragma unroll
        for (int t = 0; t < kDgChunk; ++t) {
          if (t < ntok) {
            const float o = xch[t * kDgM + row];
            if (DOWN) {
              a.partial[(size_t)it.orow[t] * a.H + it.r0 + row] = acc[t] + o;
            } else {
              // SiLU(g) u with the fast exponential and an IEEE reciprocal
              // (relative error about 1e-6)
              const float gv = acc[t];
              a.h[(size_t)(it.pos0 + t) * a.Imax + it.r0 + row] = gv * __frcp_rn(1.0f + __expf(-gv)) * o;
            }
          }
        }
      }
      epi_sync();
      if (lane == 0) mbar_arrive(&scempty[b]);
      if (warp == kDgEpi0 && lane == 0) DGT(7, jj);
      // a wait that gave up set the abort flag before the barriers above,
      // so every epilogue warp reads the same value here
      if (*abort) break;
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  pdl_trigger();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_ALLOC));
}

// Digit planes of rows x K fp32: one thread per 8 consecutive inputs, the 8
// threads of a 64-wide group adjacent in a warp.
__global__ void __launch_bounds__(256) digits_kernel(const float* __restrict__ src, const int* __restrict__ rowmap,
                                                     int nsrc, int rows, int K, int ld, uint8_t* __restrict__ dst,
                                                     float2* __restrict__ q) {
  pdl_wait();
  const int per_row = K >> 3;
  const size_t units = (size_t)rows * per_row;
  const size_t u = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool live = u < units;
  const size_t uu = live ? u : units - 1;
  const int r = (int)(uu / per_row), j = (int)(uu % per_row);
  int sr = r;
  if (rowmap) sr = min(max(rowmap[r], 0), nsrc - 1);
  const float* p = src + (size_t)sr * ld + 8 * j;
  const float4 u0 = __ldg(reinterpret_cast<const float4*>(p));
  const float4 u1 = __ldg(reinterpret_cast<const float4*>(p + 4));
  const float v[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
  float mx = 0.0f, sm = 0.0f;
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    mx = fmaxf(mx, fabsf(v[m]));
    sm += v[m];
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    sm += __shfl_xor_sync(0xFFFFFFFFu, sm, o);
  }
  pdl_trigger();
  if (!live) return;
  const int e = group_exponent(mx);
  const Digits D = make_digits(v, e);
#pragma unroll
  for (int dg = 0; dg < 3; ++dg)
    *reinterpret_cast<uint2*>(dst + ((size_t)r * 3 + dg) * K + 8 * j) = make_uint2(D.b0[dg], D.b1[dg]);
  if ((j & 7) == 0)
    q[(size_t)r * (K >> 6) + (j >> 3)] =
        make_float2(__uint_as_float((uint32_t)(127 + e - 14) << 23), sm);
}

}  // namespace

#ifdef OSM_DG_TRACE
extern "C" int osm_dbg_dg_trace(unsigned long long* out) {
  return (int)cudaMemcpyFromSymbol(out, g_dgt, sizeof(g_dgt));
}
#endif

namespace {

template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
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
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace

void launch_digits(const float* src, const int* rowmap, int nsrc, int rows, int K, int ld, uint8_t* dst,
                   float2* q, cudaStream_t s, uint64_t* launches) {
  const size_t units = (size_t)rows * (K >> 3);
  const int grid = (int)((units + 255) / 256);
  if (launches) *launches += 1;
  launch_pdl(digits_kernel, dim3(grid > 0 ? grid : 1), dim3(256), 0, s, src, rowmap, nsrc, rows, K, ld, dst, q);
}

void init_dg_attributes(int max_smem) {
  cudaFuncSetAttribute(dg_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(dg_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
}

bool dg_fits(int max_smem) {
  return DgCfg<false>::BYTES <= (size_t)max_smem && DgCfg<true>::BYTES <= (size_t)max_smem;
}

cudaError_t launch_dg_gateup(const DgArgs& a, const DgMaps& maps, int grid, cudaStream_t s,
                             uint64_t* launches) {
  if (launches) *launches += 1;
  return launch_pdl(dg_kernel<false>, dim3(grid), dim3(kDgThreads), DgCfg<false>::BYTES, s, a, maps);
}

cudaError_t launch_dg_down(const DgArgs& a, const DgMaps& maps, int grid, cudaStream_t s,
                           uint64_t* launches) {
  if (launches) *launches += 1;
  return launch_pdl(dg_kernel<true>, dim3(grid), dim3(kDgThreads), DgCfg<true>::BYTES, s, a, maps);
}

}  // namespace osm
