// osm_tc.cu -- grouped expert projections on the 5th-generation tensor cores
// with warp specialisation, for every call of three or more tokens.
//
// The expert half of run_qwen_sparse_moe_vulkan_accum (src/model/
// routed_moe.cpp:254-430: per routed expert gate/up GEMV -> SwiGLU -> down
// GEMV, then the weighted sum in pick order and the sigmoid-gated shared
// expert) runs as a grouped GEMM over chunks of pairs (token, pick) that share
// an expert.  An item is (chunk, 128 weight rows); a CTA per SM walks its
// range of items.  Its warps:
//   warp 0      producer: per 64-wide K group, one TMA copy of the item's 128
//               Q4 weight rows per matrix (tensor maps over the expert slab,
//               no multicast) and one bulk copy per activation row into a
//               ring of raw stages;
//   warp 1      MMA issuer: tcgen05.mma with A (weights) in tensor memory and
//               B (activations) in shared memory, fp32 accumulators in
//               tensor memory, double-buffered per item;
//   warps 2-9   converters: raw Q4 -> 16-bit A planes written to tensor memory
//               (tcgen05.st), raw activations -> 16-bit B planes in the
//               128-byte-swizzled K-major layout;
//   warps 10-13 epilogue: accumulators (tcgen05.ld) -> SwiGLU h rows (gate/up)
//               or expert output rows (down).
//
// Two numerics, chosen per call:
//  * PRECISE (fp32 calls, outputs within 1e-4 of the fp32 reference): bf16
//    operands in planes.  A = s q exactly as hi + lo (s q has at most 12
//    significant bits, so the bf16 residual of bf16(s q) is exact); B = x as
//    hi + mid (16 significant bits).  Three passes hi*hi + hi*mid + lo*hi per
//    K group, all into one fp32 accumulator; the bias term sum_g b[r,g] X[t,g]
//    (X = group sums of the activations, the group identity of
//    shaders/q4_gemv.comp:44-60) is one more K step at the end of the item,
//    A = the bf16 biases (exact), B = X as hi + mid.
//  * FAST (OSM_PREFILL_BF16, outputs within 2e-3): fp16 operands, one pass,
//    A = fp16(s q + b) rounded once, B = fp16 activations.
//
// MLX affine Q4 (reference_ops.cpp:11-67): eight nibbles per u32, LSB first,
// group 64 along the input dimension, bf16 scale and bias per (row, group).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "osm_common.cuh"
#include "osm_kernels.cuh"
#include "osm_tcgen05.cuh"

namespace osm {
namespace {

constexpr int kTcConv = 8;                         // converter warps
constexpr int kTcEpi = 4;                          // epilogue warps
constexpr int kTcMma2 = 2 + kTcConv + kTcEpi;     // the second MMA issuer (gate/up: up)
constexpr int kTcWarps = kTcMma2 + 1;
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kTcM = 128;                          // weight rows per item (MMA M)

template <bool PRECISE, bool DOWN>
struct TcCfg {
  static constexpr int NMAT = DOWN ? 1 : 2;        // gate and up share the activations
  static constexpr int NMAX = PRECISE ? kTcChunkPrecise : kTcChunkFast;
  static constexpr int PA = PRECISE ? 2 : 1;       // A planes
  static constexpr int PB = PRECISE ? 2 : 1;       // B planes
  static constexpr int PASSES = PRECISE ? 3 : 1;
  // PRECISE keeps the hi*hi products and the two correction passes in
  // separate accumulators: the tensor core's fp32 accumulation loses up to
  // about an ulp of the accumulator per step, so the small correction terms
  // are summed among themselves and added to the main sum once, in fp32.
  static constexpr int NACC = PRECISE ? 2 : 1;
  static constexpr int RO = DOWN ? 3 : 2;               // operand stages (one K group each)
  static constexpr int RQ = DOWN ? 8 : 4;               // weight stages (four K groups each)
  static constexpr uint32_t ACC_COLS = NMAT * NACC * NMAX;  // one accumulator buffer
  static constexpr uint32_t A_COLS = NMAT * PA * 32;    // one operand stage of A
  static constexpr uint32_t TMEM_A = 2 * ACC_COLS;
  static constexpr uint32_t TMEM_USED = TMEM_A + RO * A_COLS;
  static constexpr uint32_t TMEM_ALLOC = TMEM_USED <= 256 ? 256 : 512;
  static_assert(TMEM_USED <= 512, "tensor memory budget");
  // shared memory (offsets from a 1024-aligned base)
  static constexpr size_t QMAT = (size_t)kTcM * 128;   // 128 rows x 4 groups of Q4
  static constexpr size_t QSTAGE = (size_t)NMAT * QMAT;
  static constexpr size_t OFF_Q = 0;
  static constexpr size_t BPLANE = (size_t)NMAX * 128;
  static constexpr size_t OFF_B = OFF_Q + (size_t)RQ * QSTAGE;
  static constexpr size_t OFF_X = OFF_B + (size_t)RO * PB * BPLANE;
  static constexpr size_t XS_BYTES = PRECISE ? (size_t)NMAX * 32 * 4 : 0;
  static constexpr size_t OFF_BAR = OFF_X + XS_BYTES;
  static constexpr int NBAR = 2 * RQ + 2 * RO + 4;
  static constexpr size_t OFF_MISC = OFF_BAR + (size_t)NBAR * 8;
  static constexpr size_t BYTES = OFF_MISC + 64 + 1024;  // + base alignment slack
  // activation values a converter thread loads per K group: PRECISE 8 fp32
  // of one row (32 rows x 8 threads); FAST 8 fp16 of up to 3 rows
  // converter split: each weight row of each matrix is converted by CU
  // threads, each taking NW of the group's 8 words (NW * 4 tensor-memory
  // columns per plane)
  static constexpr int CU = kTcConv * 32 / (NMAT * kTcM);
  static constexpr int NW = 8 / CU;
  // activation rows per thread and K group: PRECISE 4 fp32 of one row (32
  // rows x 16 threads); FAST 16 bytes of up to 2 rows (96 rows x 8 chunks)
  static constexpr int NR = PRECISE ? NMAX * 16 / (kTcConv * 32)
                                    : (NMAX * 8 + kTcConv * 32 - 1) / (kTcConv * 32);
  static constexpr int BVEC = NR;                       // 16-byte vectors per thread and group
  static_assert(!PRECISE || (NMAX * 16) % (kTcConv * 32) == 0, "precise activation split");
  static_assert(CU >= 1 && 8 % CU == 0, "converter split");
};

#ifdef OSM_TC_TRACE
// debug builds: event times (ns) of CTA 0 of the last launch
__device__ unsigned long long g_tct[8][1024];
#define TCT(kind, idx)                                                              \
  do {                                                                              \
    if (!DOWN && blockIdx.x == 0 && (unsigned)(idx) < 1024u) g_tct[kind][idx] = global_ns(); \
  } while (0)
#else
#define TCT(kind, idx) \
  do {                 \
  } while (0)
#endif

struct TcItem {
  const uint8_t* ptr;
  int kind, pos0, ntok, r0, nrows, nk, slot;
};

template <bool PRECISE, bool DOWN>
__device__ __forceinline__ bool tc_item(const TcArgs& a, int item, TcItem& it) {
  using C = TcCfg<PRECISE, DOWN>;
  const int nmt = DOWN ? a.nmt_dn : a.nmt_gu;
  const int ch = item / nmt, mt = item - ch * nmt;
  const int2 cj = a.chunks[ch];
  const ActEntry en = a.act[cj.x];
  it.ptr = en.ptr;
  it.kind = en.kind;
  it.pos0 = en.off + cj.y;
  it.ntok = min(C::NMAX, en.cnt - cj.y);
  it.r0 = mt * kTcM;
  const int rows = DOWN ? a.dn.rows[en.kind] : a.gu.rows[en.kind];
  it.nrows = min(kTcM, rows - it.r0);
  it.nk = (DOWN ? a.dn.K[en.kind] : a.H) >> 6;
  it.slot = 0;
  if (en.kind == 0 && en.ptr != nullptr && a.slab_stride)
    it.slot = (int)((uint64_t)(en.ptr - a.slab) / a.slab_stride);
  return it.ntok > 0 && it.nrows > 0 && en.ptr != nullptr;
}

template <bool PRECISE, bool DOWN>
__global__ void __launch_bounds__(kTcThreads, 1) tc_kernel(const TcArgs a, const __grid_constant__ TcMaps maps) {
  using C = TcCfg<PRECISE, DOWN>;
  extern __shared__ unsigned char tcraw[];
  unsigned char* sm = tcraw + ((1024u - (smem_addr(tcraw) & 1023u)) & 1023u);
  uint64_t* qfull = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
  uint64_t* qempty = qfull + C::RQ;
  uint64_t* opfull = qempty + C::RQ;
  uint64_t* opempty = opfull + C::RO;
  uint64_t* accfull = opempty + C::RO;
  uint64_t* accempty = accfull + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + C::OFF_MISC);
  volatile int* abort = reinterpret_cast<volatile int*>(sm + C::OFF_MISC + 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < C::RQ; ++i) {
      mbar_init(&qfull[i], 1);
      mbar_init(&qempty[i], kTcConv);
    }
    for (int i = 0; i < C::RO; ++i) {
      mbar_init(&opfull[i], kTcConv);
      mbar_init(&opempty[i], C::NMAT);   // one commit per MMA issuer
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accfull[i], C::NMAT);
      mbar_init(&accempty[i], kTcEpi);
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
  const int sec0 = DOWN ? 2 : 0;  // tensor-map section of matrix 0

  if (warp == 0) {
    // ---------------- producer: weight tiles, four K groups per stage ----------------
    if (lane == 0) {
      uint32_t qs = 0;
      bool ok = true;
      for (int item = i0; item < i1 && ok; ++item) {
        TcItem it;
        if (!tc_item<PRECISE, DOWN>(a, item, it)) continue;
        for (int kb = 0; kb < (it.nk >> 2); ++kb, ++qs) {
          const int st = (int)(qs % C::RQ);
          if (qs >= (uint32_t)C::RQ && !tc_wait(&qempty[st], ((qs / C::RQ) - 1) & 1, abort, a.status)) {
            ok = false;
            break;
          }
          unsigned char* q = sm + C::OFF_Q + (size_t)st * C::QSTAGE;
          TCT(0, qs);
          mbar_arrive_expect(&qfull[st], (uint32_t)(C::NMAT * C::QMAT));
#pragma unroll
          for (int m = 0; m < C::NMAT; ++m)
            tma3(q + m * C::QMAT, &maps.m[it.kind][sec0 + m][0], kb * 32, it.r0, it.slot, &qfull[st]);
        }
      }
      // no copy may still be landing when the CTA ends: wait for the stages
      // the converters have not released
      for (uint32_t q = qs > (uint32_t)C::RQ ? qs - C::RQ : 0; q < qs; ++q)
        tc_wait(&qfull[q % C::RQ], (q / C::RQ) & 1, abort, a.status);
    }
    __syncwarp();
  } else if (warp == 1 || warp == kTcMma2) {
    // ---------------- MMA issuers: warp 1 matrix 0, warp kTcMma2 matrix 1 ----------------
    // A thread waits about 50 cycles after each tcgen05.mma it issues, so
    // gate and up are issued by two threads; descriptors and tensor-memory
    // addresses are precomputed so that each MMA costs a few integer adds.
    const int m = warp == 1 ? 0 : 1;
    if (lane == 0 && m < C::NMAT) {
      // the start-address field of a descriptor is the shared address / 16,
      // so the slots' descriptors are the first one plus a multiple
      const uint64_t bdesc0 = desc_sw128(smem_addr(sm + C::OFF_B));
      constexpr uint64_t kBdStep = (uint64_t)(C::PB * C::BPLANE) >> 4;
      const uint32_t aslot0 = tmem + C::TMEM_A + (uint32_t)(m * C::PA * 32);
      uint32_t os = 0;
      int st = 0;         // os % RO
      uint32_t ph = 0;    // (os / RO) & 1
      int j = 0;
      bool ok = true;
      // the MMAs of one operand stage for matrix m; FIRST: the item's first
      // stage (each accumulator's first MMA overwrites it)
      auto issue = [&](auto first, uint32_t dm, uint32_t ab, uint64_t bd, uint32_t idesc) {
        constexpr bool F = decltype(first)::value;
#pragma unroll
        for (int pass = 0; pass < C::PASSES; ++pass) {
          // passes: A hi x B hi (main), A hi x B mid, A lo x B hi (corrections)
          const int pa = pass == 2 ? 1 : 0, pb = pass == 1 ? 1 : 0;
          const uint32_t dd = dm + (pass > 0 ? (uint32_t)C::NMAX : 0u);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint32_t aa = ab + (uint32_t)(pa * 32 + ks * 8);
            const uint64_t bb = bd + (uint64_t)((pb * C::BPLANE + ks * 32) >> 4);
            if (F && ks == 0 && pass < 2) mma_tsk<false>(dd, aa, bb, idesc);
            else mma_tsk<true>(dd, aa, bb, idesc);
          }
        }
      };
      for (int item = i0; item < i1 && ok; ++item) {
        TcItem it;
        if (!tc_item<PRECISE, DOWN>(a, item, it)) continue;
        const int b = j & 1;
        if (j >= 2 && !tc_wait(&accempty[b], ((j >> 1) - 1) & 1, abort, a.status)) break;
        fence_after();
        const int npad = (it.ntok + 15) & ~15;
        const uint32_t idesc = idesc16(kTcM, npad, PRECISE);
        const uint32_t dm = tmem + (uint32_t)b * C::ACC_COLS + (uint32_t)(m * C::NACC * C::NMAX);
        for (int s = 0; s < it.nk; ++s) {
          if (!tc_wait(&opfull[st], ph, abort, a.status)) {
            ok = false;
            break;
          }
          if (m == 0) TCT(4, os);
          fence_after();
          const uint32_t ab = aslot0 + (uint32_t)st * C::A_COLS;
          const uint64_t bd = bdesc0 + (uint64_t)st * kBdStep;
          if (s == 0) issue(std::true_type{}, dm, ab, bd, idesc);
          else issue(std::false_type{}, dm, ab, bd, idesc);
          commit(&opempty[st]);
          if (m == 0) TCT(3, os);
          ++os;
          if (++st == C::RO) {
            st = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (PRECISE) {
          // bias step: A = the biases (one plane), B = group sums hi (into the
          // main sum) and mid (into the corrections)
          if (!tc_wait(&opfull[st], ph, abort, a.status)) break;
          fence_after();
          const uint32_t ab = aslot0 + (uint32_t)st * C::A_COLS;
          const uint64_t bd = bdesc0 + (uint64_t)st * kBdStep;
          const int ksteps = (it.nk + 15) >> 4;
#pragma unroll
          for (int pb = 0; pb < 2; ++pb)
            for (int ks = 0; ks < ksteps; ++ks)
              mma_tsk<true>(dm + (uint32_t)(pb * C::NMAX), ab + (uint32_t)(ks * 8),
                            bd + (uint64_t)((pb * C::BPLANE + ks * 32) >> 4), idesc);
          commit(&opempty[st]);
          ++os;
          if (++st == C::RO) {
            st = 0;
            ph ^= 1u;
          }
        }
        commit(&accfull[b]);
        ++j;
      }
    }
    __syncwarp();
  } else if (warp < 2 + kTcConv) {
    // ---------------- converters ----------------
    const int cw = warp - 2;                 // 0..kTcConv-1
    const int cg = cw >> 2;                  // (matrix, part of the row)
    const int row = (warp & 3) * 32 + lane;  // tensor-memory lane = weight row
    const int ct = cw * 32 + lane;           // 0..kTcConv*32-1
    const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
    const int m = cg / C::CU;                // matrix
    const int part = cg % C::CU;             // words [part*NW, part*NW + NW) of the group
    // activation unit: PRECISE row ct/16, floats 4*(ct%16)..+3 of the group;
    // FAST rows (ct + 512 j)/8, 16-byte chunk ct%8
    const int bc8 = ct & 7;
    const int bq = ct & 15;
    float* xs = reinterpret_cast<float*>(sm + C::OFF_X);
    constexpr int NR = C::NR;
    auto find = [&](int from, TcItem& it) -> int {
      for (int i = from; i < i1; ++i)
        if (tc_item<PRECISE, DOWN>(a, i, it)) return i;
      return i1;
    };
    // this thread's activation rows of an item (null past the chunk's pairs)
    auto rows_of = [&](const TcItem& it, const unsigned char* (&p)[NR]) {
#pragma unroll
      for (int j = 0; j < NR; ++j) {
        const int u = ct + kTcConv * 32 * j;
        const int n = PRECISE ? (u >> 4) : (u >> 3);
        p[j] = nullptr;
        if (n < it.ntok) {
          const int pos = it.pos0 + n;
          if (DOWN) {
            p[j] = PRECISE ? reinterpret_cast<const unsigned char*>(a.h + (size_t)pos * a.Imax)
                           : reinterpret_cast<const unsigned char*>(a.hb + (size_t)pos * a.Imax);
          } else {
            const size_t tr = (size_t)a.pair_tok[pos] * a.H;
            p[j] = PRECISE ? reinterpret_cast<const unsigned char*>(a.x + tr)
                           : reinterpret_cast<const unsigned char*>(a.xb + tr);
          }
        }
      }
    };
    // the activation values of K group g (loaded stages ahead of their use)
    auto load_b = [&](const unsigned char* const (&p)[NR], int g, uint4 (&v)[C::BVEC]) {
      if constexpr (PRECISE) {
#pragma unroll
        for (int j = 0; j < NR; ++j)
          v[j] = p[j] ? __ldg(reinterpret_cast<const uint4*>(p[j] + (size_t)g * 256 + bq * 16))
                      : make_uint4(0u, 0u, 0u, 0u);
      } else {
#pragma unroll
        for (int j = 0; j < NR; ++j)
          v[j] = p[j] ? __ldg(reinterpret_cast<const uint4*>(p[j] + (size_t)g * 128 + bc8 * 16))
                      : make_uint4(0u, 0u, 0u, 0u);
      }
    };
    // this row's scale (and bias) bf16 of groups 4kb..4kb+3
    auto load_sc = [&](const TcItem& it, int kb, uint2& s, uint2& bb) {
      s = make_uint2(0u, 0u);
      bb = make_uint2(0u, 0u);
      const int rows_k = DOWN ? a.dn.rows[it.kind] : a.gu.rows[it.kind];
      if (it.r0 + row >= rows_k) return;
      const uint64_t so = DOWN ? a.dn.s[it.kind] : (m ? a.gu.s2[it.kind] : a.gu.s[it.kind]);
      const uint64_t bo = DOWN ? a.dn.b[it.kind] : (m ? a.gu.b2[it.kind] : a.gu.b[it.kind]);
      const size_t off = ((size_t)(it.r0 + row) * it.nk + 4 * kb) * 2;
      s = __ldg(reinterpret_cast<const uint2*>(it.ptr + so + off));
      if (!PRECISE) bb = __ldg(reinterpret_cast<const uint2*>(it.ptr + bo + off));
    };

    TcItem cur, nxt;
    int icur = find(i0, cur);
    int inxt = icur < i1 ? find(icur + 1, nxt) : i1;
    const unsigned char* pc[NR];
    const unsigned char* pn[NR];
    uint4 P0[C::BVEC], P1[C::BVEC], P2[C::BVEC];
    uint2 sc = make_uint2(0u, 0u), bcv = make_uint2(0u, 0u), scn = sc, bcn = sc;
    if (icur < i1) {
      rows_of(cur, pc);
      load_b(pc, 0, P0);
      load_b(pc, 1, P1);
      load_sc(cur, 0, scn, bcn);
    }
    if (inxt < i1) rows_of(nxt, pn);
    uint32_t qs = 0, os = 0;
    int g = 0;
    bool ok = true;
    while (icur < i1 && ok) {
      const int G = cur.nk;
      // loads for two groups ahead (possibly in the next item)
      if (g + 2 < G) load_b(pc, g + 2, P2);
      else if (inxt < i1) load_b(pn, g + 2 - G, P2);
      if ((g & 3) == 0) {
        sc = scn;
        bcv = bcn;
        if (g + 4 < G) load_sc(cur, (g >> 2) + 1, scn, bcn);
        else if (inxt < i1) load_sc(nxt, 0, scn, bcn);
      }
      const int qst = (int)(qs % C::RQ), ost = (int)(os % C::RO);
      if (os >= (uint32_t)C::RO && !warp_wait(&opempty[ost], ((os / C::RO) - 1) & 1, abort, a.status)) {
        ok = false;
        break;
      }
      if (warp == 2 && lane == 0) TCT(7, os);
      if ((g & 3) == 0 && !warp_wait(&qfull[qst], (qs / C::RQ) & 1, abort, a.status)) {
        ok = false;
        break;
      }
      if (warp == 2 && lane == 0 && (g & 3) == 0) TCT(1, qs);
      fence_after();  // the MMAs that read this operand slot have completed
      const unsigned char* q = sm + C::OFF_Q + (size_t)qst * C::QSTAGE;
      const uint32_t s16 = ((g & 2) ? sc.y : sc.x) >> ((g & 1) * 16) & 0xFFFFu;
      const uint32_t abase = tmem + lane_addr + C::TMEM_A + (uint32_t)ost * C::A_COLS +
                             (uint32_t)(m * C::PA * 32);
      // ---- A: NW words of this thread's row of the group ----
      constexpr int NW = C::NW;
      uint32_t wv[NW];
      {
        // the stage is 128-byte swizzled by the TMA copy: 16-byte chunk c of
        // row r sits at chunk c ^ (r & 7), so a warp's 32 rows spread over
        // all banks
        const unsigned char* qrow = q + (size_t)m * C::QMAT + row * 128;
        const int sw = row & 7;
        const int c0 = 2 * (g & 3);  // the group's first chunk
        if constexpr (NW == 8) {
          const uint4 v0 = *reinterpret_cast<const uint4*>(qrow + ((c0 ^ sw) << 4));
          const uint4 v1 = *reinterpret_cast<const uint4*>(qrow + (((c0 + 1) ^ sw) << 4));
          wv[0] = v0.x; wv[1] = v0.y; wv[2] = v0.z; wv[3] = v0.w;
          wv[4 % NW] = v1.x; wv[5 % NW] = v1.y; wv[6 % NW] = v1.z; wv[7 % NW] = v1.w;
        } else if constexpr (NW == 4) {
          const uint4 v0 = *reinterpret_cast<const uint4*>(qrow + (((c0 + part) ^ sw) << 4));
          wv[0] = v0.x; wv[1] = v0.y; wv[2] = v0.z; wv[3] = v0.w;
        } else {
          static_assert(NW == 2, "converter split");
          const uint2 v0 = *reinterpret_cast<const uint2*>(
              qrow + (((c0 + (part >> 1)) ^ sw) << 4) + (part & 1) * 8);
          wv[0] = v0.x; wv[1] = v0.y;
        }
      }
      const uint32_t acol = (uint32_t)(part * NW * 4);
      if constexpr (PRECISE) {
        const uint32_t s2 = s16 | (s16 << 16);
        uint32_t hi[NW * 4], lo[NW * 4];
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          const uint32_t l = wv[w] & 0x0F0F0F0Fu, h = (wv[w] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const uint32_t qv = bf2_sub(nib_pair(l, h, p) | 0x43004300u, 0x43004300u);  // exact q
            const uint32_t hv = bf2_fma(qv, s2, 0x80008000u);                        // bf16(s q)
            hi[4 * w + p] = hv;
            lo[4 * w + p] = bf2_fma(qv, s2, hv ^ 0x80008000u);                       // s q - hi, exact
          }
        }
        tst<NW * 4>(abase + acol, hi);
        tst<NW * 4>(abase + 32u + acol, lo);
      } else {
        const uint32_t b16 = ((g & 2) ? bcv.y : bcv.x) >> ((g & 1) * 16) & 0xFFFFu;
        const __half sh = __float2half_rn(__uint_as_float(s16 << 16));
        const __half bh = __float2half_rn(__uint_as_float(b16 << 16));
        const __half2 s2 = __halves2half2(sh, sh), b2 = __halves2half2(bh, bh);
        const __half2 k1024 = u2h(0x64006400u);
        uint32_t av[NW * 4];
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          const uint32_t l = wv[w] & 0x0F0F0F0Fu, h = (wv[w] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const __half2 qv = __hsub2(u2h(nib_pair(l, h, p) | 0x64006400u), k1024);
            av[4 * w + p] = h2u(__hfma2(qv, s2, b2));
          }
        }
        tst<NW * 4>(abase + acol, av);
      }
      // ---- B: this thread's activation values -> swizzled planes ----
      unsigned char* bo = sm + C::OFF_B + (size_t)ost * C::PB * C::BPLANE;
      if constexpr (PRECISE) {
#pragma unroll
        for (int j = 0; j < NR; ++j) {
          const int n = (ct + kTcConv * 32 * j) >> 4;
          const float v[4] = {__uint_as_float(P0[j].x), __uint_as_float(P0[j].y), __uint_as_float(P0[j].z),
                              __uint_as_float(P0[j].w)};
          const uint32_t h0 = pack_bf2(v[0], v[1]), h1 = pack_bf2(v[2], v[3]);
          const uint32_t m0 = pack_bf2(v[0] - bf_lo(h0), v[1] - bf_hi(h0));
          const uint32_t m1 = pack_bf2(v[2] - bf_lo(h1), v[3] - bf_hi(h1));
          float sum = (v[0] + v[1]) + (v[2] + v[3]);
          const size_t off = (size_t)n * 128 + (size_t)(((bq >> 1) ^ (n & 7)) << 4) + (bq & 1) * 8;
          *reinterpret_cast<uint2*>(bo + off) = make_uint2(h0, h1);
          *reinterpret_cast<uint2*>(bo + C::BPLANE + off) = make_uint2(m0, m1);
          sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
          sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
          sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 4);
          sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 8);
          if (bq == 0) xs[n * 32 + g] = sum;
        }
      } else {
#pragma unroll
        for (int j = 0; j < NR; ++j) {
          const int u = ct + kTcConv * 32 * j;
          if (u < C::NMAX * 8) {
            const int n = u >> 3;
            *reinterpret_cast<uint4*>(bo + (size_t)n * 128 + (size_t)((bc8 ^ (n & 7)) << 4)) = P0[j];
          }
        }
      }
      wait_st();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&opfull[ost]);
        if ((g & 3) == 3) mbar_arrive(&qempty[qst]);
        if (warp == 2) TCT(2, os);
      }
      if ((g & 3) == 3) ++qs;
      ++os;
#pragma unroll
      for (int v = 0; v < C::BVEC; ++v) {
        P0[v] = P1[v];
        P1[v] = P2[v];
      }
      if (++g < G) continue;
      if constexpr (PRECISE) {
        // ---- bias step: A = this row's biases, B = group sums (hi, mid) ----
        const int bst = (int)(os % C::RO);
        if (os >= (uint32_t)C::RO && !warp_wait(&opempty[bst], ((os / C::RO) - 1) & 1, abort, a.status)) {
          ok = false;
          break;
        }
        fence_after();
        const uint32_t bbase = tmem + lane_addr + C::TMEM_A + (uint32_t)bst * C::A_COLS +
                               (uint32_t)(m * C::PA * 32);
        const int rows_k = DOWN ? a.dn.rows[cur.kind] : a.gu.rows[cur.kind];
        const bool live = cur.r0 + row < rows_k;
        const uint64_t bof = DOWN ? a.dn.b[cur.kind] : (m ? a.gu.b2[cur.kind] : a.gu.b[cur.kind]);
        const uint16_t* brow = reinterpret_cast<const uint16_t*>(cur.ptr + bof) + (size_t)(cur.r0 + row) * G;
        // the row's biases as bf16 pairs in the columns of K < 32 (groups
        // beyond G are zero; the bias step reads K < 16 ceil(G / 16) <= 32):
        // one thread per row writes all 16 columns, with more threads per
        // row parts 0 and 1 write 8 each
        if constexpr (C::CU == 1) {
          uint32_t bv[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int g0 = 2 * e;
            const uint32_t b0 = live && g0 < G ? brow[g0] : 0u;
            const uint32_t b1 = live && g0 + 1 < G ? brow[g0 + 1] : 0u;
            bv[e] = b0 | (b1 << 16);
          }
          st16(bbase, bv);
        } else {
          uint32_t bv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int g0 = 16 * part + 2 * e;
            const uint32_t b0 = live && g0 < G ? brow[g0] : 0u;
            const uint32_t b1 = live && g0 + 1 < G ? brow[g0 + 1] : 0u;
            bv[e] = b0 | (b1 << 16);
          }
          if (part < 2) st8(bbase + (uint32_t)(8 * part), bv);
        }
        unsigned char* bo = sm + C::OFF_B + (size_t)bst * C::PB * C::BPLANE;
#pragma unroll
        for (int j = 0; j < NR; ++j) {
          const int n = (ct + kTcConv * 32 * j) >> 4;
          const int g0 = 4 * bq;
          float xv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) xv[e] = (n < cur.ntok && g0 + e < G) ? xs[n * 32 + g0 + e] : 0.0f;
          const uint32_t h0 = pack_bf2(xv[0], xv[1]), h1 = pack_bf2(xv[2], xv[3]);
          const uint32_t m0 = pack_bf2(xv[0] - bf_lo(h0), xv[1] - bf_hi(h0));
          const uint32_t m1 = pack_bf2(xv[2] - bf_lo(h1), xv[3] - bf_hi(h1));
          const size_t off = (size_t)n * 128 + (size_t)(((bq >> 1) ^ (n & 7)) << 4) + (bq & 1) * 8;
          *reinterpret_cast<uint2*>(bo + off) = make_uint2(h0, h1);
          *reinterpret_cast<uint2*>(bo + C::BPLANE + off) = make_uint2(m0, m1);
        }
        wait_st();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        fence_before();
        // (a warp's group sums are its own rows: the next item's writes come
        // after this read in the same warp)
        __syncwarp();
        if (lane == 0) mbar_arrive(&opfull[bst]);
        ++os;
      }
      // next item: its first two groups are already loaded
      cur = nxt;
      icur = inxt;
#pragma unroll
      for (int j = 0; j < NR; ++j) pc[j] = pn[j];
      g = 0;
      if (icur < i1) {
        inxt = find(icur + 1, nxt);
        if (inxt < i1) rows_of(nxt, pn);
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
    int j = 0;
    bool over = false;
    for (int item = i0; item < i1; ++item) {
      TcItem it;
      if (!tc_item<PRECISE, DOWN>(a, item, it)) continue;
      const int b = j & 1;
      if (!warp_wait(&accfull[b], (j >> 1) & 1, abort, a.status)) break;
      if (warp == kTcMma2 - 1 && lane == 0) TCT(5, j);
      fence_after();
      const uint32_t acc = tmem + lane_addr + (uint32_t)b * C::ACC_COLS;
      const int npad = (it.ntok + 15) & ~15;
      const bool live = row < it.nrows;
      for (int c0 = 0; c0 < npad; c0 += 16) {
        uint32_t g[16], u[16];
        ld16(acc + (uint32_t)c0, g);
        if (!DOWN) ld16(acc + (uint32_t)(C::NACC * C::NMAX + c0), u);
        if constexpr (PRECISE) {
          uint32_t gc[16], uc[16];
          ld16(acc + (uint32_t)(C::NMAX + c0), gc);
          if (!DOWN) ld16(acc + (uint32_t)(3 * C::NMAX + c0), uc);
          wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            g[e] = __float_as_uint(__uint_as_float(g[e]) + __uint_as_float(gc[e]));
            if (!DOWN) u[e] = __float_as_uint(__uint_as_float(u[e]) + __uint_as_float(uc[e]));
          }
        }
        wait_ld();
        if (live) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int n = c0 + e;
            if (n < it.ntok) {
              // SiLU(g) u with the fast exponential and an IEEE reciprocal
              // (relative error about 1e-6, inside both tolerances)
              const float gv = __uint_as_float(g[e]);
              const float v = DOWN ? gv
                                   : gv * __frcp_rn(1.0f + __expf(-gv)) * __uint_as_float(u[e]);
              const int pos = it.pos0 + n;
              if (PRECISE) {
                if (DOWN) {
                  const size_t orow = (size_t)a.pair_tok[pos] * a.kp1 + a.pair_pick[pos];
                  a.partial[orow * a.H + it.r0 + row] = v;
                } else {
                  a.h[(size_t)pos * a.Imax + it.r0 + row] = v;
                }
              } else {
                over |= !(fabsf(v) < 65504.0f);
                const uint16_t hv = __half_as_ushort(__float2half_rn(v));
                if (DOWN) a.pb[(size_t)pos * a.H + it.r0 + row] = hv;
                else a.hb[(size_t)pos * a.Imax + it.r0 + row] = hv;
              }
            }
          }
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[b]);
      if (warp == kTcMma2 - 1 && lane == 0) TCT(6, j);
      ++j;
    }
    if (over) atomicOr(a.status, kStatusF16Range);
  }
  fence_before();
  __syncthreads();
  fence_after();
  pdl_trigger();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_ALLOC));
}

template <typename Kern>
cudaError_t launch_tc(Kern kernel, int grid, size_t smem, cudaStream_t s, const TcArgs& a,
                      const TcMaps& maps) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, a, maps);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

}  // namespace

static_assert(sizeof(CUtensorMap) == 128, "tensor map size");

#ifdef OSM_TC_TRACE
extern "C" int osm_dbg_tc_trace(unsigned long long* out) {
  return (int)cudaMemcpyFromSymbol(out, g_tct, sizeof(g_tct));
}
#endif

bool tc_encode_maps(unsigned char (*dst)[128], const uint8_t* base, const uint64_t off[3],
                    const int rows[3], const int words[3], int slots, uint64_t slot_stride) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || !base) return false;
  for (int s = 0; s < 3; ++s) {
    if ((reinterpret_cast<uintptr_t>(base) + off[s]) % 16 || rows[s] < kTcM || words[s] % 32 ||
        (words[s] * 4) % 16 || (slots > 1 && slot_stride % 16))
      return false;
    cuuint64_t dims[3] = {(cuuint64_t)words[s], (cuuint64_t)rows[s], (cuuint64_t)slots};
    cuuint64_t strides[2] = {(cuuint64_t)words[s] * 4, (cuuint64_t)(slots > 1 ? slot_stride : (uint64_t)words[s] * 4 * rows[s])};
    cuuint32_t box[3] = {32, (cuuint32_t)kTcM, 1};
    cuuint32_t es[3] = {1, 1, 1};
    const CUresult r = fn(reinterpret_cast<CUtensorMap*>(dst[s]), CU_TENSOR_MAP_DATA_TYPE_UINT32, 3,
                          const_cast<uint8_t*>(base) + off[s], dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
  }
  return true;
}

bool tc_encode_u8_rows(unsigned char* dst, const uint8_t* base, uint64_t rows, uint64_t row_bytes,
                       int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || !base || reinterpret_cast<uintptr_t>(base) % 16 || row_bytes % 128 || rows == 0 ||
      box_rows < 1 || box_rows > 256)
    return false;
  cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(reinterpret_cast<CUtensorMap*>(dst), CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base),
            dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

void init_tc_attributes(int max_smem) {
  cudaFuncSetAttribute(tc_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(tc_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(tc_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(tc_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
}

size_t tc_smem(bool precise, bool down) {
  if (precise) return down ? TcCfg<true, true>::BYTES : TcCfg<true, false>::BYTES;
  return down ? TcCfg<false, true>::BYTES : TcCfg<false, false>::BYTES;
}

bool tc_configure(TcArgs& a, int has_shared, int max_smem) {
  const int nk = has_shared ? 2 : 1;
  if (a.H % 64 || a.H > 2048 || a.Imax % 64 || a.Imax > 2048) return false;
  for (int kd = 0; kd < nk; ++kd) {
    if (a.gu.K[kd] != a.H || a.dn.rows[kd] != a.H || a.dn.K[kd] % 64 || a.dn.K[kd] > a.Imax)
      return false;
    if (a.gu.rows[kd] < kTcM || a.dn.rows[kd] < kTcM) return false;
    // scale/bias rows are read 8 bytes (four groups) at a time
    const uint64_t o[6] = {a.gu.s[kd], a.gu.b[kd], a.gu.s2[kd], a.gu.b2[kd], a.dn.s[kd], a.dn.b[kd]};
    for (uint64_t v : o)
      if (v % 8) return false;
    if ((a.H >> 6) % 4 || (a.dn.K[kd] >> 6) % 4) return false;
  }
  if (a.slab_stride % 16) return false;
  const int rmax = a.gu.rows[0] > a.gu.rows[1] ? a.gu.rows[0] : a.gu.rows[1];
  a.nmt_gu = (rmax + kTcM - 1) / kTcM;
  a.nmt_dn = (a.H + kTcM - 1) / kTcM;
  for (int p = 0; p < 2; ++p)
    for (int d = 0; d < 2; ++d)
      if (tc_smem(p != 0, d != 0) > (size_t)max_smem) return false;
  return encode_fn() != nullptr;
}

cudaError_t launch_tc_gateup(const TcArgs& a, const TcMaps& maps, bool precise, int grid,
                             cudaStream_t s, uint64_t* launches) {
  if (launches) *launches += 1;
  return precise ? launch_tc(tc_kernel<true, false>, grid, tc_smem(true, false), s, a, maps)
                 : launch_tc(tc_kernel<false, false>, grid, tc_smem(false, false), s, a, maps);
}

cudaError_t launch_tc_down(const TcArgs& a, const TcMaps& maps, bool precise, int grid,
                           cudaStream_t s, uint64_t* launches) {
  if (launches) *launches += 1;
  return precise ? launch_tc(tc_kernel<true, true>, grid, tc_smem(true, true), s, a, maps)
                 : launch_tc(tc_kernel<false, true>, grid, tc_smem(false, true), s, a, maps);
}

}  // namespace osm
