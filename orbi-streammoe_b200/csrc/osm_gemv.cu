// osm_gemv.cu -- the latency path of the expert MLPs for 1-2 tokens per call
// (replaces, for decode, the per-expert q4_gemv / swiglu / weighted_accumulate
// submits of src/model/routed_moe.cpp:320-404).
//
// Data movement: every CTA requests all of its weight rows at once with
// 16-byte cp.async copies into padded shared-memory tiles (one commit group
// per 16-row tile), so the whole working set is in flight together; the down
// kernel is launched while gate/up still runs and fetches its rows then.
//
// Arithmetic: integer tensor-core MMAs (mma.sync m16n8k32 s8 -> s32).
//  * A = 16 weight rows x 32 inputs: the nibbles q (0..15) are exact int8;
//    one 32-bit word of a row (8 nibbles) yields two int8x4 registers with
//    two LOPs (low nibbles, high nibbles).  The input order inside a 32-wide
//    slab is permuted; the activation fragments use the same permutation.
//  * B = activations as block floating point: per token and 64-wide group,
//    x = s (d0 + d1 2^-7 + d2 2^-14) with s a power of two and int8 digits
//    (|d| <= 64), exact up to s 2^-15 <= 2^-20 max|x_group|.  Columns 4t..4t+2
//    of the n=8 tile hold token t's three digit vectors, so one MMA serves
//    both digits and both tokens; the s32 sums are exact.
//  * per group: y += s_w s (D0 + D1/128 + D2/16384) + b_w sum(x) (the affine
//    dequantisation of shaders/q4_gemv.comp:44-60 applied per group), in fp32.
// dec_gateup_kernel  one CTA per SM over an even split of the (gate row, up
//                    row) pairs of all active experts, shared expert first
//                    (its rows are fetched before the routing exists); the
//                    8 warps split each tile's groups and their partial sums
//                    are added in a fixed order, then SwiGLU.
// dec_down_kernel    one CTA per block of <= 16 output rows, every active
//                    expert; warps take experts; then the CTA combines each
//                    token's picks in pick order, the shared expert last,
//                    then the residual (routed_moe.cpp:13-92, :396-404).
#include <cuda_runtime.h>
#include <stdint.h>

#include "osm_common.cuh"
#include "osm_kernels.cuh"

namespace osm {
namespace {
#ifdef OSM_PHASE_TIMING
__device__ unsigned long long g_tl[OSM_TL_SLOTS];
__device__ long long g_cyc[64];
__device__ long long g_gcyc[2][64];  // grouped kernels: [gate/up | down][stamp]
#define GCYC(k, i) do { if (blockIdx.x == 0 && threadIdx.x == 0 && (i) < 64) g_gcyc[(k)][(i)] = clock64(); } while (0)
#define CYC(i) do { if (threadIdx.x == 0 && (blockIdx.x == 0 || blockIdx.x == 70)) \
  g_cyc[(i) + (blockIdx.x == 70 ? 32 : 0)] = clock64(); } while (0)
#else
#define CYC(i) do { } while (0)
#define GCYC(k, i) do { } while (0)
#endif

constexpr int kTileRows = 16;
constexpr int kDnChunks = 4;  // most group chunks one down entry is split into

// ---- asynchronous 4/8/16-byte copies global -> shared ----
__device__ __forceinline__ void cp_async(void* dst, const void* src, int bytes) {
  if (bytes == 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
  else if (bytes == 8)
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                       uint32_t a3, uint32_t b0, uint32_t b1) {
  // not volatile: a pure function of its registers, free to interleave
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Padded row stride (bytes) for rows of rb bytes: a multiple of 16 that is 32
// mod 128, so the 8 rows a warp reads at one offset fall in distinct banks.
__host__ __device__ inline int pad_stride(int rb) { return rb + ((32 - rb % 128) + 128) % 128; }
__host__ __device__ inline size_t align16(size_t v) { return (v + 15) & ~(size_t)15; }
// Scale-row stride (bytes) for rows of rb bytes: a multiple of 16 with an odd
// quotient, so rows r = 0..7 read at one offset fall in distinct banks.
__host__ __device__ inline int scale_stride(int rb) {
  int s = (rb + 15) & ~15;
  if (((s >> 4) & 1) == 0) s += 16;
  return s;
}

// MMA rows and tile rows.  Weight rows reach shared memory in blocks of 4
// consecutive rows (one bulk copy each); the 16 rows of a tile are 4 blocks
// at a padded stride.  MMA row R reads tile row m = 4 (R & 3) + (R >> 2), so
// the 4 rows one 16-lane phase reads (R = 0..3 or 4..7, +8) sit in 4
// different blocks, hence different banks.
__host__ __device__ inline int mma_to_row(int R) { return 4 * (R & 3) + (R >> 2); }
__host__ __device__ inline int row_to_mma(int m) { return 4 * (m & 3) + (m >> 2); }

// Active entry j: from the grouping step, or in direct mode (one or two
// tokens, no grouping step) pick j % k of token j / k (j == B k: the shared
// expert, for all B tokens; pad0 holds a routed entry's token).  CG: read through L2 only (the routing
// may be read before this grid's dependency wait; see dec_down_kernel).
template <bool CG>
__device__ __forceinline__ ActEntry gemv_entry(const GemvArgs& a, int j) {
  ActEntry en;
  if (!a.direct) {
    if (!CG) return a.act[j];
    const ActEntry* p = a.act + j;
    en.ptr = reinterpret_cast<const uint8_t*>(
        __ldcg(reinterpret_cast<const unsigned long long*>(&p->ptr)));
    en.off = __ldcg(&p->off);
    en.cnt = __ldcg(&p->cnt);
    en.kind = __ldcg(&p->kind);
    en.tg0 = 0;
    en.pad0 = en.pad1 = 0;
    return en;
  }
  en.off = j;
  en.cnt = 1;
  en.tg0 = 0;
  en.pad0 = en.pad1 = 0;
  if (j < a.B * a.k) {
    en.kind = 0;
    en.pad0 = j / a.k;  // the entry's token
    if (a.pick_ptr != nullptr) {
      // the router wrote the slot base of each pick (null: bad or not resident)
      en.ptr = CG ? reinterpret_cast<const uint8_t*>(__ldcg(
                        reinterpret_cast<const unsigned long long*>(a.pick_ptr + j)))
                  : a.pick_ptr[j];
    } else {
      // the same resolution as the router's: slot of the picked expert
      en.ptr = nullptr;
      const float m = CG ? __ldcg(a.mass + j / a.k) : a.mass[j / a.k];
      if (m > 0.0f) {
        const uint32_t id = CG ? __ldcg(a.ids + j) : a.ids[j];
        if (id >= (uint32_t)a.E) {
          atomicOr(a.status, kStatusBadSlot);
        } else {
          const int slot = CG ? __ldcg(a.slot_of + id) : a.slot_of[id];
          if (slot < 0) atomicOr(a.status, kStatusNotResident);
          else en.ptr = a.slab + (size_t)slot * a.slab_stride;
        }
      }
    }
  } else {
    en.kind = 1;
    en.ptr = a.shared_ptr;
    en.cnt = a.B;
  }
  return en;
}

template <bool CG>
__device__ __forceinline__ int gemv_entries(const GemvArgs& a) {
  if (a.direct) return a.B * a.k + a.has_shared;
  return CG ? __ldcg(a.n_active) : *a.n_active;
}

// What a pair / entry holds.
struct DecMeta {
  const uint8_t* ptr;  // slot base (null: nothing to compute)
  int off, cnt, row, kind;
  int tok;             // direct mode: a routed entry's token
};

// ---- shared-memory plans (host and device agree on them) ----
struct GuLayout {
  size_t tiles, scales, xfrag, xsx, xsum, part, meta, bars, total;
  int bs;  // padded stride of a 4-row block
  int ss;  // padded scale-row stride
};
__host__ __device__ inline GuLayout gu_layout(int H, int ntile, int per_cta) {
  const size_t G = (size_t)H >> 6;
  GuLayout L;
  L.bs = pad_stride(4 * (H >> 1));
  L.ss = scale_stride((int)G * 2);
  size_t o = 0;
  L.tiles = o;  o += (size_t)ntile * 2 * 4 * L.bs;               // [tile][gate|up][block]
  L.scales = o; o += (size_t)ntile * 4 * kTileRows * L.ss;       // [tile][array][mma row]
  L.xfrag = o;  o += G * 2 * 32 * 8;                             // [g][half][lane] uint2
  L.xsx = o;    o += G * 2 * 2 * 4;                              // [token][g][even|odd]
  L.xsum = o;   o += align16(G * 2 * 4);                         // [token][g]
  L.part = o;   o += (size_t)kDecWarps * kTileRows * 2 * 2 * 4;  // [tile][chunk]: <= kDecWarps items
  L.meta = o;   o += (size_t)per_cta * sizeof(DecMeta);
  L.bars = o;   o += (size_t)ntile * 8;
  L.total = o;
  return L;
}
struct DnLayout {
  size_t wt, scales, hfrag, hsx, hsum, ys, rw, meta, bars, total;
  int bs;  // padded stride of a 4-row block
};
__host__ __device__ inline DnLayout dn_layout(int ne, int Kmax, int Imax, int P) {
  const size_t Gd = (size_t)Kmax >> 6, Gh = (size_t)Imax >> 6;
  DnLayout L;
  L.bs = pad_stride(4 * (Kmax >> 1));
  size_t o = 0;
  L.wt = o;     o += (size_t)ne * 4 * L.bs;                      // [entry][block]
  L.scales = o; o += align16((size_t)ne * 2 * kTileRows * Gd * 2);  // [entry][s|b][mma row][Gd]
  L.hfrag = o;  o += (size_t)P * Gh * 2 * 16 * 8;                // [pair][g][half][16 lanes]
  L.hsx = o;    o += (size_t)P * Gh * 2 * 4;
  L.hsum = o;   o += align16((size_t)P * Gh * 4);
  L.ys = o;     o += align16((size_t)kDnChunks * P * kTileRows * 4);  // [chunk][pair][row]
  L.rw = o;     o += align16((size_t)P * 4 + (size_t)P * 4);     // pick weights, pair of (token, pick)
  L.meta = o;   o += (size_t)ne * sizeof(DecMeta);
  L.bars = o;   o += (size_t)ne * 8;
  L.total = o;
  return L;
}

// Pair p of the CTA split: the shared expert's rows first, then the routed
// entries' rows.  Returns the entry index, or -1 (past the last entry, or a
// routed pair when shared_only).
__device__ __forceinline__ int pair_entry(const GemvArgs& a, int p, bool shared_only, int n_ent,
                                          int& row) {
  const int rs = a.has_shared ? a.gu.rows[1] : 0;
  if (p < rs) {
    row = p;
    return a.direct ? a.B * a.k : 0;
  }
  if (shared_only) return -1;
  const int q = (p - rs) / a.gu.rows[0];
  row = (p - rs) - q * a.gu.rows[0];
  const int j = a.direct ? q : a.has_shared + q;
  return (a.direct ? q < a.B * a.k : j < n_ent) ? j : -1;
}

// int8 A fragment halves of one 32-bit word of 8 nibbles
__device__ __forceinline__ uint32_t lo_nib(uint32_t w) { return w & 0x0F0F0F0Fu; }
__device__ __forceinline__ uint32_t hi_nib(uint32_t w) { return (w >> 4) & 0x0F0F0F0Fu; }

// Stages activation digits of `nrow` rows of `src` (row stride ld, K inputs)
// as B fragments -- cols16: frag[row][g][half][16 lanes] (columns 0..3);
// else frag[g][half][32 lanes] with row t in columns 4t..4t+3 (nrow <= 2) --
// digit scales sx[row][g][2] (even lanes s/128, odd lanes s/16384) and
// sums[row][g].  Row t reads src row rowmap[t] when rowmap is given.  Items
// (row, g, half, j) of one (row, g) are 8 consecutive threads.
__device__ void stage_digits(const float* __restrict__ src, int nrow, int ld, int K, bool cols16,
                             uint2* frag, float* sx, float* sums, const int* rowmap = nullptr) {
  const int G = K >> 6;
  const int items = nrow * G * 8;
  constexpr int U = 2;  // items per thread whose loads are in flight together
  for (int base = 0; base < items; base += U * blockDim.x) {
    float v[U][8];
    int itc[U];
    bool live[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int it = base + u * blockDim.x + threadIdx.x;
      live[u] = it < items;
      itc[u] = live[u] ? it : items - 1;
      const int j = itc[u] & 3, h = (itc[u] >> 2) & 1, g = (itc[u] >> 3) % G, t = (itc[u] >> 3) / G;
      const float* p = src + (size_t)(rowmap ? rowmap[t] : t) * ld + 64 * g + 16 * j + 8 * h;
      const float4 u0 = *reinterpret_cast<const float4*>(p);
      const float4 u1 = *reinterpret_cast<const float4*>(p + 4);
      v[u][0] = u0.x; v[u][1] = u0.y; v[u][2] = u0.z; v[u][3] = u0.w;
      v[u][4] = u1.x; v[u][5] = u1.y; v[u][6] = u1.z; v[u][7] = u1.w;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = itc[u] & 3, h = (itc[u] >> 2) & 1, g = (itc[u] >> 3) % G, t = (itc[u] >> 3) / G;
      float m = 0.0f, sm = 0.0f;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        m = fmaxf(m, fabsf(v[u][q]));
        sm += v[u][q];
      }
      // the 8 items of (t, g) are lanes 8c..8c+7 of this warp
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
        sm += __shfl_xor_sync(0xFFFFFFFFu, sm, o);
      }
      if (!live[u]) continue;
      const int e = group_exponent(m);
      const Digits D = make_digits(v[u], e);
      // lane n*4 + j holds column n: digit d of row t is column d (cols16:
      // one fragment per row) or column 4t + d (two rows share a fragment)
      uint2* fr = cols16 ? frag + (((size_t)t * G + g) * 2 + h) * 16
                         : frag + ((size_t)g * 2 + h) * 32 + 16 * t;
#pragma unroll
      for (int d = 0; d < 3; ++d) fr[d * 4 + j] = make_uint2(D.b0[d], D.b1[d]);
      fr[3 * 4 + j] = make_uint2(0u, 0u);
      if (h == 0 && j == 0) {
        const float s = __uint_as_float((uint32_t)(127 + e) << 23);
        sx[((size_t)t * G + g) * 2 + 0] = s * 0.0078125f;
        sx[((size_t)t * G + g) * 2 + 1] = s * 6.103515625e-05f;
        sums[(size_t)t * G + g] = sm;
      }
    }
  }
}

// ----------------------------------------------------------------------------
// gate/up + SwiGLU
// ----------------------------------------------------------------------------
__global__ void __launch_bounds__(kDecWarps * 32, 2) dec_gateup_kernel(GemvArgs a) {
  extern __shared__ __align__(128) unsigned char smraw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = a.H, G = H >> 6, rowb = H >> 1;
  const int c0 = blockIdx.x * a.per_cta;                 // a multiple of 4
  const int np = min(c0 + a.per_cta, a.total_max) - c0;  // pairs of this CTA
  const int ntile = (np + kTileRows - 1) / kTileRows;
  const GuLayout Ly = gu_layout(H, a.nbuf, a.per_cta);
  unsigned char* tiles = smraw + Ly.tiles;
  unsigned char* scales = smraw + Ly.scales;
  uint2* xfrag = reinterpret_cast<uint2*>(smraw + Ly.xfrag);
  float* xsx = reinterpret_cast<float*>(smraw + Ly.xsx);
  float* xsum = reinterpret_cast<float*>(smraw + Ly.xsum);
  float* part = reinterpret_cast<float*>(smraw + Ly.part);
  DecMeta* meta = reinterpret_cast<DecMeta*>(smraw + Ly.meta);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smraw + Ly.bars);
  const int bs = Ly.bs, sst = Ly.ss;
  TL_START(0);
  CYC(0);
  if (tid < a.nbuf) {
    mbar_init(&bars[tid], 1);
    mbar_init_fence();
  }
  // Copies of the pairs of one pass (the shared expert before the routing
  // exists, the routed experts after): weights by bulk copies of 4-row blocks
  // (single rows where a block is not one run of one expert) counted on the
  // tile's mbarrier; scale rows by 4-16 byte cp.async into MMA-row order.
  auto issue = [&](bool shared_pass) {
    auto mine = [&](const DecMeta& m) { return m.ptr != nullptr && (m.kind == 1) == shared_pass; };
    for (int bb = tid; bb < (np + 3) >> 2; bb += blockDim.x) {
      const int p0 = bb * 4, tl = p0 / kTileRows, b = (p0 % kTileRows) >> 2;
      const DecMeta m0 = meta[p0];
      bool run = p0 + 3 < np && mine(m0);
      for (int i = 1; i < 4 && run; ++i) {
        const DecMeta& m = meta[p0 + i];
        run = mine(m) && m.ptr == m0.ptr && m.kind == m0.kind && m.row == m0.row + i;
      }
      uint64_t* bar = &bars[tl];
      unsigned char* dg = tiles + (size_t)((tl * 2 + 0) * 4 + b) * bs;
      unsigned char* du = tiles + (size_t)((tl * 2 + 1) * 4 + b) * bs;
      if (run) {
        mbar_expect_tx(bar, 8u * rowb);
        const size_t off = (size_t)m0.row * rowb;
        bulk_load(dg, m0.ptr + a.gu.w[m0.kind] + off, 4u * rowb, bar);
        bulk_load(du, m0.ptr + a.gu.w2[m0.kind] + off, 4u * rowb, bar);
      } else {
        for (int i = 0; i < 4 && p0 + i < np; ++i) {
          const DecMeta& m = meta[p0 + i];
          if (!mine(m)) continue;
          mbar_expect_tx(bar, 2u * rowb);
          const size_t off = (size_t)m.row * rowb;
          bulk_load(dg + (size_t)i * rowb, m.ptr + a.gu.w[m.kind] + off, rowb, bar);
          bulk_load(du + (size_t)i * rowb, m.ptr + a.gu.w2[m.kind] + off, rowb, bar);
        }
      }
    }
    CYC(shared_pass ? 11 : 9);
    const int scb = a.cs_gu, spr = (G * 2) / scb;
    for (int q = tid; q < np * 4 * spr; q += blockDim.x) {
      const int p = q / (4 * spr), rem = q - p * 4 * spr, arr = rem / spr, c = rem - arr * spr;
      const DecMeta& m = meta[p];
      if (!mine(m)) continue;
      const int tl = p / kTileRows, R = row_to_mma(p % kTileRows);
      const uint64_t off = arr == 0 ? a.gu.s[m.kind] : arr == 1 ? a.gu.b[m.kind]
                         : arr == 2 ? a.gu.s2[m.kind] : a.gu.b2[m.kind];
      cp_async(scales + (size_t)((tl * 4 + arr) * kTileRows + R) * sst + c * scb,
               m.ptr + off + (size_t)m.row * G * 2 + c * scb, scb);
    }
    CYC(shared_pass ? 12 : 10);
    cp_commit();
  };
  // ---- the shared expert's rows do not depend on the routing ----
  for (int p = tid; p < np; p += blockDim.x) {
    int row = 0;
    DecMeta m;
    m.ptr = nullptr;
    m.kind = 0;
    m.off = m.cnt = 0;
    m.tok = 0;
    if (pair_entry(a, c0 + p, true, 0, row) >= 0) {
      m.ptr = a.shared_ptr;
      m.kind = 1;
      m.off = a.direct ? a.B * a.k : 0;
      m.cnt = a.B;
    }
    m.row = row;
    meta[p] = m;
  }
  __syncthreads();  // meta and barrier initialisation visible
  issue(true);
  CYC(1);
  // activations (complete when this grid starts: they are the router's input)
  stage_digits(a.x, a.B, H, H, false, xfrag, xsx, xsum);
  if (a.B == 1) {  // token 1's columns are zero
    for (int q = tid; q < G * 2 * 4; q += blockDim.x) {
      const int g = q >> 3, h = (q >> 2) & 1, j = q & 3;
      uint2* fr = xfrag + ((size_t)g * 2 + h) * 32;
#pragma unroll
      for (int d = 0; d < 4; ++d) fr[16 + d * 4 + j] = make_uint2(0u, 0u);
    }
  }
  pdl_wait();
  TL_WAITED(0);
  CYC(2);
  {
    const int n_ent = gemv_entries<false>(a);
    for (int p = tid; p < np; p += blockDim.x) {
      if (meta[p].kind == 1) continue;
      int row = 0;
      const int j = pair_entry(a, c0 + p, false, n_ent, row);
      DecMeta m;
      m.ptr = nullptr;
      m.kind = 0;
      m.row = row;
      m.off = m.cnt = 0;
      m.tok = 0;
      if (j >= 0) {
        const ActEntry en = gemv_entry<false>(a, j);
        m.ptr = en.ptr;
        m.kind = en.kind;
        m.off = en.off;
        m.cnt = en.cnt;
        m.tok = en.pad0;
      }
      meta[p] = m;
    }
  }
  __syncthreads();
  CYC(3);
  issue(false);
  __syncthreads();  // every expect_tx precedes the arrival
  if (tid == 0)
    for (int tl = 0; tl < ntile; ++tl) mbar_arrive(&bars[tl]);
  // the down kernel may start now: it reads the routing through L2
  pdl_trigger();
  TL_MARK(8);
  CYC(4);
  cp_wait<0>();
  __syncthreads();  // scale rows visible
  CYC(5);
  // ---- items (tile, chunk of groups) on warps, each waiting only for its
  //      tile; lanes of a quad hold one MMA row's token columns (j even:
  //      digits 0,1; j odd: digit 2) ----
  const int r = lane >> 2, j = lane & 3, t = j >> 1;
  const int ks = max(1, min(kDecWarps / max(ntile, 1), G));  // chunks per tile
  const int gpc = (G + ks - 1) / ks;
  const int ssh = sst >> 1;  // scale-row stride in bf16 elements
  for (int item = warp; item < ntile * ks; item += kDecWarps) {
    const int tl = item / ks, q = item - tl * ks;
    const int g0 = q * gpc, g1 = min(G, g0 + gpc);
    if (!mbar_wait_first(&bars[tl], 0)) {
      if (lane == 0) atomicOr(a.status, kStatusCopyTimeout);
      mbar_wait(&bars[tl], 0);  // the copies may still land: wait once more
    }
    if (item == 0) CYC(6);
    float acc[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};  // [gate|up][mma row r | r+8]
    // MMA rows r and r+8: block r & 3, rows (r >> 2) and 2 + (r >> 2) in it
    const unsigned char* rbase = tiles + (size_t)(tl * 2 * 4 + (r & 3)) * bs +
                                 (size_t)(r >> 2) * rowb + 8 * j;
    const uint16_t* scb0 = reinterpret_cast<const uint16_t*>(scales) +
                           ((size_t)(tl * 4) * kTileRows + r) * ssh;
#pragma unroll 2
    for (int g = g0; g < g1; ++g) {
      const uint2 bA = xfrag[((size_t)g * 2 + 0) * 32 + lane];
      const uint2 bB = xfrag[((size_t)g * 2 + 1) * 32 + lane];
      const float sxp = xsx[((size_t)t * G + g) * 2 + (j & 1)];
      const float xsb = (j & 1) ? 0.0f : xsum[(size_t)t * G + g];  // bias term on even lanes
#pragma unroll
      for (int mat = 0; mat < 2; ++mat) {
        const unsigned char* rb0 = rbase + (size_t)mat * 4 * bs + 32 * g;
        const uint2 w0 = *reinterpret_cast<const uint2*>(rb0);
        const uint2 w8 = *reinterpret_cast<const uint2*>(rb0 + (size_t)2 * rowb);
        int d[4] = {0, 0, 0, 0};
        mma_s8(d, lo_nib(w0.x), lo_nib(w8.x), hi_nib(w0.x), hi_nib(w8.x), bA.x, bA.y);
        mma_s8(d, lo_nib(w0.y), lo_nib(w8.y), hi_nib(w0.y), hi_nib(w8.y), bB.x, bB.y);
        // [array][mma row]: scale (2 mat), bias (2 mat + 1)
        const uint16_t* sc = scb0 + (size_t)(2 * mat) * kTileRows * ssh + g;
        const uint16_t* bi = sc + (size_t)kTileRows * ssh;
        const int i0 = (j & 1) ? d[0] : d[0] * 128 + d[1];
        const int i8 = (j & 1) ? d[2] : d[2] * 128 + d[3];
        acc[mat][0] = fmaf(bf16_bits_to_f32(sc[0]) * sxp, (float)i0, acc[mat][0]);
        acc[mat][1] = fmaf(bf16_bits_to_f32(sc[(size_t)8 * ssh]) * sxp, (float)i8, acc[mat][1]);
        acc[mat][0] = fmaf(bf16_bits_to_f32(bi[0]), xsb, acc[mat][0]);
        acc[mat][1] = fmaf(bf16_bits_to_f32(bi[(size_t)8 * ssh]), xsb, acc[mat][1]);
      }
    }
#pragma unroll
    for (int mat = 0; mat < 2; ++mat)
#pragma unroll
      for (int h = 0; h < 2; ++h) acc[mat][h] += __shfl_xor_sync(0xFFFFFFFFu, acc[mat][h], 1);
    if (!(j & 1)) {
      // part[tile][chunk][mma row][mat][token]
      float* pw = part + ((size_t)tl * ks + q) * kTileRows * 4;
#pragma unroll
      for (int mat = 0; mat < 2; ++mat) {
        pw[(r * 2 + mat) * 2 + t] = acc[mat][0];
        pw[((r + 8) * 2 + mat) * 2 + t] = acc[mat][1];
      }
    }
  }
  __syncthreads();
  CYC(7);
  // ---- fixed-order sum over chunks, SwiGLU, store h ----
  for (int qq = tid; qq < np * a.B; qq += blockDim.x) {
    const int p = qq / a.B, tk = qq - p * a.B;
    const DecMeta m = meta[p];
    if (m.ptr == nullptr) continue;
    int pos = -1;
    if (a.direct) {
      // the shared entry holds every token's pair; a routed entry one token's
      if (m.kind == 1) pos = m.off + tk;
      else if (m.tok == tk) pos = m.off;
    } else {
      for (int i = 0; i < m.cnt; ++i)
        if (a.pair_tok[m.off + i] == tk) pos = m.off + i;
    }
    if (pos < 0) continue;
    const int tl = p / kTileRows, R = row_to_mma(p % kTileRows);
    float gs = 0.0f, us = 0.0f;
    for (int q = 0; q < ks; ++q) {
      const float* pw = part + ((size_t)tl * ks + q) * kTileRows * 4;
      gs += pw[(R * 2 + 0) * 2 + tk];
      us += pw[(R * 2 + 1) * 2 + tk];
    }
    a.h[(size_t)pos * a.Imax + m.row] = __fmul_rn(ref_silu(gs), us);
  }
  CYC(8);
  TL_END(0);
}

// ----------------------------------------------------------------------------
// down + combine.  CTA = output rows [r0, r0 + rpc), rpc <= 16, every entry.
// ----------------------------------------------------------------------------
__global__ void __launch_bounds__(kDecWarps * 32, 2) dec_down_kernel(GemvArgs a) {
  extern __shared__ __align__(128) unsigned char smraw[];
  const int P = a.B * (a.k + a.has_shared);
  const int Kmax = a.dn.K[0] > a.dn.K[1] ? a.dn.K[0] : a.dn.K[1];
  const int rpc = a.rpc, r0 = blockIdx.x * rpc, nr = min(rpc, a.H - r0);
  const int GdM = Kmax >> 6, Gh = a.Imax >> 6;
  const DnLayout Ly = dn_layout(a.max_entries, Kmax, a.Imax, P);
  unsigned char* wt = smraw + Ly.wt;
  uint16_t* scales = reinterpret_cast<uint16_t*>(smraw + Ly.scales);
  uint2* hfrag = reinterpret_cast<uint2*>(smraw + Ly.hfrag);
  float* hsx = reinterpret_cast<float*>(smraw + Ly.hsx);
  float* hsum = reinterpret_cast<float*>(smraw + Ly.hsum);
  float* ys = reinterpret_cast<float*>(smraw + Ly.ys);
  float* rwt = reinterpret_cast<float*>(smraw + Ly.rw);           // [B*(k+1)] weights, shared gate last
  int* rpos = reinterpret_cast<int*>(smraw + Ly.rw) + P;          // [B*(k+1)] pair of (token, pick)
  DecMeta* meta = reinterpret_cast<DecMeta*>(smraw + Ly.meta);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smraw + Ly.bars);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bs = Ly.bs;
  TL_START(1);
  CYC(16);
  // This grid starts once every gate/up CTA has passed its own dependency
  // wait, so the routing is complete; it is read through L2.
  const int ne = min(gemv_entries<true>(a), a.max_entries);
  {
    // combine inputs: weight and pair position of every (token, pick); the
    // shared expert is pick k with the sigmoid gate as its weight
    const int kp1 = a.k + a.has_shared;
    for (int q = tid; q < a.B * kp1; q += blockDim.x) {
      const int t = q / kp1, p = q - t * kp1;
      rwt[q] = p < a.k ? __ldcg(a.weights + t * a.k + p) : __ldcg(a.sgate + t);
      rpos[q] = a.direct ? (p < a.k ? t * a.k + p : a.B * a.k + t) : __ldcg(a.tp_pos + t * kp1 + p);
    }
  }
  for (int jj = tid; jj < ne; jj += blockDim.x) {
    const ActEntry en = gemv_entry<true>(a, jj);
    DecMeta m;
    m.ptr = en.ptr;
    m.kind = en.kind;
    m.off = en.off;
    m.cnt = en.cnt;
    m.row = 0;
    m.tok = en.pad0;
    meta[jj] = m;
  }
  CYC(17);
  if (tid < ne) {
    mbar_init(&bars[tid], 1);
    mbar_init_fence();
  }
  __syncthreads();
  // rows: one bulk copy per block of <= 4 consecutive output rows
  for (int q = tid; q < ne * 4; q += blockDim.x) {
    const int jj = q >> 2, b = q & 3, n = min(4, nr - 4 * b);
    const DecMeta& m = meta[jj];
    if (m.ptr == nullptr || n <= 0) continue;
    const int rb = a.dn.K[m.kind] >> 1;
    mbar_expect_tx(&bars[jj], (uint32_t)(n * rb));
    bulk_load(wt + (size_t)(jj * 4 + b) * bs, m.ptr + a.dn.w[m.kind] + (size_t)(r0 + 4 * b) * rb,
              (uint32_t)(n * rb), &bars[jj]);
  }
  CYC(18);
  // scale rows: cp.async granules, [entry][s|b][row][GdM]
  {
    const int scb = a.cs_dn;
    const int spr = (GdM * 2) / scb;
    for (int q = tid; q < ne * 2 * nr * spr; q += blockDim.x) {
      const int jj = q / (2 * nr * spr);
      int rem = q - jj * 2 * nr * spr;
      const int arr = rem / (nr * spr);
      rem -= arr * nr * spr;
      const int rr = rem / spr, c = rem - rr * spr;
      const DecMeta& m = meta[jj];
      const int Gd = a.dn.K[m.kind] >> 6;
      if (m.ptr == nullptr || c * scb >= Gd * 2) continue;
      cp_async(reinterpret_cast<unsigned char*>(scales) +
                   ((size_t)((jj * 2 + arr) * kTileRows + row_to_mma(rr)) * GdM) * 2 + c * scb,
               m.ptr + (arr ? a.dn.b[m.kind] : a.dn.s[m.kind]) + (size_t)(r0 + rr) * Gd * 2 + c * scb,
               scb);
    }
    cp_commit();
  }
  __syncthreads();  // every row issued
  if (tid < ne) mbar_arrive(&bars[tid]);
  CYC(19);
  pdl_wait();
  TL_WAITED(1);
  CYC(20);
  stage_digits(a.h, P, a.Imax, a.Imax, true, hfrag, hsx, hsum);
  cp_wait<0>();
  __syncthreads();
  CYC(21);
  TL_MARK(12);
  // ---- items (entry, half of its groups) on warps; each entry's pairs are
  //      separate MMA columns ----
  const int r = lane >> 2, j = lane & 3;
  const float bmask = j == 0 ? 1.0f : 0.0f;  // the bias term on one lane per row
  const int ksd = max(1, min(kDnChunks, kDecWarps / max(ne, 1)));  // group chunks per entry
  for (int item = warp; item < ksd * ne; item += kDecWarps) {
    const int jj = item / ksd, half = item - jj * ksd;
    const DecMeta m = meta[jj];
    if (m.ptr == nullptr) continue;
    if (!mbar_wait_first(&bars[jj], 0)) {
      if (lane == 0) atomicOr(a.status, kStatusCopyTimeout);
      mbar_wait(&bars[jj], 0);  // the copies may still land: wait once more
    }
    const int Gd = a.dn.K[m.kind] >> 6, gh = (Gd + ksd - 1) / ksd;
    const int ga = min(Gd, half * gh), gb = min(Gd, ga + gh);
    const int rbe = a.dn.K[m.kind] >> 1;  // bytes of one of this entry's rows
    // MMA rows r and r+8: block r & 3, rows (r >> 2) and 2 + (r >> 2) in it
    const unsigned char* rb0 = wt + (size_t)(jj * 4 + (r & 3)) * bs + (size_t)(r >> 2) * rbe + 8 * j;
    const uint16_t* sc = scales + ((size_t)(jj * 2) * kTileRows) * GdM;
    const uint16_t* bi = sc + (size_t)kTileRows * GdM;
    for (int i = 0; i < m.cnt; ++i) {
      const int pos = m.off + i;
      float acc0 = 0.0f, acc8 = 0.0f;
#pragma unroll 4
      for (int g = ga; g < gb; ++g) {
        const uint2 w0 = *reinterpret_cast<const uint2*>(rb0 + 32 * g);
        const uint2 w8 = *reinterpret_cast<const uint2*>(rb0 + (size_t)2 * rbe + 32 * g);
        const uint2* fr = hfrag + (((size_t)pos * Gh + g) * 2) * 16;
        const uint2 bA = lane < 16 ? fr[lane] : make_uint2(0u, 0u);  // columns 4..7 are zero
        const uint2 bB = lane < 16 ? fr[16 + lane] : make_uint2(0u, 0u);
        int d[4] = {0, 0, 0, 0};
        mma_s8(d, lo_nib(w0.x), lo_nib(w8.x), hi_nib(w0.x), hi_nib(w8.x), bA.x, bA.y);
        mma_s8(d, lo_nib(w0.y), lo_nib(w8.y), hi_nib(w0.y), hi_nib(w8.y), bB.x, bB.y);
        const float sxp = hsx[((size_t)pos * Gh + g) * 2 + (j & 1)];
        const float hb = bmask * hsum[(size_t)pos * Gh + g];
        const int i0 = (j & 1) ? d[0] : d[0] * 128 + d[1];
        const int i8 = (j & 1) ? d[2] : d[2] * 128 + d[3];
        acc0 = fmaf(bf16_bits_to_f32(sc[(size_t)r * GdM + g]) * sxp, (float)i0, acc0);
        acc8 = fmaf(bf16_bits_to_f32(sc[(size_t)(r + 8) * GdM + g]) * sxp, (float)i8, acc8);
        acc0 = fmaf(bf16_bits_to_f32(bi[(size_t)r * GdM + g]), hb, acc0);
        acc8 = fmaf(bf16_bits_to_f32(bi[(size_t)(r + 8) * GdM + g]), hb, acc8);
      }
      acc0 += __shfl_xor_sync(0xFFFFFFFFu, acc0, 1);
      acc8 += __shfl_xor_sync(0xFFFFFFFFu, acc8, 1);
      if (j == 0) {
        float* yh = ys + ((size_t)half * P + pos) * kTileRows;
        const int m0 = mma_to_row(r), m8 = mma_to_row(r + 8);
        if (m0 < nr) yh[m0] = acc0;
        if (m8 < nr) yh[m8] = acc8;
      }
    }
  }
  __syncthreads();
  CYC(22);
  TL_MARK(13);
  pdl_trigger();
  // combine in pick order, shared expert last, then the residual
  const int kp1 = a.k + a.has_shared;
  for (int i = tid; i < a.B * nr; i += blockDim.x) {
    const int t = i / nr, rr = i - t * nr;
    float acc = 0.0f;
    for (int p = 0; p < kp1; ++p) {
      const int pos = rpos[t * kp1 + p];
      float y = ys[(size_t)pos * kTileRows + rr];
      for (int c = 1; c < ksd; ++c) y += ys[((size_t)c * P + pos) * kTileRows + rr];
      acc = __fadd_rn(acc, __fmul_rn(rwt[t * kp1 + p], y));
    }
    if (a.residual) acc = __fadd_rn(a.residual[(size_t)t * a.H + r0 + rr], acc);
    a.out[(size_t)t * a.H + r0 + rr] = acc;
  }
  CYC(23);
  TL_END(1);
}

// ============================================================================
// Three or more tokens: grouped projections.
//
// Work items are (chunk of up to 8 pairs of one active expert, block of
// rows), numbered chunk-major so that a CTA's contiguous run of items mostly
// shares its chunk, whose activation digits are staged once.  One producer
// thread streams each item's weight rows and scale rows into a ring of
// stages with bulk copies (full barrier: copies landed; empty barrier: all 8
// consumer warps are done with the stage), writing the item's descriptor at
// the head of the stage.  The MMA tile's 8 columns are the chunk's 8 tokens
// and its three digit planes are three MMAs (digit-major), so one A fragment
// serves every token; the consumer warps split the input groups and their
// partial sums are added in a fixed order.
// ============================================================================
constexpr int kChunk = 8;       // pairs per chunk = MMA columns
constexpr int kGuBlk = 32;      // gate/up rows per item (2 MMA row tiles)
constexpr int kDnBlk = 64;      // down output rows per item (4 MMA row tiles)
constexpr int kCons = 8;        // consumer warps
constexpr int kGrpThreads = (kCons + 1) * 32;
constexpr int kMaxStages = 8;
constexpr int kStageHdr = 128;  // item descriptor at the head of each stage

struct GrpDesc {
  const uint8_t* ptr;
  int kind, rb, pos0, ntok, chunk, end;
};

struct GrpLayout {
  size_t dig, q, stage, stage_bytes, wts, scales, part, part_bytes, crow, bars, total;
  int bs, nst;
};
__host__ __device__ inline size_t align128(size_t v) { return (v + 127) & ~(size_t)127; }

// gate/up stage: [descriptor][gate: 8 blocks of 4 rows][up: 8 blocks][scales:
// gate_s, gate_b, up_s, up_b, 32 rows of G bf16 each]
__host__ __device__ inline GrpLayout grp_gu_layout(int H, int nst) {
  const size_t G = (size_t)H >> 6;
  GrpLayout L;
  L.nst = nst;
  L.bs = pad_stride(4 * (H >> 1));
  size_t o = 0;
  L.dig = o;   o += G * 2 * 3 * 32 * 8;
  L.q = o;     o += G * kChunk * 16;
  L.wts = kStageHdr;
  L.scales = kStageHdr + (size_t)2 * (kGuBlk / 4) * L.bs;
  L.stage_bytes = align128(L.scales + (size_t)4 * kGuBlk * G * 2);
  o = align128(o);
  L.stage = o; o += (size_t)nst * L.stage_bytes;
  L.part_bytes = (size_t)kCons * 32 * 8 * 4;
  L.part = o;  o += 2 * L.part_bytes;
  L.crow = o;  o += 64;
  L.bars = o;  o += 2 * kMaxStages * 8;
  L.total = o;
  return L;
}

// down stage: [descriptor][16 blocks of 4 rows][scales: down_s, down_b, 64
// rows of K/64 bf16 each]
__host__ __device__ inline GrpLayout grp_dn_layout(int Kmax, int Imax, int nst) {
  const size_t Gh = (size_t)Imax >> 6, Gk = (size_t)Kmax >> 6;
  GrpLayout L;
  L.nst = nst;
  L.bs = pad_stride(4 * (Kmax >> 1));
  size_t o = 0;
  L.dig = o;   o += Gh * 2 * 3 * 32 * 8;
  L.q = o;     o += Gh * kChunk * 16;
  L.wts = kStageHdr;
  L.scales = kStageHdr + (size_t)(kDnBlk / 4) * L.bs;
  L.stage_bytes = align128(L.scales + (size_t)2 * kDnBlk * Gk * 2);
  o = align128(o);
  L.stage = o; o += (size_t)nst * L.stage_bytes;
  L.part_bytes = (size_t)kCons * 32 * 4 * 4;
  L.part = o;  o += 2 * L.part_bytes;
  L.crow = o;  o += 64;
  L.bars = o;  o += 2 * kMaxStages * 8;
  L.total = o;
  return L;
}

// Digit-major activation fragments of a chunk (consumer threads only):
// dig[g][half][digit][t*4 + j] (uint2) for slots t < 8 (slots >= nrow are
// zero) and q[g][t] = {s/128, s/16384, sum(x), 0}.  The 8 items of (t, g) are
// consecutive lanes of one warp; a thread's loads are issued ahead of its
// conversions.
__device__ void stage_digits_dm(const float* __restrict__ src, const int* rowmap, int nrow,
                                int ld, int K, uint2* dig, float4* q, int tid) {
  constexpr int U = 4;
  const int G = K >> 6;
  const int items = kChunk * G * 8;  // a multiple of 64: warps are all live or all idle
  for (int base = 0; base < items; base += U * kCons * 32) {
    float v[U][8];
    int itc[U];
    bool live[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int it = base + u * kCons * 32 + tid;
      live[u] = it < items;
      itc[u] = live[u] ? it : items - 1;
      const int j = itc[u] & 3, h = (itc[u] >> 2) & 1, g = (itc[u] >> 3) % G, t = (itc[u] >> 3) / G;
      if (t < nrow) {
        const float* p = src + (size_t)rowmap[t] * ld + 64 * g + 16 * j + 8 * h;
        const float4 u0 = __ldcg(reinterpret_cast<const float4*>(p));
        const float4 u1 = __ldcg(reinterpret_cast<const float4*>(p + 4));
        v[u][0] = u0.x; v[u][1] = u0.y; v[u][2] = u0.z; v[u][3] = u0.w;
        v[u][4] = u1.x; v[u][5] = u1.y; v[u][6] = u1.z; v[u][7] = u1.w;
      } else {
#pragma unroll
        for (int m = 0; m < 8; ++m) v[u][m] = 0.0f;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (base + u * kCons * 32 + (tid & ~31) >= items) break;  // the whole warp is idle
      const int j = itc[u] & 3, h = (itc[u] >> 2) & 1, g = (itc[u] >> 3) % G, t = (itc[u] >> 3) / G;
      float mx = 0.0f, sm = 0.0f;
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        mx = fmaxf(mx, fabsf(v[u][m]));
        sm += v[u][m];
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
        sm += __shfl_xor_sync(0xFFFFFFFFu, sm, o);
      }
      if (!live[u]) continue;
      const int e = group_exponent(mx);
      const Digits D = make_digits(v[u], e);
#pragma unroll
      for (int d = 0; d < 3; ++d)
        dig[(((size_t)g * 2 + h) * 3 + d) * 32 + t * 4 + j] = make_uint2(D.b0[d], D.b1[d]);
      if (h == 0 && j == 0) {
        const float s = __uint_as_float((uint32_t)(127 + e) << 23);
        q[(size_t)g * kChunk + t] =
            t < nrow ? make_float4(s * 0.0078125f, s * 6.103515625e-05f, sm, 0.0f)
                     : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
    }
  }
}

// B fragments of group g: b[digit][half].
__device__ __forceinline__ void load_b_dm(uint2 (&b)[3][2], const uint2* dig, int g, int lane) {
#pragma unroll
  for (int d = 0; d < 3; ++d)
#pragma unroll
    for (int h = 0; h < 2; ++h) b[d][h] = dig[(((size_t)g * 2 + h) * 3 + d) * 32 + lane];
}

// One group of one 16-row tile against the chunk's 8 tokens.  Each digit
// plane has its own s32 tile (two dependent MMAs each, so the three planes
// overlap in the pipe); V = D0 2^14 + D1 2^7 + D2 exactly
// (|V| < 64*15*64*16384*1.01 < 2^31).
__device__ __forceinline__ void mma_group_dm(int (&V)[4], uint2 w0, uint2 w8, const uint2 (&b)[3][2]) {
  const uint32_t a0 = lo_nib(w0.x), a1 = lo_nib(w8.x), a2 = hi_nib(w0.x), a3 = hi_nib(w8.x);
  const uint32_t c0 = lo_nib(w0.y), c1 = lo_nib(w8.y), c2 = hi_nib(w0.y), c3 = hi_nib(w8.y);
  int D[3][4];
#pragma unroll
  for (int d = 0; d < 3; ++d) {
    D[d][0] = D[d][1] = D[d][2] = D[d][3] = 0;
    mma_s8(D[d], a0, a1, a2, a3, b[d][0].x, b[d][0].y);
  }
#pragma unroll
  for (int d = 0; d < 3; ++d) mma_s8(D[d], c0, c1, c2, c3, b[d][1].x, b[d][1].y);
#pragma unroll
  for (int i = 0; i < 4; ++i) V[i] = D[0][i] * 16384 + D[1][i] * 128 + D[2][i];
}

// acc[hh][tt] += s_w * (s / 2^14) V + b_w * sum(x), for MMA rows r (hh 0) and
// r+8 (hh 1) and this lane's tokens 2j, 2j+1 (tt); sb packs the row's bf16
// scale (low half) and bias (high half).
__device__ __forceinline__ void epilogue_dm(float (&acc)[2][2], const int (&V)[4], uint32_t sb0,
                                            uint32_t sb8, float4 q0, float4 q1) {
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const uint32_t sb = hh ? sb8 : sb0;
    const float sw = __uint_as_float(sb << 16), bw = __uint_as_float(sb & 0xFFFF0000u);
#pragma unroll
    for (int tt = 0; tt < 2; ++tt) {
      const float4 q = tt ? q1 : q0;
      acc[hh][tt] = fmaf(bw, q.z, fmaf(sw, q.y * (float)V[2 * hh + tt], acc[hh][tt]));
    }
  }
}

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kCons * 32) : "memory");
}
// Named barrier of the consumer warps that also ORs a flag across them.
__device__ __forceinline__ bool consumer_sync_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 2, %2, p;\n"
      " selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(kCons * 32)
      : "memory");
  return r != 0;
}

// Item -> descriptor; false when the item has no work (a chunk's rows beyond
// a smaller expert kind, or an expert without a slot).
__device__ __forceinline__ bool grp_decode(const GrpArgs& a, int item, int nrb, bool down,
                                           int& last_ch, ActEntry& en, int2& cj, GrpDesc& d) {
  const int rb = item % nrb, ch = item / nrb;
  if (ch != last_ch) {
    cj = a.chunks[ch];
    en = a.act[cj.x];
    last_ch = ch;
  }
  const int ntok = min(kChunk, en.cnt - cj.y);
  const int rows = down ? a.dn.rows[en.kind] : a.gu.rows[en.kind];
  d.ptr = en.ptr;
  d.kind = en.kind;
  d.rb = rb;
  d.pos0 = en.off + cj.y;
  d.ntok = ntok;
  d.chunk = ch;
  d.end = 0;
  return ntok > 0 && en.ptr != nullptr && rb * (down ? kDnBlk : kGuBlk) < rows;
}

// Producer thread: items [i0, i1) into the stage ring, then an end marker;
// finally waits (bounded) for its copies still in flight.
template <bool DOWN>
__device__ void grp_produce(const GrpArgs& a, const GrpLayout& Ly, unsigned char* smraw,
                            uint64_t* full, uint64_t* empty, int i0, int i1, int nrb) {
  const int nst = Ly.nst;
  uint32_t n = 0;
  bool ok = true;
  int last_ch = -1;
  ActEntry en{};
  int2 cj = make_int2(0, 0);
  for (int item = i0; item < i1; ++item) {
    GrpDesc d;
    if (!grp_decode(a, item, nrb, DOWN, last_ch, en, cj, d)) continue;
    const int s = (int)(n % nst);
    const uint32_t k = n / nst;
    if (k > 0 && !mbar_wait(&empty[s], (k - 1) & 1)) {
      atomicOr(a.status, kStatusCopyTimeout);
      ok = false;
      break;
    }
    unsigned char* base = smraw + Ly.stage + (size_t)s * Ly.stage_bytes;
    *reinterpret_cast<GrpDesc*>(base) = d;
    if (!DOWN) {
      const int H = a.H, G = H >> 6, rowb = H >> 1;
      const int nrow = min(kGuBlk, a.gu.rows[d.kind] - d.rb * kGuBlk);  // a multiple of 4
      const uint32_t sbytes = (uint32_t)(nrow * G * 2);
      mbar_arrive_expect(&full[s], (uint32_t)(2 * nrow * rowb) + 4u * sbytes);
      const size_t r0 = (size_t)d.rb * kGuBlk;
      for (int b = 0; b < nrow / 4; ++b) {
        const size_t off = (r0 + 4 * b) * rowb;
        bulk_load(base + Ly.wts + (size_t)b * Ly.bs, d.ptr + a.gu.w[d.kind] + off, 4u * rowb, &full[s]);
        bulk_load(base + Ly.wts + (size_t)(kGuBlk / 4 + b) * Ly.bs, d.ptr + a.gu.w2[d.kind] + off,
                  4u * rowb, &full[s]);
      }
      const uint64_t so[4] = {a.gu.s[d.kind], a.gu.b[d.kind], a.gu.s2[d.kind], a.gu.b2[d.kind]};
      for (int arr = 0; arr < 4; ++arr)
        bulk_load(base + Ly.scales + (size_t)arr * kGuBlk * G * 2, d.ptr + so[arr] + r0 * G * 2, sbytes,
                  &full[s]);
    } else {
      const int K = a.dn.K[d.kind], rbe = K >> 1, Gd = K >> 6;
      const int r0 = d.rb * kDnBlk;
      const int nrow = min(kDnBlk, a.dn.rows[d.kind] - r0);  // a multiple of 64
      const uint32_t sbytes = (uint32_t)(nrow * Gd * 2);
      mbar_arrive_expect(&full[s], (uint32_t)(nrow * rbe) + 2u * sbytes);
      for (int b = 0; b < nrow / 4; ++b)
        bulk_load(base + Ly.wts + (size_t)b * Ly.bs, d.ptr + a.dn.w[d.kind] + (size_t)(r0 + 4 * b) * rbe,
                  4u * rbe, &full[s]);
      bulk_load(base + Ly.scales, d.ptr + a.dn.s[d.kind] + (size_t)r0 * Gd * 2, sbytes, &full[s]);
      bulk_load(base + Ly.scales + (size_t)kDnBlk * Gd * 2, d.ptr + a.dn.b[d.kind] + (size_t)r0 * Gd * 2,
                sbytes, &full[s]);
    }
    ++n;
  }
  if (ok) {
    const int s = (int)(n % nst);
    const uint32_t k = n / nst;
    if (k > 0 && !mbar_wait(&empty[s], (k - 1) & 1)) {
      atomicOr(a.status, kStatusCopyTimeout);
    } else {
      GrpDesc d{};
      d.end = 1;
      *reinterpret_cast<GrpDesc*>(smraw + Ly.stage + (size_t)s * Ly.stage_bytes) = d;
      mbar_arrive(&full[s]);
    }
  }
  // copies of the last uses of the other stages may still be landing
  for (uint32_t m = n + 1 > (uint32_t)nst ? n + 1 - nst : 0; m < n; ++m)
    mbar_wait(&full[m % nst], (m / nst) & 1);
}

__global__ void __launch_bounds__(kGrpThreads, 1) grp_gateup_kernel(GrpArgs a) {
  extern __shared__ __align__(128) unsigned char smraw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = a.H, G = H >> 6, rowb = H >> 1;
  const GrpLayout Ly = grp_gu_layout(H, a.st_gu);
  uint64_t* full = reinterpret_cast<uint64_t*>(smraw + Ly.bars);
  uint64_t* empty = full + kMaxStages;
  GCYC(0, 0);
  TL_START(2);
  if (tid == 0) {
    for (int s = 0; s < Ly.nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCons);
    }
    mbar_init_fence();
  }
  __syncthreads();
  pdl_wait();
  GCYC(0, 1);
  TL_WAITED(2);
  const int nrb = a.rb_gu;
  const int n_items = *a.n_ch * nrb;
  const int per = (n_items + gridDim.x - 1) / gridDim.x;
  const int i0 = min(n_items, (int)blockIdx.x * per), i1 = min(n_items, i0 + per);
  if (warp == kCons) {
    if (lane == 0) grp_produce<false>(a, Ly, smraw, full, empty, i0, i1, nrb);
    return;
  }
  uint2* dig = reinterpret_cast<uint2*>(smraw + Ly.dig);
  float4* xq = reinterpret_cast<float4*>(smraw + Ly.q);
  int* crow = reinterpret_cast<int*>(smraw + Ly.crow);
  const int r = lane >> 2, j = lane & 3;
  const int rt = warp & 1, kq = warp >> 1;  // row tile, input quarter
  const int gq = (G + 3) / 4, ga = min(G, kq * gq), gb = min(G, ga + gq);
  const int m0 = rt * 16 + mma_to_row(r);   // tile rows of MMA rows r and r+8 (m0 + 2)
  uint32_t n = 0;
  int cur_chunk = -1, pb = 0;
  for (;; ++n) {
    const int s = (int)(n % Ly.nst);
    bool bad = false;
    if (!mbar_wait_first(&full[s], (n / Ly.nst) & 1)) {
      if (lane == 0) atomicOr(a.status, kStatusCopyTimeout);
      bad = !mbar_wait(&full[s], (n / Ly.nst) & 1);
    }
    if (consumer_sync_or(bad)) break;
    const unsigned char* base = smraw + Ly.stage + (size_t)s * Ly.stage_bytes;
    const GrpDesc cur = *reinterpret_cast<const GrpDesc*>(base);
    if (cur.end) break;
    GCYC(0, 2 + 3 * (n & 15));
    if (cur.chunk != cur_chunk) {
      if (tid < kChunk) crow[tid] = tid < cur.ntok ? a.pair_tok[cur.pos0 + tid] : 0;
      consumer_sync();
      stage_digits_dm(a.x, crow, cur.ntok, H, H, dig, xq, tid);
      consumer_sync();
      cur_chunk = cur.chunk;
    }
    GCYC(0, 3 + 3 * (n & 15));
    // scale/bias pairs of this lane's two rows over its input groups
    const uint16_t* scr = reinterpret_cast<const uint16_t*>(base + Ly.scales);
    uint32_t sb[2][2][8];
#pragma unroll
    for (int mat = 0; mat < 2; ++mat)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const uint16_t* sr = scr + ((size_t)(2 * mat) * kGuBlk + m0 + 2 * hh) * G + ga;
        const uint16_t* br = sr + (size_t)kGuBlk * G;
        if (G == 32) {
          const uint4 sv = *reinterpret_cast<const uint4*>(sr), bv = *reinterpret_cast<const uint4*>(br);
          const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w}, bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            sb[mat][hh][2 * u] = __byte_perm(sw[u], bw[u], 0x5410);
            sb[mat][hh][2 * u + 1] = __byte_perm(sw[u], bw[u], 0x7632);
          }
        } else {
#pragma unroll
          for (int u = 0; u < 8; ++u)
            sb[mat][hh][u] = ga + u < gb ? (uint32_t)sr[u] | ((uint32_t)br[u] << 16) : 0u;
        }
      }
    const unsigned char* rbase = base + Ly.wts + (size_t)(rt * 4 + (r & 3)) * Ly.bs + (size_t)(r >> 2) * rowb + 8 * j;
    float acc[2][2][2] = {};  // [gate|up][row r | r+8][token 2j | 2j+1]
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int g = ga + u;
      if (g < gb) {
        const float4 q0 = xq[(size_t)g * kChunk + 2 * j], q1 = xq[(size_t)g * kChunk + 2 * j + 1];
        uint2 bf[3][2];
        load_b_dm(bf, dig, g, lane);
#pragma unroll
        for (int mat = 0; mat < 2; ++mat) {
          const unsigned char* rb0 = rbase + (size_t)mat * (kGuBlk / 4) * Ly.bs + 32 * g;
          const uint2 w0 = *reinterpret_cast<const uint2*>(rb0);
          const uint2 w8 = *reinterpret_cast<const uint2*>(rb0 + (size_t)2 * rowb);
          int V[4];
          mma_group_dm(V, w0, w8, bf);
          epilogue_dm(acc[mat], V, sb[mat][0][u], sb[mat][1][u], q0, q1);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with the stage
    float* part = reinterpret_cast<float*>(smraw + Ly.part + (size_t)pb * Ly.part_bytes);
    float* pw = part + ((size_t)warp * 32 + lane) * 8;
#pragma unroll
    for (int mat = 0; mat < 2; ++mat)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
#pragma unroll
        for (int tt = 0; tt < 2; ++tt) pw[(mat * 2 + hh) * 2 + tt] = acc[mat][hh][tt];
    consumer_sync();
    GCYC(0, 4 + 3 * (n & 15));
    // fixed-order sum of the four input quarters, SwiGLU, store h: one
    // (row, token) per consumer thread
    {
      const int ort = tid >> 7, ol = (tid >> 2) & 31, ohh = (tid >> 1) & 1, ott = tid & 1;
      float gs = 0.0f, us = 0.0f;
#pragma unroll
      for (int qq = 0; qq < 4; ++qq) {
        const float* pp = part + ((size_t)(qq * 2 + ort) * 32 + ol) * 8;
        gs += pp[(0 * 2 + ohh) * 2 + ott];
        us += pp[(1 * 2 + ohh) * 2 + ott];
      }
      const int row = cur.rb * kGuBlk + ort * 16 + mma_to_row((ol >> 2) + 8 * ohh);
      const int t = 2 * (ol & 3) + ott;
      if (t < cur.ntok && row < a.gu.rows[cur.kind])
        a.h[(size_t)(cur.pos0 + t) * a.Imax + row] = __fmul_rn(ref_silu(gs), us);
    }
    pb ^= 1;
  }
  GCYC(0, 63);
  TL_END(2);
  pdl_trigger();
}

__global__ void __launch_bounds__(kGrpThreads, 1) grp_down_kernel(GrpArgs a) {
  extern __shared__ __align__(128) unsigned char smraw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Kmax = a.dn.K[0] > a.dn.K[1] ? a.dn.K[0] : a.dn.K[1];
  const GrpLayout Ly = grp_dn_layout(Kmax, a.Imax, a.st_dn);
  uint64_t* full = reinterpret_cast<uint64_t*>(smraw + Ly.bars);
  uint64_t* empty = full + kMaxStages;
  GCYC(1, 0);
  TL_START(3);
  if (tid == 0) {
    for (int s = 0; s < Ly.nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCons);
    }
    mbar_init_fence();
  }
  __syncthreads();
  pdl_wait();
  GCYC(1, 1);
  TL_WAITED(3);
  const int nrb = a.ob_dn;
  const int n_items = *a.n_ch * nrb;
  const int per = (n_items + gridDim.x - 1) / gridDim.x;
  const int i0 = min(n_items, (int)blockIdx.x * per), i1 = min(n_items, i0 + per);
  if (warp == kCons) {
    if (lane == 0) grp_produce<true>(a, Ly, smraw, full, empty, i0, i1, nrb);
    return;
  }
  uint2* dig = reinterpret_cast<uint2*>(smraw + Ly.dig);
  float4* hq = reinterpret_cast<float4*>(smraw + Ly.q);
  int* crow = reinterpret_cast<int*>(smraw + Ly.crow);
  const int r = lane >> 2, j = lane & 3;
  const int rt = warp & 3, kh = warp >> 2;  // row tile, input half
  const int m0 = rt * 16 + mma_to_row(r);
  int* corow = crow + kChunk;                // partial row of each pair of the chunk
  uint32_t n = 0;
  int cur_chunk = -1, pb = 0;
  for (;; ++n) {
    const int s = (int)(n % Ly.nst);
    bool bad = false;
    if (!mbar_wait_first(&full[s], (n / Ly.nst) & 1)) {
      if (lane == 0) atomicOr(a.status, kStatusCopyTimeout);
      bad = !mbar_wait(&full[s], (n / Ly.nst) & 1);
    }
    if (consumer_sync_or(bad)) break;
    const unsigned char* base = smraw + Ly.stage + (size_t)s * Ly.stage_bytes;
    const GrpDesc cur = *reinterpret_cast<const GrpDesc*>(base);
    if (cur.end) break;
    GCYC(1, 2 + 3 * (n & 15));
    if (cur.chunk != cur_chunk) {
      if (tid < kChunk) {
        const int pos = cur.pos0 + tid;
        crow[tid] = tid < cur.ntok ? pos : cur.pos0;
        corow[tid] = tid < cur.ntok ? a.pair_tok[pos] * a.kp1 + a.pair_pick[pos] : 0;
      }
      consumer_sync();
      stage_digits_dm(a.h, crow, cur.ntok, a.Imax, a.Imax, dig, hq, tid);
      consumer_sync();
      cur_chunk = cur.chunk;
    }
    GCYC(1, 3 + 3 * (n & 15));
    const int rbe = a.dn.K[cur.kind] >> 1, Gd = a.dn.K[cur.kind] >> 6;
    const int gh = (Gd + 1) >> 1, ga = min(Gd, kh * gh), gb = min(Gd, ga + gh);
    const uint16_t* sr0 = reinterpret_cast<const uint16_t*>(base + Ly.scales) + (size_t)m0 * Gd + ga;
    uint32_t sb[2][6];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const uint16_t* sr = sr0 + (size_t)(2 * hh) * Gd;
      const uint16_t* br = sr + (size_t)kDnBlk * Gd;
      if (Gd == 8) {
        const uint2 sv = *reinterpret_cast<const uint2*>(sr), bv = *reinterpret_cast<const uint2*>(br);
        sb[hh][0] = __byte_perm(sv.x, bv.x, 0x5410);
        sb[hh][1] = __byte_perm(sv.x, bv.x, 0x7632);
        sb[hh][2] = __byte_perm(sv.y, bv.y, 0x5410);
        sb[hh][3] = __byte_perm(sv.y, bv.y, 0x7632);
        sb[hh][4] = sb[hh][5] = 0u;
      } else {
#pragma unroll
        for (int u = 0; u < 6; ++u)
          sb[hh][u] = ga + u < gb ? (uint32_t)sr[u] | ((uint32_t)br[u] << 16) : 0u;
      }
    }
    const unsigned char* rbase = base + Ly.wts + (size_t)(rt * 4 + (r & 3)) * Ly.bs + (size_t)(r >> 2) * rbe + 8 * j;
    float acc[2][2] = {};  // [row r | r+8][pair 2j | 2j+1]
#pragma unroll
    for (int u = 0; u < 6; ++u) {
      const int g = ga + u;
      if (g < gb) {
        const float4 q0 = hq[(size_t)g * kChunk + 2 * j], q1 = hq[(size_t)g * kChunk + 2 * j + 1];
        const uint2 w0 = *reinterpret_cast<const uint2*>(rbase + 32 * g);
        const uint2 w8 = *reinterpret_cast<const uint2*>(rbase + (size_t)2 * rbe + 32 * g);
        uint2 bf[3][2];
        load_b_dm(bf, dig, g, lane);
        int V[4];
        mma_group_dm(V, w0, w8, bf);
        epilogue_dm(acc, V, sb[0][u], sb[1][u], q0, q1);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    float* part = reinterpret_cast<float*>(smraw + Ly.part + (size_t)pb * Ly.part_bytes);
    float* pw = part + ((size_t)warp * 32 + lane) * 4;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
      for (int tt = 0; tt < 2; ++tt) pw[hh * 2 + tt] = acc[hh][tt];
    consumer_sync();
    GCYC(1, 4 + 3 * (n & 15));
    // fixed-order sum of the two input halves, store partial rows: two
    // (row, pair) outputs per consumer thread
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int o = tid + half * kCons * 32;
      const int ort = o >> 7, ol = (o >> 2) & 31, ohh = (o >> 1) & 1, ott = o & 1;
      const int c = ohh * 2 + ott;
      const float v = part[((size_t)ort * 32 + ol) * 4 + c] + part[((size_t)(4 + ort) * 32 + ol) * 4 + c];
      const int row = cur.rb * kDnBlk + ort * 16 + mma_to_row((ol >> 2) + 8 * ohh);
      const int t = 2 * (ol & 3) + ott;
      if (t < cur.ntok && row < a.dn.rows[cur.kind]) a.partial[(size_t)corow[t] * a.H + row] = v;
    }
    pb ^= 1;
  }
  GCYC(1, 63);
  TL_END(3);
  pdl_trigger();
}

template <typename K, typename... Args>
void launch_pdl(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
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

// Largest copy granule (16, 8 or 4 bytes) dividing every offset and the
// row length n; 0 when none does.
int granule(const uint64_t* offs, int count, uint64_t n) {
  for (int g = 16; g >= 4; g >>= 1) {
    bool ok = n % g == 0;
    for (int i = 0; i < count; ++i) ok = ok && offs[i] % g == 0;
    if (ok) return g;
  }
  return 0;
}

}  // namespace

void init_gemv_attributes(int max_smem) {
  cudaFuncSetAttribute(dec_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(dec_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  // the largest shared-memory carveout, so a down CTA fits beside a gate/up CTA
  cudaFuncSetAttribute(dec_gateup_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  cudaFuncSetAttribute(dec_down_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
}

bool gemv_configure(GemvArgs& a, int max_active, int num_sms, int max_smem, GemvLaunch* out) {
  if (a.B < 1 || a.B > 2 || num_sms < 1) return false;
  const int nk = a.has_shared ? 2 : 1;
  // the input dims are whole 64-groups in 32-wide MMA slabs; rows copy in
  // 16-byte chunks
  if (a.H % 128 || a.Imax % 64) return false;
  for (int kd = 0; kd < nk; ++kd) {
    if (a.gu.K[kd] != a.H || a.dn.K[kd] % 64 || a.dn.rows[kd] != a.H) return false;
    if (a.gu.w[kd] % 16 || a.gu.w2[kd] % 16 || a.dn.w[kd] % 16) return false;
  }
  if (a.slab_stride % 16 || reinterpret_cast<uintptr_t>(a.slab) % 16 ||
      reinterpret_cast<uintptr_t>(a.shared_ptr) % 16)
    return false;
  // scale rows: G bf16 per gate/up row, Gd per down row
  {
    uint64_t o[9];
    int n = 0;
    for (int kd = 0; kd < nk; ++kd) {
      o[n++] = a.gu.s[kd]; o[n++] = a.gu.b[kd]; o[n++] = a.gu.s2[kd]; o[n++] = a.gu.b2[kd];
    }
    o[n++] = a.slab_stride;
    a.cs_gu = granule(o, n, (uint64_t)(a.H >> 6) * 2);
    n = 0;
    for (int kd = 0; kd < nk; ++kd) {
      o[n++] = a.dn.s[kd]; o[n++] = a.dn.b[kd];
    }
    o[n++] = a.slab_stride;
    int cs = 16;
    for (int kd = 0; kd < nk; ++kd) {
      const int c = granule(o, n, (uint64_t)(a.dn.K[kd] >> 6) * 2);
      if (c < cs) cs = c;
    }
    a.cs_dn = cs;
    if (a.cs_gu == 0 || a.cs_dn == 0) return false;
  }
  const int rs = a.has_shared ? a.gu.rows[1] : 0;
  a.total_max = rs + (max_active - a.has_shared) * a.gu.rows[0];
  int grid = num_sms;
  const int need = (a.total_max + kTileRows - 1) / kTileRows;
  if (need < grid) grid = need < 1 ? 1 : need;
  a.per_cta = (a.total_max + grid - 1) / grid;
  a.per_cta = (a.per_cta + 3) & ~3;  // CTA ranges start on 4-row blocks
  grid = (a.total_max + a.per_cta - 1) / a.per_cta;
  a.nbuf = (a.per_cta + kTileRows - 1) / kTileRows;  // tiles per CTA
  if (a.nbuf > 8) return false;
  const size_t gu_smem = gu_layout(a.H, a.nbuf, a.per_cta).total;
  a.max_entries = max_active;
  int rpc = (a.H + num_sms - 1) / num_sms;
  if (rpc < 1) rpc = 1;
  if (rpc > kTileRows) return false;
  a.rpc = rpc;
  const int Kmax = a.dn.K[0] > a.dn.K[1] ? a.dn.K[0] : a.dn.K[1];
  if (Kmax > a.Imax) return false;
  const int P = a.B * (a.k + a.has_shared);
  const size_t dn_smem = dn_layout(a.max_entries, Kmax, a.Imax, P).total;
  if (gu_smem > (size_t)max_smem || dn_smem > (size_t)max_smem) return false;
  out->grid_gu = grid;
  out->grid_dn = (a.H + rpc - 1) / rpc;
  out->smem_gu = gu_smem;
  out->smem_dn = dn_smem;
  return true;
}

void launch_gemv_gateup(const GemvArgs& a, const GemvLaunch& l, cudaStream_t s,
                        uint64_t* launches) {
  launch_pdl(dec_gateup_kernel, dim3(l.grid_gu), dim3(kDecWarps * 32), l.smem_gu, s, a);
  if (launches) *launches += 1;
}

void launch_gemv_down(const GemvArgs& a, const GemvLaunch& l, cudaStream_t s, uint64_t* launches) {
  launch_pdl(dec_down_kernel, dim3(l.grid_dn), dim3(kDecWarps * 32), l.smem_dn, s, a);
  if (launches) *launches += 1;
}


void init_grouped_attributes(int max_smem) {
  cudaFuncSetAttribute(grp_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(grp_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
}

bool grouped_configure(GrpArgs& a, int max_smem, size_t* smem_gu, size_t* smem_dn) {
  const int nk = a.has_shared ? 2 : 1;
  if (a.H % 128 || a.Imax % 128 || a.H > 2048) return false;
  for (int kd = 0; kd < nk; ++kd) {
    if (a.gu.K[kd] != a.H || a.dn.rows[kd] != a.H || a.dn.K[kd] % 128 || a.dn.K[kd] > 768)
      return false;
    if (a.gu.rows[kd] % 4) return false;  // whole 4-row copy blocks
    // bulk copies: 16-byte aligned sources
    const uint64_t o[9] = {a.gu.w[kd], a.gu.w2[kd], a.dn.w[kd], a.gu.s[kd], a.gu.b[kd],
                           a.gu.s2[kd], a.gu.b2[kd], a.dn.s[kd], a.dn.b[kd]};
    for (uint64_t v : o)
      if (v % 16) return false;
  }
  if (a.slab_stride % 16) return false;
  const int rmax = a.gu.rows[0] > a.gu.rows[1] ? a.gu.rows[0] : a.gu.rows[1];
  a.rb_gu = (rmax + kGuBlk - 1) / kGuBlk;
  a.ob_dn = (a.H + kDnBlk - 1) / kDnBlk;
  const int Kmax = a.dn.K[0] > a.dn.K[1] ? a.dn.K[0] : a.dn.K[1];
  if (Kmax > a.Imax) return false;
  // as many stages as fit, up to kMaxStages; at least two
  int st = kMaxStages;
  while (st >= 2 && grp_gu_layout(a.H, st).total > (size_t)max_smem) --st;
  a.st_gu = st;
  st = kMaxStages;
  while (st >= 2 && grp_dn_layout(Kmax, a.Imax, st).total > (size_t)max_smem) --st;
  a.st_dn = st;
  if (a.st_gu < 2 || a.st_dn < 2) return false;
  *smem_gu = grp_gu_layout(a.H, a.st_gu).total;
  *smem_dn = grp_dn_layout(Kmax, a.Imax, a.st_dn).total;
  return true;
}

void launch_grouped_gateup(const GrpArgs& a, int grid, size_t smem, cudaStream_t s,
                           uint64_t* launches) {
  launch_pdl(grp_gateup_kernel, dim3(grid), dim3(kGrpThreads), smem, s, a);
  if (launches) *launches += 1;
}

void launch_grouped_down(const GrpArgs& a, int grid, size_t smem, cudaStream_t s,
                         uint64_t* launches) {
  launch_pdl(grp_down_kernel, dim3(grid), dim3(kGrpThreads), smem, s, a);
  if (launches) *launches += 1;
}
}  // namespace osm

#ifdef OSM_PHASE_TIMING
extern "C" int osm_dbg_timeline_gemv(unsigned long long* out) {
  unsigned long long init[OSM_TL_SLOTS];
  for (int i = 0; i < OSM_TL_SLOTS; ++i) init[i] = (i % 4 == 0) ? ~0ull : 0ull;
  cudaMemcpyFromSymbol(out, osm::g_tl, sizeof(init));
  return (int)cudaMemcpyToSymbol(osm::g_tl, init, sizeof(init));
}
extern "C" int osm_dbg_cycles_grouped(long long* out) {
  return (int)cudaMemcpyFromSymbol(out, osm::g_gcyc, 128 * sizeof(long long));
}
extern "C" int osm_dbg_cycles_gemv(long long* out) {
  return (int)cudaMemcpyFromSymbol(out, osm::g_cyc, 64 * sizeof(long long));
}
#endif

namespace osm {
cudaError_t set_first_wait_polls_gemv(uint32_t polls) { return set_first_wait_polls(polls); }
}  // namespace osm
