// osm_router.cu -- the Qwen router on sm_100a (replaces route_qwen_top_k_cpu,
// src/model/qwen_router.cpp:11-94, and the host grouping of
// src/model/routed_moe.cpp:320-370).
//
// router_logits_kernel<EXP, TOKS>
//   fp32 logits on CUDA cores.  Lane l of a warp owns the contiguous chunk
//   [l*c, (l+1)*c) of the hidden dimension (weights stored in that order, see
//   osm_kernels.cuh), so each logit comes with a rigorous bound on its distance
//   to the reference's sequential fp32 sum (reference_ops.cpp:85-91): the
//   running-error bound u * sum_i |s_i| of the sequential order, whose partial
//   sums s_i are bounded by the chunk prefix |P_l| plus the in-chunk partials,
//   plus the error of this kernel's own order.
// router_select_kernel (one block per token)
//   1. top-(k+1) by (logit desc, id asc) with redux.sync; certified when every
//      adjacent gap exceeds twice the largest bound plus a floor that keeps
//      distinct logits at distinct probabilities;
//   2. otherwise the candidates within twice the bound of the k-th logit get
//      their logits recomputed exactly as the reference does (sequential fp32,
//      rows staged in shared memory) and are ordered by them;
//   3. if exact logits are themselves (near) equal, the whole token is routed
//      by the reference's arithmetic: all logits sequential, softmax with a
//      sequential sum, stable top-k (reference_ops.cpp:130-212).
//   Then the shared-expert scalar gate, the activation fragments and, in the
//   last block, the grouping of (token, pick) pairs by expert.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "osm_common.cuh"
#include "osm_kernels.cuh"

#ifdef OSM_PHASE_TIMING
#include <cstdio>
#define OSM_STAMP(i) do { if (threadIdx.x == 0 || threadIdx.x == 32) { ts_[(i)] = clock64(); if ((i) == 0) gt0_ = gtime(); } } while (0)
#else
#define OSM_STAMP(i) do { } while (0)
#endif

namespace osm {
namespace {
#ifdef OSM_PHASE_TIMING
__device__ unsigned long long g_tl[OSM_TL_SLOTS];
__device__ long long g_rcyc[16];
__device__ long long g_gts[12];
#define GRP_STAMP(i) do { if (threadIdx.x == 0) g_gts[(i)] = clock64(); } while (0)
#else
#define GRP_STAMP(i) do { } while (0)
#endif

constexpr float kU = 5.9604644775390625e-8f;  // 2^-24
constexpr int kLogitWarps = 4;
constexpr int kMaxVec = 8;                    // H <= 2048 on the register path
constexpr int kSelThreads = 512;
constexpr int kMaxCand = 16;                  // candidates of the partial exact path
constexpr int kPartChunk = 512;               // h staged at a time on the partial exact path
constexpr int kFullTile = 16;                 // h per tile on the full exact path

__device__ __forceinline__ void unpack8(const uint4 q, float w[8]) {
  const uint32_t ww[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int jj = 0; jj < 8; ++jj) w[jj] = bf16_bits_to_f32((ww[jj >> 1] >> ((jj & 1) * 16)) & 0xFFFFu);
}

// Eight 8-bit affine weights: fl(fl(scale * q) + bias) each, the operation
// order of cpu::dequantize_affine_rows (reference_ops.cpp:11-67).
__device__ __forceinline__ void deq8(uint2 q, uint32_t meta, float w[8]) {
  const float sc = bf16_bits_to_f32(meta & 0xFFFFu), bi = bf16_bits_to_f32(meta >> 16);
  const uint32_t qq[2] = {q.x, q.y};
#pragma unroll
  for (int jj = 0; jj < 8; ++jj)
    w[jj] = __fadd_rn(__fmul_rn(sc, (float)((qq[jj >> 2] >> (8 * (jj & 3))) & 0xFFu)), bi);
}

// Eight consecutive weights of vector (e, m, lane) of the router layout.
__device__ __forceinline__ void load8(const RouterArgs& a, int e, int m, int lane, float w[8]) {
  const size_t v = ((size_t)e * a.g.nvec + m) * 32 + lane;
  if (a.g.q8) {
    const int h = lane * a.g.c + 8 * m;  // the vector's first h: one 64-group
    deq8(__ldg(reinterpret_cast<const uint2*>(a.wp) + v),
         __ldg(a.qmeta + (size_t)e * (a.g.H >> 6) + (h >> 6)), w);
    return;
  }
  if (a.g.f32w) {
    const float4* p = reinterpret_cast<const float4*>(a.wp) + 2 * v;
    const float4 x0 = __ldg(p), x1 = __ldg(p + 1);
    w[0] = x0.x; w[1] = x0.y; w[2] = x0.z; w[3] = x0.w;
    w[4] = x1.x; w[5] = x1.y; w[6] = x1.z; w[7] = x1.w;
  } else {
    unpack8(__ldg(a.wp + v), w);
  }
}

// ----------------------------------------------------------------------------
// exact logits (3+ tokens)
//
// router_exact_kernel<TT, F32>: every (token, expert) logit by the
// reference's own arithmetic -- a sequential fp32 sum over h = 0..H-1 of
// separately rounded products (matvec_row_major, reference_ops.cpp:85-91),
// then the bias -- so the selection needs no error bound (bounds are 0).  A
// block owns 128 experts (one per thread) and TT tokens.  The experts' router
// rows stream through a ring of 16 KB tiles (128 rows x 128 bytes, one bulk
// copy each, started before the wait on the predecessor since the weights
// never change); the row-swizzled chunks make each thread's 16-byte row reads
// conflict-free.  The tokens' x[h] come from shared memory, and the TT sums
// advance two at a time with packed f32x2 multiplies and adds (each lane
// rounded like a scalar mul.rn / add.rn).
// ----------------------------------------------------------------------------
constexpr int kExThreads = 128;
constexpr int kExStages = 4;
constexpr int kExTile = 16384;

__device__ __forceinline__ float2 fmul2_rn(float2 a, float2 b) {
  float2 r;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " mul.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}\n"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
__device__ __forceinline__ float2 fadd2_rn(float2 a, float2 b) {
  float2 r;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " add.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}\n"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}

// STG: stages of the router-tile ring (fewer for more tokens per thread, so
// that two blocks still fit an SM)
template <int TT, bool F32, int STG = kExStages>
__global__ void __launch_bounds__(kExThreads) router_exact_kernel(RouterArgs a) {
  constexpr int EPC = F32 ? 4 : 8;  // weights per 16-byte chunk
  constexpr int HPT = 8 * EPC;      // h per tile
  extern __shared__ __align__(128) unsigned char exsm[];
  __shared__ __align__(8) uint64_t full[STG];
  unsigned char* ring = exsm;
  float* xs = reinterpret_cast<float*>(exsm + STG * kExTile);  // [H][TT]
  const int E = a.g.E, H = a.g.H, nht = H / HPT;
  const int tid = threadIdx.x, e = blockIdx.x * kExThreads + tid, t0 = blockIdx.y * TT;
  const unsigned char* src = static_cast<const unsigned char*>(a.wx) + (size_t)blockIdx.x * nht * kExTile;
  TL_START(0);
  if (tid == 0) {
    for (int s = 0; s < STG; ++s) mbar_init(&full[s], 1);
    mbar_init_fence();
    for (int s = 0; s < STG && s < nht; ++s) {
      mbar_arrive_expect(&full[s], kExTile);
      bulk_load(ring + s * kExTile, src + (size_t)s * kExTile, kExTile, &full[s]);
    }
  }
  pdl_wait();
  TL_WAITED(0);
  for (int i = tid; i < TT * H; i += kExThreads) {
    const int t = i / H, h = i - t * H;
    xs[h * TT + t] = t0 + t < a.B ? a.x[(size_t)(t0 + t) * H + h] : 0.0f;
  }
  __syncthreads();
  pdl_trigger();
  float acc[TT];
#pragma unroll
  for (int t = 0; t < TT; ++t) acc[t] = 0.0f;
  const int sw = tid & 7;
  for (int j = 0; j < nht; ++j) {
    const int s = j % STG;
    const uint32_t par = (uint32_t)(j / STG) & 1u;
    if (!mbar_wait_first(&full[s], par)) {
      if (tid == 0) atomicOr(a.status, kStatusCopyTimeout);
      mbar_wait(&full[s], par);  // the copy may still land: wait once more
    }
    const uint4* row = reinterpret_cast<const uint4*>(ring + s * kExTile + tid * 128);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 q = row[c ^ sw];
      const int h0 = j * HPT + c * EPC;
      float w[EPC];
      if constexpr (F32) {
        w[0] = __uint_as_float(q.x); w[1] = __uint_as_float(q.y);
        w[2] = __uint_as_float(q.z); w[EPC - 1] = __uint_as_float(q.w);
      } else {
        const uint32_t qq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          w[2 * jj] = __uint_as_float(qq[jj] << 16);
          w[2 * jj + 1] = __uint_as_float(qq[jj] & 0xFFFF0000u);
        }
      }
      if constexpr (TT == 1) {
        float xv[EPC];
#pragma unroll
        for (int u = 0; u < EPC; u += 4) {
          const float4 x4 = reinterpret_cast<const float4*>(xs + h0)[u >> 2];
          xv[u] = x4.x; xv[u + 1] = x4.y; xv[u + 2] = x4.z; xv[u + 3] = x4.w;
        }
#pragma unroll
        for (int jj = 0; jj < EPC; ++jj) acc[0] = __fadd_rn(acc[0], __fmul_rn(w[jj], xv[jj]));
      } else {
#pragma unroll
        for (int jj = 0; jj < EPC; ++jj) {
          const float2* xp = reinterpret_cast<const float2*>(xs + (size_t)(h0 + jj) * TT);
#pragma unroll
          for (int t = 0; t < TT; t += 2) {
            const float2 p2 = fmul2_rn(make_float2(w[jj], w[jj]), xp[t >> 1]);
            const float2 s2 = fadd2_rn(make_float2(acc[t], acc[t + 1]), p2);
            acc[t] = s2.x;
            acc[t + 1] = s2.y;
          }
        }
      }
    }
    __syncthreads();  // every thread is done with stage s
    if (tid == 0 && j + STG < nht) {
      mbar_arrive_expect(&full[s], kExTile);
      bulk_load(ring + s * kExTile, src + (size_t)(j + STG) * kExTile, kExTile, &full[s]);
    }
  }
  if (e < E) {
    const float bias = a.bias != nullptr ? a.bias[e] : 0.0f;
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      if (t0 + t < a.B) {
        const float v = a.bias != nullptr ? __fadd_rn(acc[t], bias) : acc[t];
        a.logits[(size_t)(t0 + t) * E + e] = v;
        a.bounds[(size_t)(t0 + t) * E + e] = 0.0f;
      }
    }
  }
  TL_END(0);
}

// router_exact2_kernel<TT, FMT, STG, NW>: the same sums as
// router_exact_kernel (one thread per expert and TT tokens, h in order), with
// the tokens' x streamed beside the router rows instead of staged whole.  A
// block owns 32 * NW experts (NW consumer warps; the rows of 32 NW experts
// are one contiguous quarter, half or whole of a 16 KB router tile) and TT
// tokens; each ring stage holds those rows of one tile and the matching HPT
// values of each of the TT rows of x ([t][h], TT bulk copies), filled by a
// producer warp behind full/empty mbarriers.  Small batches take one warp of
// experts per block and one token per thread, so that the 2 * H dependent
// operations of each sum run on as many SMs as possible.  FMT: router
// weights as bf16 (0), fp32 (1) or 8-bit affine (2, dequantised in the
// reference's operation order as they are read).  Needs x 16-byte aligned and
// H a multiple of HPT.
template <int TT, int FMT, int STG, int NW>
__global__ void __launch_bounds__(NW * 32 + 32) router_exact2_kernel(RouterArgs a) {
  constexpr int EPC = FMT == 1 ? 4 : FMT == 0 ? 8 : 16;  // weights per 16-byte chunk
  constexpr int HPT = 8 * EPC;       // h per tile
  constexpr int EXPB = 32 * NW;      // experts per block
  constexpr int WB = EXPB * 128;     // router bytes per stage
  constexpr int XB = TT * HPT * 4;   // x bytes per stage
  constexpr int SB = WB + XB;        // stage bytes
  constexpr int kEx2Consumers = NW;
  extern __shared__ __align__(128) unsigned char exsm[];
  __shared__ __align__(8) uint64_t full[STG], empty[STG];
  const int E = a.g.E, H = a.g.H, nht = H / HPT;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = blockIdx.y * TT;
  const int nt = min(TT, a.B - t0);  // rows of x this block copies
  const int e0 = blockIdx.x * EXPB;
  const unsigned char* src = static_cast<const unsigned char*>(a.wx) +
                             (size_t)(e0 / kExThreads) * nht * kExTile + (size_t)(e0 % kExThreads) * 128;
  TL_START(0);
  if (tid == 0) {
    for (int st = 0; st < STG; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], kEx2Consumers);
    }
    mbar_init_fence();
  }
  __syncthreads();
  if (warp == kEx2Consumers) {
    // ---- producer: router tiles (immutable) may go before the PDL wait;
    //      x segments after it ----
    if (lane == 0) {
      for (int st = 0; st < STG && st < nht; ++st) {
        mbar_arrive_expect(&full[st], (uint32_t)(WB + nt * HPT * 4));
        bulk_load(exsm + st * SB, src + (size_t)st * kExTile, WB, &full[st]);
      }
    }
    pdl_wait();
    if (lane == 0) {
      int issued = min(STG, nht);  // stages whose router tile is on its way
      for (int j = 0; j < nht; ++j) {
        const int st = j % STG;
        if (j >= STG) {
          if (!mbar_wait(&empty[st], (uint32_t)((j / STG) - 1) & 1u)) {
            atomicOr(a.status, kStatusCopyTimeout);
            break;
          }
          issued = j + 1;
          mbar_arrive_expect(&full[st], (uint32_t)(WB + nt * HPT * 4));
          bulk_load(exsm + st * SB, src + (size_t)j * kExTile, WB, &full[st]);
        }
        for (int t = 0; t < nt; ++t)
          bulk_load(exsm + st * SB + WB + t * HPT * 4, a.x + (size_t)(t0 + t) * H + (size_t)j * HPT,
                    HPT * 4, &full[st]);
      }
      // copies of the last stages may still be landing: wait for them
      for (int j = max(0, issued - STG); j < issued; ++j)
        mbar_wait(&full[j % STG], (uint32_t)(j / STG) & 1u);
    }
    __syncwarp();
    return;
  }
  const int e = e0 + tid;
  float acc[TT];
#pragma unroll
  for (int t = 0; t < TT; ++t) acc[t] = 0.0f;
  const int sw = tid & 7;
  for (int j = 0; j < nht; ++j) {
    const int st = j % STG;
    const uint32_t par = (uint32_t)(j / STG) & 1u;
    if (!mbar_wait_first(&full[st], par)) {
      if (tid == 0) atomicOr(a.status, kStatusCopyTimeout);
      mbar_wait(&full[st], par);  // the copies may still land: wait once more
    }
    // the select kernel may launch once x has been read here: its first
    // stage's x copies were issued after the producer's dependency wait, so
    // the select can stage x itself before its own wait
    if (j == 0) pdl_trigger();
    const uint4* row = reinterpret_cast<const uint4*>(exsm + st * SB + tid * 128);
    const float4* xt = reinterpret_cast<const float4*>(exsm + st * SB + WB);  // [TT][HPT]
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 q = row[c ^ sw];
      float w[EPC];
      if constexpr (FMT == 2) {
        const uint32_t meta =
            __ldg(a.qmeta + (size_t)min(e, E - 1) * (H >> 6) + ((j * HPT + c * EPC) >> 6));
        deq8(make_uint2(q.x, q.y), meta, w);
        deq8(make_uint2(q.z, q.w), meta, w + 8);
      } else if constexpr (FMT == 1) {
        w[0] = __uint_as_float(q.x); w[1] = __uint_as_float(q.y);
        w[2] = __uint_as_float(q.z); w[EPC - 1] = __uint_as_float(q.w);
      } else {
        const uint32_t qq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          w[2 * jj] = __uint_as_float(qq[jj] << 16);
          w[2 * jj + 1] = __uint_as_float(qq[jj] & 0xFFFF0000u);
        }
      }
      // four values of h at a time: x of the TT tokens there (broadcast
      // reads), then the TT sums advance over them in h order
#pragma unroll
      for (int u = 0; u < EPC; u += 4) {
        float xv[TT][4];
#pragma unroll
        for (int t = 0; t < TT; ++t) {
          const float4 x4 = xt[t * (HPT / 4) + c * (EPC / 4) + (u >> 2)];
          xv[t][0] = x4.x; xv[t][1] = x4.y; xv[t][2] = x4.z; xv[t][3] = x4.w;
        }
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const float wj = w[u + jj];
          if constexpr (TT == 1) {
            acc[0] = __fadd_rn(acc[0], __fmul_rn(wj, xv[0][jj]));
          } else {
#pragma unroll
            for (int t = 0; t < TT; t += 2) {
              const float2 p2 = fmul2_rn(make_float2(wj, wj), make_float2(xv[t][jj], xv[t + 1][jj]));
              const float2 s2 = fadd2_rn(make_float2(acc[t], acc[t + 1]), p2);
              acc[t] = s2.x;
              acc[t + 1] = s2.y;
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
  if (e < E) {
    const float bias = a.bias != nullptr ? a.bias[e] : 0.0f;
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      if (t0 + t < a.B) {
        const float v = a.bias != nullptr ? __fadd_rn(acc[t], bias) : acc[t];
        a.logits[(size_t)(t0 + t) * E + e] = v;
        a.bounds[(size_t)(t0 + t) * E + e] = 0.0f;
      }
    }
  }
  TL_END(0);
}

// ----------------------------------------------------------------------------
// logits
// ----------------------------------------------------------------------------
template <int EXP, int TOKS>
__global__ void __launch_bounds__(kLogitWarps * 32) router_logits_kernel(RouterArgs a) {
  extern __shared__ float4 smem4[];
  const RouterGeom g = a.g;
  const int cp = g.c + 4;  // padded lane chunk: conflict-free float4 reads
  float* xs = reinterpret_cast<float*>(smem4);  // [TOKS][32][cp]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e0 = (blockIdx.x * kLogitWarps + warp) * EXP;
  const bool reg_path = !g.f32w && !g.q8 && g.nvec <= kMaxVec;
#ifdef OSM_PHASE_TIMING
  const unsigned long long lg0 = gtime();
#endif
  TL_START(0);
  // The weights are immutable: fetch them before waiting on the predecessor.
  uint4 wv[EXP][kMaxVec];
#pragma unroll
  for (int q = 0; q < EXP; ++q)
#pragma unroll
    for (int m = 0; m < kMaxVec; ++m) {
      wv[q][m] = make_uint4(0u, 0u, 0u, 0u);
      if (reg_path && m < g.nvec && e0 + q < g.E)
        wv[q][m] = __ldg(a.wp + ((size_t)(e0 + q) * g.nvec + m) * 32 + lane);
    }
  pdl_wait();
  TL_WAITED(0);
  const int t0 = blockIdx.y * TOKS;
  const int nv4 = g.Hp >> 2;
  const bool vec_ok = (g.H & 3) == 0;
#pragma unroll 4
  for (int i = threadIdx.x; i < TOKS * nv4; i += blockDim.x) {
    const int t = i / nv4, h = (i - t * nv4) * 4;
    float4 val = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (t0 + t < a.B && h < g.H) {
      const float* src = a.x + (size_t)(t0 + t) * g.H + h;
      if (vec_ok) {
        val = *reinterpret_cast<const float4*>(src);
      } else {
        val.x = src[0];
        if (h + 1 < g.H) val.y = src[1];
        if (h + 2 < g.H) val.z = src[2];
        if (h + 3 < g.H) val.w = src[3];
      }
    }
    const int l = h / g.c, o = h - l * g.c;
    *reinterpret_cast<float4*>(xs + (t * 32 + l) * cp + o) = val;
  }
  __syncthreads();
  pdl_trigger();
  if (e0 >= g.E) {
    TL_END(0);
    return;
  }
  float tacc[EXP][TOKS], aacc[EXP][TOKS], sacc[EXP][TOKS];
#pragma unroll
  for (int q = 0; q < EXP; ++q)
#pragma unroll
    for (int t = 0; t < TOKS; ++t) tacc[q][t] = aacc[q][t] = sacc[q][t] = 0.0f;
  auto step = [&](int m, const float (&w)[EXP][8]) {
#pragma unroll
    for (int t = 0; t < TOKS; ++t) {
      const float4* xp = reinterpret_cast<const float4*>(xs + (t * 32 + lane) * cp + 8 * m);
      const float4 xa = xp[0], xb = xp[1];
      const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
      for (int q = 0; q < EXP; ++q) {
        // |partial sum| at the start of this 8-element block: the partial
        // sums inside the block are bounded by it plus the block's |w x|.
        sacc[q][t] += fabsf(tacc[q][t]);
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          tacc[q][t] = fmaf(w[q][jj], xv[jj], tacc[q][t]);
          aacc[q][t] = fmaf(fabsf(w[q][jj]), fabsf(xv[jj]), aacc[q][t]);
        }
      }
    }
  };
  if (reg_path) {
#pragma unroll
    for (int m = 0; m < kMaxVec; ++m) {
      if (m < g.nvec) {
        float w[EXP][8];
#pragma unroll
        for (int q = 0; q < EXP; ++q) unpack8(wv[q][m], w[q]);
        step(m, w);
      }
    }
  } else {
    for (int m = 0; m < g.nvec; ++m) {
      float w[EXP][8];
#pragma unroll
      for (int q = 0; q < EXP; ++q) {
        if (e0 + q < g.E) {
          load8(a, e0 + q, m, lane, w[q]);
        } else {
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) w[q][jj] = 0.0f;
        }
      }
      step(m, w);
    }
  }
  const float n = (float)g.Hp;
  const float gam = n * kU / (1.0f - n * kU);
#pragma unroll
  for (int q = 0; q < EXP; ++q) {
#pragma unroll
    for (int t = 0; t < TOKS; ++t) {
      const float T = tacc[q][t];
      float incl = T;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += y;
      }
      float P = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
      if (lane == 0) P = 0.0f;
      const float logit = warp_sum(T);
      const float Q = warp_sum(fabsf(T));
      const float S = warp_sum(8.0f * (sacc[q][t] + aacc[q][t]));
      const float Pa = warp_sum(fabsf(P));
      const float A = warp_sum(aacc[q][t]);
      float bound = 1.001f * kU *
                    ((float)g.c * Pa + 2.0f * S + 5.0f * Q + A * (1.0f + 3.0f * n * gam));
      float outl = logit;
      const int e = e0 + q;
      if (a.bias != nullptr && e < g.E) {
        outl = __fadd_rn(logit, a.bias[e]);
        bound = bound + 2.002f * kU * (fabsf(outl) + bound);
      }
      if (lane == 0 && e < g.E && t0 + t < a.B) {
        a.logits[(size_t)(t0 + t) * g.E + e] = outl;
        a.bounds[(size_t)(t0 + t) * g.E + e] = bound;
      }
    }
  }
  TL_END(0);
#ifdef OSM_PHASE_PRINT
  if (threadIdx.x == 0 && (blockIdx.x == 0 || blockIdx.x == 7) && blockIdx.y == 0)
    printf("logits cta %d: g %llu..%llu\n", (int)blockIdx.x, lg0, gtime());
#endif
}

// ----------------------------------------------------------------------------
// selection
// ----------------------------------------------------------------------------
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// Best n (<= number of valid entries) of the lane-strided values v[i]
// (index i*32 + lane, valid when < E) by (value desc, index asc).  Keys are
// 64-bit: order key of the value, then the complement of the index.  Each lane
// sorts its NV keys with a bitonic network (independent compare-swaps), then
// n merge rounds take the warp maximum of the lane heads with a shuffle
// butterfly; the winning lane shifts its sorted keys by one.  Lane 0 writes
// sel_id / sel_v.
template <int NV>
__device__ __forceinline__ void warp_select_n(const float (&v)[32], int E, int n, int* sel_id,
                                              float* sel_v) {
  const int lane = threadIdx.x & 31;
  unsigned long long key[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int id = i * 32 + lane;
    key[i] = id < E ? (((unsigned long long)ord_key(v[i]) << 32) | (0xFFFFFFFFu - (uint32_t)id))
                    : 0ull;
  }
#pragma unroll
  for (int kk = 2; kk <= NV; kk <<= 1) {
#pragma unroll
    for (int jj = kk >> 1; jj > 0; jj >>= 1) {
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int l = i ^ jj;
        if (l > i) {
          const bool desc = (i & kk) == 0;
          const unsigned long long a = key[i], b = key[l];
          const bool sw = desc ? (a < b) : (a > b);
          key[i] = sw ? b : a;
          key[l] = sw ? a : b;
        }
      }
    }
  }
  for (int r = 0; r < n; ++r) {
    unsigned long long m = key[0];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, m, o);
      if (other > m) m = other;
    }
    const int win = (int)(0xFFFFFFFFu - (uint32_t)(m & 0xFFFFFFFFull));
    const uint32_t kk32 = (uint32_t)(m >> 32);
    const uint32_t u = (kk32 & 0x80000000u) ? (kk32 & 0x7FFFFFFFu) : ~kk32;
    if (lane == 0) {
      sel_id[r] = win;
      sel_v[r] = __uint_as_float(u);
    }
    if ((win & 31) == lane) {
#pragma unroll
      for (int i = 0; i + 1 < NV; ++i) key[i] = key[i + 1];
      key[NV - 1] = 0ull;
    }
  }
  __syncwarp();
}

__device__ __forceinline__ void warp_select(const float (&v)[32], int E, int n, int* sel_id,
                                            float* sel_v) {
  if (E <= 512) warp_select_n<16>(v, E, n, sel_id, sel_v);
  else warp_select_n<32>(v, E, n, sel_id, sel_v);
}

// Block-wide exclusive scan of n (<= 4*blockDim) ints in smem `v`, in place;
// returns the total.  `red` holds 32 ints.
__device__ int block_exclusive_scan(int* v, int n, int* red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int C = (n + blockDim.x - 1) / blockDim.x;
  const int i0 = tid * C;
  int loc[4];
  int s = 0;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    loc[q] = (q < C && i0 + q < n) ? v[i0 + q] : 0;
    s += loc[q];
  }
  int incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  __syncthreads();
  if (lane == 31) red[warp] = incl;
  __syncthreads();
  int base = 0;
  for (int w = 0; w < warp; ++w) base += red[w];
  int total = 0;
  const int nw = blockDim.x >> 5;
  for (int w = 0; w < nw; ++w) total += red[w];
  int run = base + incl - s;
  __syncthreads();
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (q < C && i0 + q < n) v[i0 + q] = run;
    run += loc[q];
  }
  __syncthreads();
  return total;
}

// Exclusive scan of n ints in smem by warp 0 (each lane a run of ceil(n/32)
// consecutive values, one shuffle scan over the lanes' sums); a block-wide
// scan beyond 1024 values.  The caller has synchronised after writing v.
// Returns the total.
__device__ int small_or_block_scan(int* v, int n, int* red) {
  if (n > 1024) return block_exclusive_scan(v, n, red);
  __shared__ int s_tot;
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const int per = (n + 31) >> 5;
    const int i0 = lane * per;
    const int i1 = min(n, i0 + per);
    int sum = 0;
    for (int i = i0; i < i1; ++i) sum += v[i];
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    int run = incl - sum;
    for (int i = i0; i < i1; ++i) {
      const int x = v[i];
      v[i] = run;
      run += x;
    }
    if (lane == 31) s_tot = incl;
  }
  __syncthreads();
  return s_tot;
}

// Group (token, pick) pairs by expert.  The shared expert (id E) is active
// index 0 when present, so later kernels can fetch its weights early.  The
// order of the other experts and of tokens inside an expert is arbitrary:
// every token's result is computed independently of its position.
__device__ void group_pairs(const RouterArgs& a, int* sm, int* red) {
  const int E = a.g.E, k = a.g.k, B = a.B;
  const int has_sh = a.shared_slot != nullptr;
  const int NE = E + has_sh;
  int* cnt = sm;
  int* actidx = sm + NE;
  int* cur = sm + 2 * NE;
  int* expert_of = sm + 3 * NE;
  int* off = sm + 4 * NE;
  __shared__ int s_nact;
  GRP_STAMP(0);
  for (int i = threadIdx.x; i < NE; i += blockDim.x) {
    cnt[i] = 0;
    cur[i] = 0;
    actidx[i] = -1;
  }
  if (threadIdx.x == 0) s_nact = has_sh;
  __syncthreads();
  if (has_sh && threadIdx.x == 0) {
    actidx[E] = 0;
    cnt[E] = B;
  }
  // picks are read eight per thread ahead of their atomics
  for (int p0 = threadIdx.x; p0 < B * k; p0 += 8 * blockDim.x) {
    uint32_t ev[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int p = p0 + u * blockDim.x;
      ev[u] = p < B * k ? __ldcg(a.ids + p) : 0xFFFFFFFFu;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (p0 + u * (int)blockDim.x >= B * k) break;
      const uint32_t e = ev[u];
      if (e >= (uint32_t)E) {
        if (e != kEpEmpty) atomicOr(a.status, kStatusBadSlot);  // kEpEmpty: an empty slot
        continue;
      }
      if (atomicAdd(&cnt[e], 1) == 0) actidx[e] = atomicAdd(&s_nact, 1);
    }
  }
  __syncthreads();
  GRP_STAMP(1);
  const int n_active = s_nact;
  for (int e = threadIdx.x; e < NE; e += blockDim.x)
    if (actidx[e] >= 0) expert_of[actidx[e]] = e;
  __syncthreads();
  for (int j = threadIdx.x; j < n_active; j += blockDim.x) off[j] = cnt[expert_of[j]];
  __syncthreads();
  small_or_block_scan(off, n_active, red);
  // token groups per active expert (cur[] is free until the scatter)
  for (int j = threadIdx.x; j < n_active; j += blockDim.x)
    cur[j] = (cnt[expert_of[j]] + kTokGroup - 1) / kTokGroup;
  __syncthreads();
  const int n_tg = small_or_block_scan(cur, n_active, red);
  GRP_STAMP(2);
  for (int j = threadIdx.x; j < n_active; j += blockDim.x) {
    const int e = expert_of[j];
    ActEntry en;
    en.off = off[j];
    en.cnt = cnt[e];
    en.tg0 = cur[j];
    en.pad0 = en.pad1 = 0;
    if (e == E) {
      en.kind = 1;
      en.ptr = a.shared_slot;
    } else {
      en.kind = 0;
      const int slot = a.slot_of[e];
      if (slot < 0) {
        atomicOr(a.status, kStatusNotResident);
        en.ptr = nullptr;
      } else {
        en.ptr = a.slab + (size_t)slot * a.slab_stride;
      }
    }
    a.act[j] = en;
    const int ng = (en.cnt + kTokGroup - 1) / kTokGroup;
    for (int q = 0; q < ng; ++q) {
      a.tg_expert[en.tg0 + q] = j;
      a.tg_begin[en.tg0 + q] = q * kTokGroup;
    }
  }
  __syncthreads();
  GRP_STAMP(3);
  if (a.chunks) {
    // chunks of chunk_pairs pairs of each active entry, in entry order
    const int cp = a.chunk_pairs > 0 ? a.chunk_pairs : 8;
    for (int j = threadIdx.x; j < n_active; j += blockDim.x)
      cur[j] = (cnt[expert_of[j]] + cp - 1) / cp;
    __syncthreads();
    const int n_ch = small_or_block_scan(cur, n_active, red);
    for (int j = threadIdx.x; j < n_active; j += blockDim.x) {
      const int nc = (cnt[expert_of[j]] + cp - 1) / cp;
      for (int q = 0; q < nc; ++q) a.chunks[cur[j] + q] = make_int2(j, cp * q);
    }
    if (threadIdx.x == 0) *a.n_ch = n_ch;
    __syncthreads();
  }
  GRP_STAMP(4);
  if (a.defer_scatter) {
    // many pairs: each expert's first position and a zero cursor for
    // scatter_pairs_kernel, which places the pairs across the whole GPU
    for (int e = threadIdx.x; e < NE; e += blockDim.x) {
      a.counts[e] = actidx[e] >= 0 ? off[actidx[e]] : 0;
      a.cursor[e] = 0;
    }
  } else {
    for (int i = threadIdx.x; i < NE; i += blockDim.x) cur[i] = 0;
    __syncthreads();
    for (int p0 = threadIdx.x; p0 < B * k; p0 += 8 * blockDim.x) {
      uint32_t ev[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int p = p0 + u * blockDim.x;
        ev[u] = p < B * k ? __ldcg(a.ids + p) : 0xFFFFFFFFu;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int p = p0 + u * blockDim.x;
        if (p >= B * k) break;
        const uint32_t e = ev[u];
        if (e >= (uint32_t)E) continue;
        const int pos = off[actidx[e]] + atomicAdd(&cur[e], 1);
        a.pair_tok[pos] = p / k;
        a.pair_pick[pos] = p % k;
        if (a.tp_pos) a.tp_pos[(p / k) * (k + has_sh) + p % k] = pos;
      }
    }
    if (has_sh)
      for (int t = threadIdx.x; t < B; t += blockDim.x) {
        a.pair_tok[off[0] + t] = t;
        a.pair_pick[off[0] + t] = k;
        if (a.tp_pos) a.tp_pos[t * (k + 1) + k] = off[0] + t;
      }
  }
  GRP_STAMP(5);
  if (threadIdx.x == 0) {
    *a.n_active = n_active;
    *a.n_tg = n_tg;
  }
}

// Softmax weights of the picks from logits lsel[0..k) (lsel[0] the largest)
// with the sum over the fast logits v[] (lane-strided); lane j handles pick j.
// Slot base of expert id (null, with a status bit, when the id is out of
// range or the expert is not resident).
__device__ __forceinline__ const uint8_t* slot_base(const RouterArgs& a, uint32_t id) {
  if (id >= (uint32_t)a.g.E) {
    atomicOr(a.status, kStatusBadSlot);
    return nullptr;
  }
  const int slot = a.slot_of[id];
  if (slot < 0) {
    atomicOr(a.status, kStatusNotResident);
    return nullptr;
  }
  return a.slab + (size_t)slot * a.slab_stride;
}

// Weights of the k picks (warp 0): p_j = exp(l_j - mx) / s, where s is the sum
// of exp(l_e - mx) over every expert, then renormalised over the picks.
__device__ __forceinline__ void write_weights(const RouterArgs& a, int tok, float s, float mx,
                                              const int* sid, const float* lsel) {
  const int lane = threadIdx.x & 31;
  const int k = a.g.k;
  const float p = lane < k ? __fdiv_rn(__expf(__fsub_rn(lsel[lane], mx)), s) : 0.0f;
  const float mass = warp_sum(p);
  if (lane == 0 && (!(mass > 0.0f) || !isfinite(mass) || !(s > 0.0f) || !isfinite(s)))
    atomicOr(a.status, kStatusBadMass);
  if (lane < k) {
    const float wv = a.norm ? __fdiv_rn(p, mass) : p;
    a.ids[(size_t)tok * k + lane] = (uint32_t)sid[lane];
    a.weights[(size_t)tok * k + lane] = wv;
    if (a.ids_out) a.ids_out[(size_t)tok * k + lane] = (uint32_t)sid[lane];
    if (a.weights_out) a.weights_out[(size_t)tok * k + lane] = wv;
    if (a.pick_ptr) a.pick_ptr[(size_t)tok * k + lane] = slot_base(a, (uint32_t)sid[lane]);
  }
  if (lane == 0) {
    a.mass[tok] = mass;
    if (a.mass_out) a.mass_out[tok] = mass;
  }
}

// Sorts one key per lane across the warp, largest first (bitonic network).
__device__ __forceinline__ unsigned long long warp_sort_desc(unsigned long long key) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, key, stride);
      const bool lower = (lane & stride) == 0;
      const bool take_max = lower == ((lane & size) == 0 || size == 32);
      key = take_max ? (other > key ? other : key) : (other < key ? other : key);
    }
  }
  return key;
}

// Top 32 of two descending lists held one key per lane: a, and b read in
// reverse (b_rev[lane] = b[31 - lane]).  max(a, b_rev) holds the 32 largest
// keys as a bitonic sequence; a half-cleaner cascade sorts it descending.
__device__ __forceinline__ unsigned long long merge_top(unsigned long long a,
                                                        unsigned long long b_rev) {
  const int lane = threadIdx.x & 31;
  unsigned long long c = a > b_rev ? a : b_rev;
#pragma unroll
  for (int stride = 16; stride > 0; stride >>= 1) {
    const unsigned long long o = __shfl_xor_sync(0xFFFFFFFFu, c, stride);
    const bool lower = (lane & stride) == 0;
    c = lower ? (o > c ? o : c) : (o < c ? o : c);
  }
  return c;
}

__device__ __forceinline__ unsigned long long sel_key(float v, int id) {
  return ((unsigned long long)ord_key(v) << 32) | (0xFFFFFFFFu - (uint32_t)id);
}
__device__ __forceinline__ int key_id(unsigned long long key) {
  return (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
}
__device__ __forceinline__ float key_value(unsigned long long key) {
  const uint32_t kk32 = (uint32_t)(key >> 32);
  return __uint_as_float((kk32 & 0x80000000u) ? (kk32 & 0x7FFFFFFFu) : ~kk32);
}

// True when consecutive (exact) logits are far enough apart that their
// probabilities cannot round to the same value.
__device__ __forceinline__ bool distinct_p(float hi, float lo, float mx) {
  return __fsub_rd(hi, lo) > 1e-6f + 3e-7f * (fabsf(hi - mx) + fabsf(lo - mx));
}

template <int TPB>
__global__ void __launch_bounds__(TPB, 1024 / TPB) router_select_kernel(RouterArgs a) {
  extern __shared__ float4 smem4[];
  float* xs = reinterpret_cast<float*>(smem4);  // [H]
  char* uni = reinterpret_cast<char*>(xs + ((a.g.H + 3) & ~3));
  __shared__ float red[32];
  __shared__ int sel_id[kMaxTopK + 1];
  __shared__ float sel_v[kMaxTopK + 1];
  __shared__ int cand_id[kMaxCand];
  __shared__ float cand_l[kMaxCand];
  __shared__ int s_flag, s_ncand;
  __shared__ float s_bm, s_bcast, s_sum, s_mx;
  __shared__ float sg_part[TPB / 32];
  __shared__ float s_red2[TPB / 32];
  __shared__ unsigned long long s_top[TPB];
  const RouterGeom g = a.g;
  const int tok = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int k = g.k;
#ifdef OSM_PHASE_TIMING
  __shared__ long long ts_[16];
  __shared__ unsigned long long gt0_;
#endif
  OSM_STAMP(0);
  TL_START(1);
  // the shared gate row is immutable: fetch it before waiting
  constexpr int kSgRegs = 4;
  float sgw[kSgRegs];
#pragma unroll
  for (int j = 0; j < kSgRegs; ++j) {
    const int h = tid + j * TPB;
    sgw[j] = (a.sgate_w != nullptr && h < g.H) ? a.sgate_w[h] : 0.0f;
  }
  const float* x = a.x + (size_t)tok * g.H;
  int nonfinite = 0;
  auto stage_x = [&]() {
    if ((g.H & 3) == 0) {
      for (int i = tid; i < (g.H >> 2); i += blockDim.x) {
        const float4 v = reinterpret_cast<const float4*>(x)[i];
        reinterpret_cast<float4*>(xs)[i] = v;
        if (!isfinite(v.x) || !isfinite(v.y) || !isfinite(v.z) || !isfinite(v.w)) nonfinite = 1;
      }
    } else {
      for (int h = tid; h < g.H; h += blockDim.x) {
        const float v = x[h];
        xs[h] = v;
        if (!isfinite(v)) nonfinite = 1;
      }
    }
  };
  // Everything that needs only x: staging, the finiteness check, the fp16 /
  // fragment copies for the expert kernels and the shared expert's gate.
  auto prologue = [&]() {
    stage_x();
    if (tid == 0) {
      s_flag = 0;
      s_ncand = 0;
    }
    nonfinite = __syncthreads_or(nonfinite);
    if (a.xbf != nullptr) {  // fp16 copy of x for the prefill tensor-core path
      bool over = false;
      for (int h = tid; h < g.H; h += blockDim.x) {
        const float v = xs[h];
        over |= fabsf(v) >= 65504.0f;
        a.xbf[(size_t)tok * g.H + h] = __half_as_ushort(__float2half_rn(v));
      }
      if (over) atomicOr(a.status, kStatusF16Range);
    }
    if (nonfinite && tid == 0) atomicOr(a.status, kStatusNonFinite);
    // activation fragments of the tensor-core path
    if (a.xfrag != nullptr) {
      const int nch = g.H >> 3;
      for (int c = tid; c < nch; c += blockDim.x) {
        const float4 p = reinterpret_cast<const float4*>(xs)[2 * c];
        const float4 q = reinterpret_cast<const float4*>(xs)[2 * c + 1];
        const float xc[8] = {p.x, p.y, p.z, p.w, q.x, q.y, q.z, q.w};
        uint32_t hi[8], lo[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) split_bf16(xc[j], hi[j], lo[j]);
        float fs = xc[0];
#pragma unroll
        for (int j = 1; j < 8; ++j) fs = __fadd_rn(fs, xc[j]);
        uint4* dst = a.xfrag + ((size_t)tok * nch + c) * 2;
        dst[0] = make_uint4(pack2(hi[0], hi[4]), pack2(hi[1], hi[5]), pack2(hi[2], hi[6]),
                            pack2(hi[3], hi[7]));
        dst[1] = make_uint4(pack2(lo[0], lo[4]), pack2(lo[1], lo[5]), pack2(lo[2], lo[6]),
                            pack2(lo[3], lo[7]));
        a.xfsum8[(size_t)tok * nch + c] = fs;
      }
    }
    if (a.sgate_w != nullptr) {
      float d = 0.0f;
#pragma unroll
      for (int j = 0; j < kSgRegs; ++j) {
        const int h = tid + j * TPB;
        if (h < g.H) d = fmaf(sgw[j], xs[h], d);
      }
      for (int h = tid + kSgRegs * TPB; h < g.H; h += blockDim.x) d = fmaf(a.sgate_w[h], xs[h], d);
      d = warp_sum(d);
      if (lane == 0) sg_part[warp] = d;
    }
    __syncthreads();
    // ---- shared expert scalar gate ----
    if (tid == blockDim.x - 32) {
      if (a.sgate_w != nullptr) {
        float dot = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) dot += sg_part[w];
        const float sgv = ref_sigmoid(dot);
        a.sgate[tok] = sgv;
        if (a.sgate_out) a.sgate_out[tok] = sgv;
      } else {
        if (a.sgate) a.sgate[tok] = 0.0f;
        if (a.sgate_out) a.sgate_out[tok] = 0.0f;
      }
    }
  };
  // With routing, this grid follows the logits kernel, which waited for the
  // producer of x before it let this grid launch: x is complete, and the
  // prologue overlaps the logits (the scratch it writes is no longer read by
  // the previous call, whose kernels ended before the logits kernel waited).
  // Given routing (osm_moe_experts), x may come from the kernel just before:
  // the prologue runs after the wait.
  const bool early_x = !a.skip_route;
  if (early_x) prologue();
  pdl_wait();
  // the expert kernels may launch now: they stage their inputs and prefetch
  // the shared expert while this grid selects, then wait for it
  pdl_trigger();
  OSM_STAMP(1);
  TL_WAITED(1);
  if (!early_x) prologue();
  // this thread's experts: tid and tid + TPB (E <= 2 * TPB)
  float lv[2] = {-INFINITY, -INFINITY};
  float bmax = 0.0f;
  if (!a.skip_route) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int e = tid + r * TPB;
      if (e < g.E) {
        lv[r] = a.logits[(size_t)tok * g.E + e];
        bmax = fmaxf(bmax, a.bounds[(size_t)tok * g.E + e]);
      }
    }
  }
  OSM_STAMP(2);
  const bool route = !nonfinite && !a.skip_route;  // block-uniform
  const int nsel = k + 1 <= g.E ? k + 1 : k;
  const int nl = (g.E + 31) >> 5;  // lists of 32 experts
  // ---- 1. fast path: certified top-k over the fast logits.  Each warp sorts
  //      its 32 (or 2 x 32) keys; a tree of bitonic merges through shared
  //      memory leaves the top 32 of all experts in warp 0. ----
  unsigned long long top = 0ull;
  if (route) {
    const int e0 = warp * 32 + lane;
    top = warp_sort_desc(e0 < g.E ? sel_key(lv[0], e0) : 0ull);
    if (nl > TPB / 32) {  // E > 512: fold in the second list
      const int e1 = e0 + TPB;
      const unsigned long long k1 = warp_sort_desc(e1 < g.E ? sel_key(lv[1], e1) : 0ull);
      top = merge_top(top, __shfl_sync(0xFFFFFFFFu, k1, 31 - lane));
    }
    s_top[warp * 32 + lane] = top;
  bmax = warp_max(bmax);
    if (lane == 0) s_red2[warp] = bmax;
  }
  __syncthreads();
  OSM_STAMP(3);
  for (int step = 1; step < TPB / 32; step <<= 1) {
    if (route && (warp & (2 * step - 1)) == 0) {
      top = merge_top(top, s_top[(warp + step) * 32 + 31 - lane]);
      s_top[warp * 32 + lane] = top;
    }
    __syncthreads();
  }
  if (route && warp == 0 && lane < nsel && nsel <= 32) {
    sel_id[lane] = key_id(top);
    sel_v[lane] = key_value(top);
  }
  __syncthreads();
  OSM_STAMP(4);
  float mx = 0.0f;
  if (route) {
    mx = sel_v[0];
    float es = 0.0f;
#pragma unroll
    for (int r = 0; r < 2; ++r)
      if (tid + r * TPB < g.E) es += __expf(__fsub_rn(lv[r], mx));
    es = warp_sum(es);
    if (lane == 0) red[warp] = es;
  }
  __syncthreads();
  OSM_STAMP(5);
  if (warp == 0 && route) {
    const int nw = blockDim.x >> 5;
    const float ssum = warp_sum(lane < nw ? red[lane] : 0.0f);
    const float bm = warp_max(lane < nw ? s_red2[lane] : 0.0f);
    bool ok_j = true;
    if (lane + 1 < nsel) {
      const float need = 2.0f * bm * 1.0001f + 1e-6f +
                         3e-7f * (fabsf(sel_v[lane] - mx) + fabsf(sel_v[lane + 1] - mx));
      ok_j = __fsub_rd(sel_v[lane], sel_v[lane + 1]) > need;
    }
    const bool ok = __all_sync(0xFFFFFFFFu, ok_j) && !a.force_exact && isfinite(mx) && nsel <= 32;
    if (ok) {
      write_weights(a, tok, ssum, mx, sel_id, sel_v);
    } else if (lane == 0) {
      s_flag = a.force_exact ? 2 : 1;
      s_bm = bm;
      s_sum = ssum;
      s_mx = mx;
    }
    OSM_STAMP(6);
  }
  if (warp == 1) OSM_STAMP(7);
  __syncthreads();
  OSM_STAMP(8);
  // ---- 2. partial exact path: recompute the ambiguous candidates ----
  if (s_flag == 1) {
    if (tid == 0) atomicAdd(a.exact_count, 1ull);
    const float thr = sel_v[k - 1] - 2.0f * s_bm * 1.0001f - 1e-6f;
    for (int e = tid; e < g.E; e += blockDim.x) {
      if (a.logits[(size_t)tok * g.E + e] >= thr) {
        const int idx = atomicAdd(&s_ncand, 1);
        if (idx < kMaxCand) cand_id[idx] = e;
      }
    }
    __syncthreads();
    const int nc = s_ncand;
    if (nc > kMaxCand || g.f32w || g.q8 || nc < k) {
      if (tid == 0) s_flag = 2;
    } else {
      // rows of the candidates, kPartChunk values of h at a time, transposed:
      // wt[(h - hc) * kMaxCand + j] (bf16)
      uint16_t* wt = reinterpret_cast<uint16_t*>(uni);
      constexpr int vpc = kPartChunk / 8;  // 8-element vectors per row and chunk
      // the reference's sequential sum, carried across the chunks in h order:
      // products are independent of the running sum, so a batch of them is
      // formed ahead of the add chain
      float acc = 0.0f;
      for (int hc = 0; hc < g.H; hc += kPartChunk) {
        for (int i = tid; i < nc * vpc; i += blockDim.x) {
          const int j = i / vpc, h0 = hc + 8 * (i - j * vpc);
          if (h0 >= g.H) continue;
          const int l = h0 / g.c, m = (h0 - l * g.c) >> 3;
          const uint4 q = __ldg(a.wp + ((size_t)cand_id[j] * g.nvec + m) * 32 + l);
          const uint32_t ww[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int jj = 0; jj < 8; ++jj)
            if (h0 + jj < g.H)
              wt[(h0 - hc + jj) * kMaxCand + j] = (uint16_t)((ww[jj >> 1] >> ((jj & 1) * 16)) & 0xFFFFu);
        }
        __syncthreads();
        if (tid < nc) {
          const int he = min(g.H, hc + kPartChunk);
          int h = hc;
          for (; h + 64 <= he; h += 64) {
            float pr[64];
#pragma unroll
            for (int u = 0; u < 64; ++u)
              pr[u] = __fmul_rn(bf16_bits_to_f32(wt[(h - hc + u) * kMaxCand + tid]), xs[h + u]);
#pragma unroll
            for (int u = 0; u < 64; ++u) acc = __fadd_rn(acc, pr[u]);
          }
          for (; h < he; ++h)
            acc = __fadd_rn(acc, __fmul_rn(bf16_bits_to_f32(wt[(h - hc) * kMaxCand + tid]), xs[h]));
        }
        __syncthreads();  // the chunk's rows are read before the next overwrite
      }
      if (tid < nc) {
        if (a.bias != nullptr) acc = __fadd_rn(acc, a.bias[cand_id[tid]]);
        cand_l[tid] = acc;
      }
      __syncthreads();
      if (warp == 0) {
        // rank the candidates by (exact logit desc, id asc)
        const float myl = lane < nc ? cand_l[lane] : -INFINITY;
        const int myid = lane < nc ? cand_id[lane] : 0x7FFFFFFF;
        int rank = 0;
        for (int i = 0; i < nc; ++i) {
          const float ol = cand_l[i];
          const int oi = cand_id[i];
          if (better(ol, oi, myl, myid)) ++rank;
        }
        __syncwarp();
        if (lane < nc) {
          sel_id[rank] = myid;
          sel_v[rank] = myl;
        }
        __syncwarp();
        bool ok = isfinite(sel_v[0]);
        const int npair = k < nc ? k : nc - 1;  // pairs (r, r+1) that decide ids/order
        for (int r = 0; r < npair; ++r)
          if (!distinct_p(sel_v[r], sel_v[r + 1], sel_v[0])) ok = false;
        if (ok) write_weights(a, tok, s_sum, s_mx, sel_id, sel_v);
        else if (lane == 0) s_flag = 2;
      }
    }
    __syncthreads();
  }
  // ---- 3. full exact path: the reference's arithmetic for the whole token ----
  if (s_flag == 2) {
    float* lex = reinterpret_cast<float*>(uni);                  // [E]
    uint16_t* tile = reinterpret_cast<uint16_t*>(lex + g.E);      // [kFullTile][E]
    float* tilef = reinterpret_cast<float*>(lex + g.E);           // fp32 router tiles
    float acc[2] = {0.0f, 0.0f};  // experts tid, tid + 512
    for (int h0 = 0; h0 < g.H; h0 += kFullTile) {
      // stage h in [h0, h0 + kFullTile) of every row, transposed [hh][e]
      const int nvt = kFullTile / 8;
      for (int i = tid; i < g.E * nvt; i += blockDim.x) {
        const int e = i / nvt, vv = i - e * nvt;
        const int h = h0 + vv * 8;
        if (h >= g.Hp) continue;
        const int l = h / g.c, o = h - l * g.c;
        float w8[8];
        load8(a, e, o >> 3, l, w8);
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          if (g.f32w || g.q8) tilef[(vv * 8 + jj) * g.E + e] = w8[jj];
          else tile[(vv * 8 + jj) * g.E + e] = (uint16_t)(__float_as_uint(w8[jj]) >> 16);
        }
      }
      __syncthreads();
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int e = tid + r * TPB;
        if (e < g.E) {
          const int nh = min(kFullTile, g.H - h0);
          float pr[kFullTile];
#pragma unroll
          for (int hh = 0; hh < kFullTile; ++hh) {
            const float w = hh < nh ? (g.f32w || g.q8 ? tilef[hh * g.E + e] : bf16_bits_to_f32(tile[hh * g.E + e])) : 0.0f;
            pr[hh] = __fmul_rn(w, xs[h0 + (hh < nh ? hh : 0)]);
          }
#pragma unroll
          for (int hh = 0; hh < kFullTile; ++hh)
            if (hh < nh) acc[r] = __fadd_rn(acc[r], pr[hh]);
        }
      }
      __syncthreads();
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int e = tid + r * TPB;
      if (e < g.E) {
        lex[e] = a.bias != nullptr ? __fadd_rn(acc[r], a.bias[e]) : acc[r];
        if (a.logits_out) a.logits_out[(size_t)tok * g.E + e] = lex[e];
      }
    }
    __syncthreads();
    float m = -INFINITY;
    for (int e = tid; e < g.E; e += blockDim.x) m = fmaxf(m, lex[e]);
    const float mx = block_reduce_max(m, red);
    for (int e = tid; e < g.E; e += blockDim.x)
      lex[e] = (float)exp((double)__fsub_rn(lex[e], mx));
    __syncthreads();
    if (tid == 0) {
      float s = 0.0f;
      for (int e = 0; e < g.E; ++e) s = __fadd_rn(s, lex[e]);
      s_bcast = s;
      if (!(s > 0.0f) || !isfinite(s)) atomicOr(a.status, kStatusBadMass);
    }
    __syncthreads();
    const float sum = s_bcast;
    for (int e = tid; e < g.E; e += blockDim.x) lex[e] = __fdiv_rn(lex[e], sum);
    __syncthreads();
    if (warp == 0) {
      float pv[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int id = i * 32 + lane;
        pv[i] = id < g.E ? lex[id] : -INFINITY;
      }
      warp_select(pv, g.E, k, sel_id, sel_v);
      if (lane == 0) {
        float mass = 0.0f;
        for (int j = 0; j < k; ++j) mass = __fadd_rn(mass, sel_v[j]);
        if (!(mass > 0.0f) || !isfinite(mass)) atomicOr(a.status, kStatusBadMass);
        for (int j = 0; j < k; ++j) {
          a.ids[(size_t)tok * k + j] = (uint32_t)sel_id[j];
          a.weights[(size_t)tok * k + j] = a.norm ? __fdiv_rn(sel_v[j], mass) : sel_v[j];
          if (a.pick_ptr) a.pick_ptr[(size_t)tok * k + j] = slot_base(a, (uint32_t)sel_id[j]);
        }
        a.mass[tok] = mass;
      }
    }
    if (tid == 0 && !a.force_exact) atomicAdd(a.exact_count, 0ull);
  }
  OSM_STAMP(10);
  if (s_flag == 2 && a.force_exact && tid == 0) atomicAdd(a.exact_count, 1ull);
  if (nonfinite && tid == 0 && !a.skip_route) {
    for (int j = 0; j < k; ++j) {
      a.ids[(size_t)tok * k + j] = 0;
      a.weights[(size_t)tok * k + j] = 0.0f;
      if (a.pick_ptr) a.pick_ptr[(size_t)tok * k + j] = nullptr;
    }
    a.mass[tok] = 0.0f;
  }
  __syncthreads();
  OSM_STAMP(11);
  if ((s_flag == 2 || nonfinite) && tid < k && !a.skip_route) {
    if (a.ids_out) a.ids_out[(size_t)tok * k + tid] = a.ids[(size_t)tok * k + tid];
    if (a.weights_out) a.weights_out[(size_t)tok * k + tid] = a.weights[(size_t)tok * k + tid];
  }
  if ((s_flag == 2 || nonfinite) && tid == 0 && a.mass_out && !a.skip_route) a.mass_out[tok] = a.mass[tok];
  // given routing (osm_moe_experts): slot bases of the caller's picks
  if (a.skip_route && a.pick_ptr && tid < k)
    a.pick_ptr[(size_t)tok * k + tid] = slot_base(a, a.ids[(size_t)tok * k + tid]);
  OSM_STAMP(9);
  if (!a.do_group) TL_END(1);
#ifdef OSM_PHASE_TIMING
  if (blockIdx.x == 0 && tid == 0)
    for (int i = 0; i < 12; ++i) g_rcyc[i] = ts_[i] - ts_[0];
#endif
#ifdef OSM_PHASE_PRINT
  if (!a.do_group && tid == 0) {
    printf("select(nogroup) tok %d: g %llu..%llu", tok, gt0_, gtime());
    for (int i = 1; i < 10; ++i) printf(" %d:%lld", i, ts_[i] - ts_[0]);
    printf("\n");
  }
#endif
  if (!a.do_group) return;
  // ---- the last block groups (token, pick) pairs by expert ----
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
  __syncthreads();
  OSM_STAMP(10);
  if (tid == 0) {
    const unsigned int prev = atomicAdd(a.ticket, 1u);
    s_flag = (prev == gridDim.x - 1) ? 3 : 0;
  }
  __syncthreads();
  OSM_STAMP(11);
  if (s_flag != 3) return;
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
  OSM_STAMP(12);
  TL_MARK(8);
  group_pairs(a, reinterpret_cast<int*>(uni), reinterpret_cast<int*>(red));
  if (tid == 0) *a.ticket = 0u;
  __syncthreads();
  OSM_STAMP(13);
  TL_MARK(9);
  TL_END(1);
#ifdef OSM_PHASE_PRINT
  if (tid == 0) {
    printf("select tok %d:", tok);
    for (int i = 1; i < 14; ++i) printf(" %d:%lld", i, ts_[i] - ts_[0]);
    printf(" | group:");
    for (int i = 1; i < 6; ++i) printf(" %d:%lld", i, g_gts[i] - g_gts[0]);
    printf("\n");
  }
#endif
}

// Places (token, pick) pairs at their expert's next position (positions
// inside an expert are arbitrary: every pair's result is independent of its
// place), then the shared expert's pairs in token order.  One thread per pair.
__global__ void __launch_bounds__(256) scatter_pairs_kernel(RouterArgs a) {
  pdl_wait();
  pdl_trigger();
  const int E = a.g.E, k = a.g.k, B = a.B;
  const int has_sh = a.shared_slot != nullptr;
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p < B * k) {
    const uint32_t e = __ldcg(a.ids + p);
    if (e >= (uint32_t)E) return;
    const int pos = __ldcg(a.counts + e) + atomicAdd(a.cursor + e, 1);
    a.pair_tok[pos] = p / k;
    a.pair_pick[pos] = p % k;
    if (a.tp_pos) a.tp_pos[(p / k) * (k + has_sh) + p % k] = pos;
  } else if (has_sh && p < B * k + B) {
    const int t = p - B * k;
    const int pos = __ldcg(a.counts + E) + t;
    a.pair_tok[pos] = t;
    a.pair_pick[pos] = k;
    if (a.tp_pos) a.tp_pos[t * (k + 1) + k] = pos;
  }
}

// Binds a routing that the select kernel left in a.ids / a.mass to the slab
// (pick_ptr, when requested: null for a token the select refused, whose
// mass it set to 0, as the select itself does) and, with a.do_group, groups
// the (token, pick) pairs by expert.
__global__ void __launch_bounds__(kSelThreads) group_kernel(RouterArgs a) {
  extern __shared__ float4 smem4[];
  __shared__ int red[32];
  pdl_wait();
  pdl_trigger();
  if (a.pick_ptr)
    for (int p = threadIdx.x; p < a.B * a.g.k; p += blockDim.x)
      a.pick_ptr[p] = __ldcg(a.mass + p / a.g.k) > 0.0f ? slot_base(a, __ldcg(a.ids + p)) : nullptr;
  if (a.do_group) group_pairs(a, reinterpret_cast<int*>(smem4), red);
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

template <int EXP, int TOKS>
void launch_logits_t(const RouterArgs& a, cudaStream_t s) {
  const RouterGeom& g = a.g;
  const dim3 grid((g.E + EXP * kLogitWarps - 1) / (EXP * kLogitWarps), (a.B + TOKS - 1) / TOKS);
  const size_t sm = (size_t)TOKS * 32 * (g.c + 4) * sizeof(float);
  launch_pdl(router_logits_kernel<EXP, TOKS>, grid, dim3(kLogitWarps * 32), sm, s, a);
}

size_t select_smem(const RouterGeom& g) {
  const size_t xs = (size_t)((g.H + 3) & ~3) * sizeof(float);
  const size_t partial = (size_t)kPartChunk * kMaxCand * sizeof(uint16_t);
  const size_t full = (size_t)g.E * sizeof(float) + (size_t)kFullTile * g.E * sizeof(float);
  const size_t grp = (size_t)5 * (g.E + 1) * sizeof(int);
  size_t u = partial;
  if (full > u) u = full;
  if (grp > u) u = grp;
  return xs + u;
}

template <int TT, bool F32, int STG = kExStages>
void launch_exact_t(const RouterArgs& a, cudaStream_t s) {
  const dim3 grid((a.g.E + kExThreads - 1) / kExThreads, (a.B + TT - 1) / TT);
  const size_t sm = (size_t)STG * kExTile + (size_t)TT * a.g.H * sizeof(float);
  launch_pdl(router_exact_kernel<TT, F32, STG>, grid, dim3(kExThreads), sm, s, a);
}

template <int TT, int FMT, int STG, int NW>
void launch_exact2_t(const RouterArgs& a, cudaStream_t s) {
  constexpr int HPT = FMT == 1 ? 32 : FMT == 0 ? 64 : 128;
  const dim3 grid((a.g.E + 32 * NW - 1) / (32 * NW), (a.B + TT - 1) / TT);
  const size_t sm = (size_t)STG * (32 * NW * 128 + TT * HPT * 4);
  launch_pdl(router_exact2_kernel<TT, FMT, STG, NW>, grid, dim3(NW * 32 + 32), sm, s, a);
}

template <int FMT>
void launch_exact2(const RouterArgs& a, cudaStream_t s) {
  // tokens per thread and experts per block grow with the batch
  if (a.B <= 16) launch_exact2_t<1, FMT, 4, 1>(a, s);
  else if (a.B <= 64) launch_exact2_t<2, FMT, 4, 1>(a, s);
  else if (a.B <= 512) launch_exact2_t<4, FMT, 4, 2>(a, s);
  else launch_exact2_t<8, FMT, 4, 4>(a, s);
}

template <bool F32>
void launch_exact(const RouterArgs& a, cudaStream_t s) {
  const int HPT = F32 ? 32 : 64;
  if ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && a.g.H % HPT == 0 && a.g.E % 32 == 0) {
    launch_exact2<F32 ? 1 : 0>(a, s);
    return;
  }
  // tokens per thread grow with the batch; the sequential sum's latency
  // (H dependent adds) bounds small batches
  if (a.B <= 16) launch_exact_t<1, F32>(a, s);
  else if (a.B <= 64) launch_exact_t<2, F32>(a, s);
  else if (a.B < 2048) launch_exact_t<4, F32>(a, s);
  else launch_exact_t<8, F32, 2>(a, s);
}

}  // namespace

// 1-2 tokens: certified fast logits (the selection checks their bounds);
// 3+ tokens: exact logits, one thread per (expert, token group).
void launch_router_logits(const RouterArgs& a, cudaStream_t s, uint64_t* launches) {
  if (a.B <= 2) {
    launch_logits_t<1, 1>(a, s);
  } else if (a.g.q8) {
    launch_exact2<2>(a, s);  // the layer guarantees H % 128, E % 32 and an aligned x
  } else if (a.g.f32w) {
    launch_exact<true>(a, s);
  } else {
    launch_exact<false>(a, s);
  }
  if (launches) *launches += 1;
}

// One token per block: 512 threads while the tokens fit one wave of such
// blocks (two per SM on 148 SMs), 256 beyond (twice the tokens resident per
// SM, more work per thread); 256 threads take up to 512 experts.
constexpr int kSelWideTokens = 2 * 148;
void launch_router_select(const RouterArgs& a, cudaStream_t s, uint64_t* launches) {
  const size_t sm = select_smem(a.g);
  if (a.B <= kSelWideTokens || a.g.E > 2 * 256)
    launch_pdl(router_select_kernel<512>, dim3(a.B), dim3(512), sm, s, a);
  else
    launch_pdl(router_select_kernel<256>, dim3(a.B), dim3(256), sm, s, a);
  if (launches) *launches += 1;
  if (a.defer_scatter && a.do_group) {
    const int n = a.B * (a.g.k + 1);
    launch_pdl(scatter_pairs_kernel, dim3((n + 255) / 256), dim3(256), 0, s, a);
    if (launches) *launches += 1;
  }
}

void init_router_attributes(int max_smem) {
  cudaFuncSetAttribute(router_logits_kernel<1, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_logits_kernel<2, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact_kernel<1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact_kernel<2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact_kernel<4, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact_kernel<1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact_kernel<2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact_kernel<4, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact_kernel<8, false, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact_kernel<8, true, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact2_kernel<1, 0, 4, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact2_kernel<2, 0, 4, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact2_kernel<4, 0, 4, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact2_kernel<8, 0, 4, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact2_kernel<1, 1, 4, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact2_kernel<2, 1, 4, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact2_kernel<4, 1, 4, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact2_kernel<8, 1, 4, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact2_kernel<1, 2, 4, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact2_kernel<2, 2, 4, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact2_kernel<4, 2, 4, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_exact2_kernel<8, 2, 4, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_select_kernel<512>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(router_select_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
}

void launch_group(const RouterArgs& a, cudaStream_t s, uint64_t* launches) {
  const size_t sm = (size_t)5 * (a.g.E + 1) * sizeof(int);
  launch_pdl(group_kernel, dim3(1), dim3(kSelThreads), sm, s, a);
  if (launches) *launches += 1;
  if (a.defer_scatter && a.do_group) {
    const int n = a.B * (a.g.k + 1);
    launch_pdl(scatter_pairs_kernel, dim3((n + 255) / 256), dim3(256), 0, s, a);
    if (launches) *launches += 1;
  }
}

}  // namespace osm

#ifdef OSM_PHASE_TIMING
extern "C" int osm_dbg_cycles_router(long long* out) {
  return (int)cudaMemcpyFromSymbol(out, osm::g_rcyc, 16 * sizeof(long long));
}
extern "C" int osm_dbg_timeline_router(unsigned long long* out) {
  unsigned long long init[OSM_TL_SLOTS];
  for (int i = 0; i < OSM_TL_SLOTS; ++i) init[i] = (i == 0 || i == 4) ? ~0ull : 0ull;
  cudaMemcpyFromSymbol(out, osm::g_tl, sizeof(init));
  return (int)cudaMemcpyToSymbol(osm::g_tl, init, sizeof(init));
}
#endif

namespace osm {
cudaError_t set_first_wait_polls_router(uint32_t polls) { return set_first_wait_polls(polls); }
}  // namespace osm
