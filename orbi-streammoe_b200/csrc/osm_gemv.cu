// osm_gemv.cu -- the latency path of the expert MLPs for 1-2 tokens per call
// (replaces, for decode, the per-expert q4_gemv / swiglu / weighted_accumulate
// submits of src/model/routed_moe.cpp:320-404).
//
// With one or two tokens a tensor-core tile wastes most of its columns, so the
// dot products run on CUDA cores in fp32:
//  * a 16-byte chunk of a Q4 row holds 32 nibbles of one 64-wide group; the
//    nibbles are turned into floats without shifts: OR-ing the nibble in place
//    into the mantissa of 2^23 gives 2^23 + q*16^k exactly, and the activation
//    is stored pre-multiplied by 16^-k (an exact power of two), so
//    sum (v - 2^23) * x' = sum q * x exactly per product;
//  * fp32x2 packed FMA/ADD (sm_100) halve the instruction count;
//  * each group is reduced as s * sum(q x) + b * sum(x) (shaders/
//    q4_gemv.comp:44-60), then across lanes.
// gemv_gateup_kernel  one warp per (gate row, up row) pair, lanes over the
//                     input chunks; SwiGLU in the epilogue; h in fp32.
// gemv_down_kernel    one CTA per 8 output rows, warps over the active experts,
//                     half-warps over rows; the CTA then combines every token's
//                     picks in pick order, the shared expert last, then the
//                     residual (routed_moe.cpp:13-92, :396-404), so no partial
//                     buffer or combine kernel is needed.
#include <cuda_runtime.h>
#include <stdint.h>

#include "osm_common.cuh"
#include "osm_kernels.cuh"

#ifdef OSM_PHASE_TIMING
#include <cstdio>
#define GV_STAMP(i) do { if (threadIdx.x == 0) gts_[(i)] = clock64(); } while (0)
#else
#define GV_STAMP(i) do { } while (0)
#endif

namespace osm {
namespace {

constexpr int kGvWarps = 8;
constexpr int kChunkPad = 36;  // floats per staged 32-value chunk (bank spread)
constexpr float kTwo23 = 8388608.0f;

// 16^-k for the nibble at word position k; positions 5..7 are read from the
// word shifted right by 20, so they use 16^-(k-5).
__device__ __forceinline__ float pos_scale(int k) {
  const int e = k <= 4 ? 4 * k : 4 * (k - 5);
  return __uint_as_float((uint32_t)(127 - e) << 23);
}

__device__ __forceinline__ unsigned long long f2pack(float lo, float hi) {
  unsigned long long d;
  asm("mov.b64 %0, {%1,%2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
__device__ __forceinline__ void f2unpack(unsigned long long d, float& lo, float& hi) {
  asm("mov.b64 {%0,%1}, %2;" : "=f"(lo), "=f"(hi) : "l"(d));
}

// sum over the 32 nibbles of chunk q (4 words) of q_j * x_j, with xp the
// pre-scaled activations of the chunk (32 floats).
__device__ __forceinline__ float chunk_dot(uint4 q, const float* xp) {
  const unsigned long long m23 = f2pack(-kTwo23, -kTwo23);
  unsigned long long acc = f2pack(0.0f, 0.0f);
  const uint32_t ws[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int wi = 0; wi < 4; ++wi) {
    const uint32_t w = ws[wi];
    const uint32_t w5 = w >> 20;
    const float4 xa = *reinterpret_cast<const float4*>(xp + 8 * wi);
    const float4 xb = *reinterpret_cast<const float4*>(xp + 8 * wi + 4);
    float v[8];
    v[0] = __uint_as_float(0x4B000000u | (w & 0x0000000Fu));
    v[1] = __uint_as_float(0x4B000000u | (w & 0x000000F0u));
    v[2] = __uint_as_float(0x4B000000u | (w & 0x00000F00u));
    v[3] = __uint_as_float(0x4B000000u | (w & 0x0000F000u));
    v[4] = __uint_as_float(0x4B000000u | (w & 0x000F0000u));
    v[5] = __uint_as_float(0x4B000000u | (w5 & 0x0000000Fu));
    v[6] = __uint_as_float(0x4B000000u | (w5 & 0x000000F0u));
    v[7] = __uint_as_float(0x4B000000u | (w5 & 0x00000F00u));
    const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      unsigned long long q2 = f2pack(v[2 * p], v[2 * p + 1]);
      asm("add.rn.f32x2 %0, %0, %1;" : "+l"(q2) : "l"(m23));
      asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(q2), "l"(f2pack(xv[2 * p], xv[2 * p + 1])));
    }
  }
  float lo, hi;
  f2unpack(acc, lo, hi);
  return lo + hi;
}

// Stage activations of length K (token rows of `src`) as pre-scaled chunks:
// dst[t][c][kChunkPad], and the plain chunk sums sums[t][c].  One thread per
// 32-value chunk: its 8 float4 loads are all in flight at once.
__device__ void stage_chunks(const float* __restrict__ src, int rows, int K, float* dst,
                             float* sums) {
  const int nch = K >> 5;
  for (int i = threadIdx.x; i < rows * nch; i += blockDim.x) {
    const int t = i / nch, c = i - t * nch;
    const float4* s4 = reinterpret_cast<const float4*>(src + (size_t)t * K + c * 32);
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = s4[u];
    float acc = 0.0f;
    float4* d4 = reinterpret_cast<float4*>(dst + (size_t)i * kChunkPad);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      acc += v[u].x;
      acc += v[u].y;
      acc += v[u].z;
      acc += v[u].w;
      // positions 4u..4u+3 of the chunk: word position (4u + e) & 7
      const int k0 = (4 * u) & 7;
      d4[u] = make_float4(v[u].x * pos_scale(k0), v[u].y * pos_scale(k0 + 1),
                          v[u].z * pos_scale(k0 + 2), v[u].w * pos_scale(k0 + 3));
    }
    sums[i] = acc;
  }
}

// Active entry j: from the grouping step, or in direct mode pick j of the one
// token (j == k: the shared expert).
__device__ __forceinline__ ActEntry gemv_entry(const GemvArgs& a, int j) {
  if (!a.direct) return a.act[j];
  ActEntry en;
  en.off = j;
  en.cnt = 1;
  en.tg0 = 0;
  en.pad0 = en.pad1 = 0;
  if (j < a.k) {
    en.kind = 0;
    const uint32_t e = a.ids[j];
    const int slot = a.slot_of[e];
    if (slot < 0) {
      if (threadIdx.x == 0) atomicOr(a.status, kStatusNotResident);
      en.ptr = nullptr;
    } else {
      en.ptr = a.slab + (size_t)slot * a.slab_stride;
    }
  } else {
    en.kind = 1;
    en.ptr = a.shared_ptr;
  }
  return en;
}

__device__ __forceinline__ int gemv_entries(const GemvArgs& a) {
  return a.direct ? a.k + a.has_shared : *a.n_active;
}

// ----------------------------------------------------------------------------
// gate/up + SwiGLU.  Item = (active expert j, 16 row pairs); warp w owns row
// pairs r0 + 2w, r0 + 2w + 1.
// ----------------------------------------------------------------------------
__global__ void __launch_bounds__(kGvWarps * 32) gemv_gateup_kernel(GemvArgs a, int tiles) {
  extern __shared__ float4 sm4[];
  float* xs = reinterpret_cast<float*>(sm4);             // [B][H/32][36]
  const int nch = a.H >> 5;
  float* xsum = xs + a.B * nch * kChunkPad;              // [B][H/32]
#ifdef OSM_PHASE_TIMING
  __shared__ long long gts_[8];
#endif
  GV_STAMP(0);
  // x is complete when this kernel starts (the router's predecessor).
  stage_chunks(a.x, a.B, a.H, xs, xsum);
  GV_STAMP(1);
  pdl_wait();
  pdl_trigger();
  __syncthreads();
  GV_STAMP(2);
  const int n_items = gemv_entries(a) * tiles;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int j = item / tiles, tile = item - (item / tiles) * tiles;
    const ActEntry en = gemv_entry(a, j);
    if (en.ptr == nullptr) continue;
    const int kind = en.kind;
    const int rows = a.gu.rows[kind];
    const int G = a.gu.K[kind] >> 6;
    const uint8_t* base = en.ptr;
    const uint4* Wg = reinterpret_cast<const uint4*>(base + a.gu.w[kind]);
    const uint4* Wu = reinterpret_cast<const uint4*>(base + a.gu.w2[kind]);
    const uint16_t* Sg = reinterpret_cast<const uint16_t*>(base + a.gu.s[kind]);
    const uint16_t* Bg = reinterpret_cast<const uint16_t*>(base + a.gu.b[kind]);
    const uint16_t* Su = reinterpret_cast<const uint16_t*>(base + a.gu.s2[kind]);
    const uint16_t* Bu = reinterpret_cast<const uint16_t*>(base + a.gu.b2[kind]);
    const int cpr = a.gu.K[kind] >> 5;  // 16-byte chunks per row
    GV_STAMP(3);
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int r = tile * 2 * kGvWarps + 2 * warp + rr;
      if (r >= rows) continue;
      // chunks c = lane, lane + 32 (K = 2048: one 64-group per two chunks)
      uint4 qg[2], qu[2];
      float sg[2], bg[2], su[2], bu[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int c = lane + 32 * u;
        if (c < cpr) {
          qg[u] = __ldg(Wg + (size_t)r * cpr + c);
          qu[u] = __ldg(Wu + (size_t)r * cpr + c);
          sg[u] = bf16_bits_to_f32(__ldg(Sg + (size_t)r * G + (c >> 1)));
          bg[u] = bf16_bits_to_f32(__ldg(Bg + (size_t)r * G + (c >> 1)));
          su[u] = bf16_bits_to_f32(__ldg(Su + (size_t)r * G + (c >> 1)));
          bu[u] = bf16_bits_to_f32(__ldg(Bu + (size_t)r * G + (c >> 1)));
        }
      }
      for (int i = 0; i < en.cnt; ++i) {
        const int pos = en.off + i;
        const int t = a.direct ? 0 : a.pair_tok[pos];
        float gacc = 0.0f, uacc = 0.0f;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int c = lane + 32 * u;
          if (c < cpr) {
            const float* xp = xs + (t * nch + c) * kChunkPad;
            const float xsm = xsum[t * nch + c];
            gacc = fmaf(bg[u], xsm, fmaf(sg[u], chunk_dot(qg[u], xp), gacc));
            uacc = fmaf(bu[u], xsm, fmaf(su[u], chunk_dot(qu[u], xp), uacc));
          }
        }
        gacc = warp_sum(gacc);
        uacc = warp_sum(uacc);
        if (lane == 0) a.h[(size_t)pos * a.Imax + r] = __fmul_rn(ref_silu(gacc), uacc);
      }
      if (rr == 0) GV_STAMP(4);
    }
    GV_STAMP(5);
  }
#ifdef OSM_PHASE_TIMING
  if (threadIdx.x == 0 && (blockIdx.x == 0 || blockIdx.x == 200))
    printf("gateup cta %d: 1:%lld 2:%lld 3:%lld 4:%lld 5:%lld\n", (int)blockIdx.x, gts_[1] - gts_[0],
           gts_[2] - gts_[0], gts_[3] - gts_[0], gts_[4] - gts_[0], gts_[5] - gts_[0]);
#endif
}

// ----------------------------------------------------------------------------
// down + combine.  CTA = 8 output rows for every token.
// ----------------------------------------------------------------------------
template <int CH>  // 16-byte chunks per lane and row: 1 for K <= 512, 2 for K <= 1024
__global__ void __launch_bounds__(kGvWarps * 32, 2) gemv_down_kernel(GemvArgs a) {
  extern __shared__ float4 sm4[];
  const int P = a.B * (a.k + a.has_shared);
  const int nch = a.Imax >> 5;
  float* hs = reinterpret_cast<float*>(sm4);        // [P][Imax/32][36]
  float* hsum = hs + P * nch * kChunkPad;            // [P][Imax/32]
  float* ys = hsum + P * nch;                        // [P][8]
#ifdef OSM_PHASE_TIMING
  __shared__ long long gts_[8];
#endif
  GV_STAMP(0);
  pdl_wait();
  pdl_trigger();
  GV_STAMP(1);
  stage_chunks(a.h, P, a.Imax, hs, hsum);
  __syncthreads();
  GV_STAMP(2);
  const int n_active = gemv_entries(a);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = lane >> 4, hl = lane & 15;
  const int r0 = blockIdx.x * 8;
  for (int j = warp; j < n_active; j += kGvWarps) {
    const ActEntry en = gemv_entry(a, j);
    if (en.ptr == nullptr) continue;
    const int kind = en.kind;
    const int K = a.dn.K[kind];
    const int G = K >> 6, cpr = K >> 5;
    const uint4* W = reinterpret_cast<const uint4*>(en.ptr + a.dn.w[kind]);
    const uint16_t* S = reinterpret_cast<const uint16_t*>(en.ptr + a.dn.s[kind]);
    const uint16_t* Bb = reinterpret_cast<const uint16_t*>(en.ptr + a.dn.b[kind]);
    // rows r0 + 2*step + half, chunks c = hl, hl + 16, ...
    uint4 q[4][CH];
    float s[4][CH], b[4][CH];
#pragma unroll
    for (int st = 0; st < 4; ++st) {
      const int r = r0 + 2 * st + half;
#pragma unroll
      for (int u = 0; u < CH; ++u) {
        const int c = hl + 16 * u;
        if (c < cpr) {
          q[st][u] = __ldg(W + (size_t)r * cpr + c);
          s[st][u] = bf16_bits_to_f32(__ldg(S + (size_t)r * G + (c >> 1)));
          b[st][u] = bf16_bits_to_f32(__ldg(Bb + (size_t)r * G + (c >> 1)));
        }
      }
    }
    for (int i = 0; i < en.cnt; ++i) {
      const int pos = en.off + i;
#pragma unroll
      for (int st = 0; st < 4; ++st) {
        float acc = 0.0f;
#pragma unroll
        for (int u = 0; u < CH; ++u) {
          const int c = hl + 16 * u;
          if (c < cpr) {
            const float* hp = hs + (pos * nch + c) * kChunkPad;
            acc = fmaf(b[st][u], hsum[pos * nch + c], fmaf(s[st][u], chunk_dot(q[st][u], hp), acc));
          }
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
        if (hl == 0) ys[pos * 8 + 2 * st + half] = acc;
      }
    }
  }
  __syncthreads();
  GV_STAMP(3);
  // combine in pick order, shared expert last, then the residual
  const int kp1 = a.k + a.has_shared;
  for (int i = threadIdx.x; i < a.B * 8; i += blockDim.x) {
    const int t = i >> 3, rr = i & 7;
    float acc = 0.0f;
    for (int p = 0; p < a.k; ++p) {
      const int pos = a.direct ? p : a.tp_pos[t * kp1 + p];
      acc = __fadd_rn(acc, __fmul_rn(a.weights[t * a.k + p], ys[pos * 8 + rr]));
    }
    if (a.has_shared) {
      const int pos = a.direct ? a.k : a.tp_pos[t * kp1 + a.k];
      acc = __fadd_rn(acc, __fmul_rn(a.sgate[t], ys[pos * 8 + rr]));
    }
    if (a.residual) acc = __fadd_rn(a.residual[(size_t)t * a.H + r0 + rr], acc);
    a.out[(size_t)t * a.H + r0 + rr] = acc;
  }
  GV_STAMP(4);
#ifdef OSM_PHASE_TIMING
  if (threadIdx.x == 0 && (blockIdx.x == 0 || blockIdx.x == 200))
    printf("down cta %d: 1:%lld 2:%lld 3:%lld 4:%lld\n", (int)blockIdx.x, gts_[1] - gts_[0],
           gts_[2] - gts_[0], gts_[3] - gts_[0], gts_[4] - gts_[0]);
#endif
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

}  // namespace

void init_gemv_attributes(int max_smem) {
  cudaFuncSetAttribute(gemv_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(gemv_down_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  cudaFuncSetAttribute(gemv_down_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
}

void launch_gemv_gateup(const GemvArgs& a, int max_active, int grid_cap, cudaStream_t s,
                        uint64_t* launches) {
  const int Imax = a.Imax;
  const int tiles = (Imax + 2 * kGvWarps - 1) / (2 * kGvWarps);
  const int nch = a.H >> 5;
  const size_t smem = (size_t)a.B * nch * (kChunkPad + 1) * sizeof(float);
  long long items = (long long)tiles * max_active;
  int grid = (int)(items < grid_cap ? items : grid_cap);
  if (grid < 1) grid = 1;
  launch_pdl(gemv_gateup_kernel, dim3(grid), dim3(kGvWarps * 32), smem, s, a, tiles);
  if (launches) *launches += 1;
}

void launch_gemv_down(const GemvArgs& a, cudaStream_t s, uint64_t* launches) {
  const int P = a.B * (a.k + a.has_shared);
  const int nch = a.Imax >> 5;
  const size_t smem = ((size_t)P * nch * (kChunkPad + 1) + (size_t)P * 8) * sizeof(float);
  const int kmax = a.dn.K[0] > a.dn.K[1] ? a.dn.K[0] : a.dn.K[1];
  if (kmax <= 512) launch_pdl(gemv_down_kernel<1>, dim3(a.H / 8), dim3(kGvWarps * 32), smem, s, a);
  else launch_pdl(gemv_down_kernel<2>, dim3(a.H / 8), dim3(kGvWarps * 32), smem, s, a);
  if (launches) *launches += 1;
}

}  // namespace osm
