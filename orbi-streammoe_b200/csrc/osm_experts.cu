// osm_experts.cu -- Q4 expert projections on sm_100a (replace
// shaders/q4_gemv.comp, shaders/swiglu.comp and the per-expert submits of
// src/backend/vulkan_resident_expert.cpp:286-365).
//
// proj_kernel<PAIRED, KSPLIT, MAXG> computes, for every active expert and
// every token routed to it, one output tile with mma.sync m16n8k16:
//   A = 16 weight rows x 16 inputs: the Q4 nibbles as exact bf16 integers,
//   B = 16 inputs x 8 tokens: the activation split into bf16 hi + lo,
//   D = fp32 per 64-input group, then acc += s * D + b * sum(x)
// (the group identity of shaders/q4_gemv.comp:44-60 with the reference's
// dequantised value s*q + b).  PAIRED tiles hold gate rows r..r+7 in MMA rows
// 0-7 and the matching up rows in MMA rows 8-15, so each thread owns gate and
// up of the same (row, token) and applies SwiGLU in registers; the result is
// written as the next projection's activation fragments.  KSPLIT warps share
// one tile's input range; 4 / KSPLIT tiles per CTA.
#include <cuda_runtime.h>
#include <stdint.h>

#include "osm_common.cuh"
#include "osm_kernels.cuh"

#ifdef OSM_PHASE_TIMING
#include <cstdio>
#define OSM_PSTAMP(i) do { if (threadIdx.x == 0) pts_[(i)] = clock64(); } while (0)
#else
#define OSM_PSTAMP(i) do { } while (0)
#endif

namespace osm {
namespace {

constexpr int kWarps = 4;

__device__ __forceinline__ void mma_group(float d[4], uint2 wl, uint2 wh, const uint4 (&xf)[4]) {
#pragma unroll
  for (int jj = 0; jj < 2; ++jj) {
    const uint32_t wlo = jj ? wl.y : wl.x;
    const uint32_t whi = jj ? wh.y : wh.x;
    const uint4 xh = xf[2 * jj], xl = xf[2 * jj + 1];
    {
      const uint32_t a0 = nibble_pair_bf16(wlo, 0), a2 = nibble_pair_bf16(wlo, 1);
      const uint32_t a1 = nibble_pair_bf16(whi, 0), a3 = nibble_pair_bf16(whi, 1);
      mma_bf16_16816(d, a0, a1, a2, a3, xh.x, xh.y);
      mma_bf16_16816(d, a0, a1, a2, a3, xl.x, xl.y);
    }
    {
      const uint32_t a0 = nibble_pair_bf16(wlo, 2), a2 = nibble_pair_bf16(wlo, 3);
      const uint32_t a1 = nibble_pair_bf16(whi, 2), a3 = nibble_pair_bf16(whi, 3);
      mma_bf16_16816(d, a0, a1, a2, a3, xh.z, xh.w);
      mma_bf16_16816(d, a0, a1, a2, a3, xl.z, xl.w);
    }
  }
}

// One work item: token group `tg` (up to kTokGroup tokens of one active
// expert) x CTA tile `bx` (TILES row tiles).  Activation fragments of each
// 8-token chunk are staged in shared memory by the whole CTA at once (xs:
// [8][KW*2 + 1] uint4, padded against bank conflicts).
template <bool PAIRED, int KSPLIT, int MAXG>
__device__ __forceinline__ void proj_item(const ProjArgs& a, int item, int tiles, bool first,
                                          int& n_items, uint4* xs) {
  constexpr int TILES = kWarps / KSPLIT;
  constexpr int TROWS = PAIRED ? 8 : 16;
  const int tg = item / tiles, bx = item - (item / tiles) * tiles;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, t = lane & 3;
  const int tile = warp / KSPLIT, ks = warp - tile * KSPLIT;
  // Token group 0 belongs to the shared expert when there is one: its weights
  // are known before the routing is, so they are fetched before the wait.
  const bool early = first && a.shared_first && tg == 0;
  const uint8_t* base = early ? a.shared_ptr : nullptr;
  int kind = 1;
  uint2 wl[MAXG], wh[MAXG];
  uint32_t sp[MAXG], bp[MAXG];  // bf16 pairs (lo row, hi row) of scale / bias
  int rows = 0, K = 0, r0 = 0, G = 0, KW = 0;
  auto fetch = [&]() {
    rows = a.sec.rows[kind];
    K = a.sec.K[kind];
    G = K >> 6;
    KW = K >> 3;
    r0 = (bx * TILES + tile) * TROWS;
    const uintptr_t ub = reinterpret_cast<uintptr_t>(base);
    const uint32_t* Wlo = reinterpret_cast<const uint32_t*>(ub + a.sec.w[kind]);
    const uint16_t* Slo = reinterpret_cast<const uint16_t*>(ub + a.sec.s[kind]);
    const uint16_t* Blo = reinterpret_cast<const uint16_t*>(ub + a.sec.b[kind]);
    const uint32_t* Whi = PAIRED ? reinterpret_cast<const uint32_t*>(ub + a.sec.w2[kind]) : Wlo;
    const uint16_t* Shi = PAIRED ? reinterpret_cast<const uint16_t*>(ub + a.sec.s2[kind]) : Slo;
    const uint16_t* Bhi = PAIRED ? reinterpret_cast<const uint16_t*>(ub + a.sec.b2[kind]) : Blo;
    const int row_lo = r0 + gid;
    const int row_hi = PAIRED ? r0 + gid : r0 + 8 + gid;
    const bool live = r0 < rows;
#pragma unroll
    for (int i = 0; i < MAXG; ++i) {
      const int g = ks + KSPLIT * i;
      if (live && g < G) {
        wl[i] = __ldg(reinterpret_cast<const uint2*>(Wlo + (size_t)row_lo * KW + g * 8 + 2 * t));
        wh[i] = __ldg(reinterpret_cast<const uint2*>(Whi + (size_t)row_hi * KW + g * 8 + 2 * t));
        sp[i] = pack2(__ldg(Slo + (size_t)row_lo * G + g), __ldg(Shi + (size_t)row_hi * G + g));
        bp[i] = pack2(__ldg(Blo + (size_t)row_lo * G + g), __ldg(Bhi + (size_t)row_hi * G + g));
      } else {
        wl[i] = wh[i] = make_uint2(0u, 0u);
        sp[i] = bp[i] = 0u;
      }
    }
  };
#ifdef OSM_PHASE_TIMING
  __shared__ long long pts_[12];
#endif
  OSM_PSTAMP(0);
  if (early) fetch();
  if (first) {
    pdl_wait();
    n_items = *a.n_tg * tiles;
  }
  OSM_PSTAMP(1);
  if (item >= n_items) return;
  const int j = a.tg_expert[tg];
  const ActEntry en = a.act[j];
  OSM_PSTAMP(2);
  if (!early) {
    base = en.ptr;
    kind = en.kind;
    if (base == nullptr && !a.raw) return;  // non-resident expert (status already set)
    fetch();
  }
  OSM_PSTAMP(3);
  if ((bx * TILES) * TROWS >= rows) return;

  __shared__ float fsg[8][33];
  __shared__ int rowof[8];
  __shared__ float red[kWarps][32][4];
  __shared__ float hs[TILES][8][9];
  const int t_begin = a.tg_begin[tg];
  const int t_end = min(en.cnt, t_begin + kTokGroup);
  const bool live = r0 < rows;
  const int xstride = KW * 2 + 1;
  for (int c0 = t_begin; c0 < t_end; c0 += 8) {
    const int nv = min(8, t_end - c0);
    if (threadIdx.x < 8) {
      const int p = en.off + c0 + threadIdx.x;
      rowof[threadIdx.x] = threadIdx.x < nv ? (a.frag_by_pair ? p : a.pair_tok[p]) : 0;
    }
    __syncthreads();
    OSM_PSTAMP(4);
    // stage the chunk's activation fragments and group sums (all loads in flight)
    const int per_tok = KW * 2;
#pragma unroll 8
    for (int i = threadIdx.x; i < nv * per_tok; i += blockDim.x) {
      const int n = i / per_tok, r = i - n * per_tok;
      xs[n * xstride + r] = __ldg(a.frag + (size_t)rowof[n] * a.frag_stride * 2 + r);
    }
    for (int i = threadIdx.x; i < 8 * G; i += blockDim.x) {
      const int n = i / G, g = i - n * G;
      float s = 0.0f;
      if (n < nv) {
        const float4* f = reinterpret_cast<const float4*>(a.fsum8 + (size_t)rowof[n] * a.frag_stride + g * 8);
        const float4 u = f[0], w = f[1];
        s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(u.x, u.y), u.z), u.w), w.x), w.y), w.z), w.w);
      }
      fsg[n][g] = s;
    }
    __syncthreads();
    OSM_PSTAMP(5);
    const bool has_tok = gid < nv;
    const uint4* xrow = xs + (has_tok ? gid : 0) * xstride;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int i = 0; i < MAXG; ++i) {
      const int g = ks + KSPLIT * i;
      if (g < G) {
        uint4 xf[4];
        if (has_tok) {
          const int c = 8 * g + 2 * t;
          xf[0] = xrow[2 * c];
          xf[1] = xrow[2 * c + 1];
          xf[2] = xrow[2 * c + 2];
          xf[3] = xrow[2 * c + 3];
        } else {
          xf[0] = xf[1] = xf[2] = xf[3] = make_uint4(0u, 0u, 0u, 0u);
        }
        float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        mma_group(d, wl[i], wh[i], xf);
        const float f0 = fsg[2 * t][g], f1 = fsg[2 * t + 1][g];
        const float sl = bf16_bits_to_f32(sp[i] & 0xFFFFu), sh = bf16_bits_to_f32(sp[i] >> 16);
        const float bl = bf16_bits_to_f32(bp[i] & 0xFFFFu), bh = bf16_bits_to_f32(bp[i] >> 16);
        acc[0] = fmaf(bl, f0, fmaf(sl, d[0], acc[0]));
        acc[1] = fmaf(bl, f1, fmaf(sl, d[1], acc[1]));
        acc[2] = fmaf(bh, f0, fmaf(sh, d[2], acc[2]));
        acc[3] = fmaf(bh, f1, fmaf(sh, d[3], acc[3]));
      }
    }
    OSM_PSTAMP(6);
    float tot[4] = {acc[0], acc[1], acc[2], acc[3]};
    if (KSPLIT > 1) {
#pragma unroll
      for (int q = 0; q < 4; ++q) red[warp][lane][q] = acc[q];
      __syncthreads();
      if (ks == 0) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float s = red[warp][lane][q];
#pragma unroll
          for (int w = 1; w < KSPLIT; ++w) s = __fadd_rn(s, red[warp + w][lane][q]);
          tot[q] = s;
        }
      }
    }
    if (ks == 0 && live) {
      if (PAIRED) {
        // thread (gid, t): gate/up of intermediate row r0+gid, tokens 2t, 2t+1
        hs[tile][gid][2 * t] = __fmul_rn(ref_silu(tot[0]), tot[2]);
        hs[tile][gid][2 * t + 1] = __fmul_rn(ref_silu(tot[1]), tot[3]);
        __syncwarp();
        if (lane < nv) {
          const int p = en.off + c0 + lane;
          const int hch = a.hK >> 3;
          uint32_t hi[8], lo[8];
          float fs = hs[tile][0][lane];
#pragma unroll
          for (int r = 0; r < 8; ++r) split_bf16(hs[tile][r][lane], hi[r], lo[r]);
#pragma unroll
          for (int r = 1; r < 8; ++r) fs = __fadd_rn(fs, hs[tile][r][lane]);
          uint4* dst = a.hfrag + ((size_t)p * hch + (r0 >> 3)) * 2;
          dst[0] = make_uint4(pack2(hi[0], hi[4]), pack2(hi[1], hi[5]), pack2(hi[2], hi[6]),
                              pack2(hi[3], hi[7]));
          dst[1] = make_uint4(pack2(lo[0], lo[4]), pack2(lo[1], lo[5]), pack2(lo[2], lo[6]),
                              pack2(lo[3], lo[7]));
          a.hfsum8[(size_t)p * hch + (r0 >> 3)] = fs;
        }
      } else {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int n = 2 * t + q;
          if (n < nv) {
            const int p = en.off + c0 + n;
            const int orow = a.out_row ? a.out_row[p] : a.pair_tok[p] * a.kp1 + a.pair_pick[p];
            float* o = a.out + (size_t)orow * a.ostride;
            o[r0 + gid] = tot[q];
            o[r0 + 8 + gid] = tot[2 + q];
          }
        }
      }
    }
    __syncthreads();
    OSM_PSTAMP(7);
  }
#ifdef OSM_PHASE_TIMING
  if (threadIdx.x == 0 && (blockIdx.x == 0 || blockIdx.x == 300 || blockIdx.x == 700))
    printf("proj%d cta %d item %d: 1:%lld 2:%lld 3:%lld 4:%lld 5:%lld 6:%lld 7:%lld\n", (int)PAIRED,
           (int)blockIdx.x, item, pts_[1] - pts_[0], pts_[2] - pts_[0], pts_[3] - pts_[0],
           pts_[4] - pts_[0], pts_[5] - pts_[0], pts_[6] - pts_[0], pts_[7] - pts_[0]);
#endif
}

// Persistent grid: CTAs stride over (token group, CTA tile) items; the number
// of token groups is only known on the device.
template <bool PAIRED, int KSPLIT, int MAXG>
__global__ void __launch_bounds__(kWarps * 32, PAIRED ? 5 : 4) proj_kernel(ProjArgs a, int tiles) {
  extern __shared__ uint4 xs_dyn[];
  int n_items = 0x7FFFFFFF;
  bool first = true;
  for (int item = blockIdx.x; first || item < n_items; item += gridDim.x) {
    if (!first) __syncthreads();
    proj_item<PAIRED, KSPLIT, MAXG>(a, item, tiles, first, n_items, xs_dyn);
    first = false;
  }
  pdl_trigger();
}

__global__ void frag_prep_kernel(const float* __restrict__ x, int rows, int K,
                                 uint4* __restrict__ frag, float* __restrict__ fsum8) {
  pdl_wait();
  pdl_trigger();
  const int nch = K >> 3;
  const size_t total = (size_t)rows * nch;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / nch, c = i - r * nch;
    const float* xc = x + r * K + c * 8;
    const float4 p = *reinterpret_cast<const float4*>(xc);
    const float4 q = *reinterpret_cast<const float4*>(xc + 4);
    const float v[8] = {p.x, p.y, p.z, p.w, q.x, q.y, q.z, q.w};
    uint32_t hi[8], lo[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) split_bf16(v[j], hi[j], lo[j]);
    float fs = v[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) fs = __fadd_rn(fs, v[j]);
    frag[i * 2] = make_uint4(pack2(hi[0], hi[4]), pack2(hi[1], hi[5]), pack2(hi[2], hi[6]),
                             pack2(hi[3], hi[7]));
    frag[i * 2 + 1] = make_uint4(pack2(lo[0], lo[4]), pack2(lo[1], lo[5]), pack2(lo[2], lo[6]),
                                 pack2(lo[3], lo[7]));
    fsum8[i] = fs;
  }
}

// Expert list for a single expert over `T` tokens (standalone projections).
__global__ void setup_single_kernel(int T, const uint8_t* ptr, int* n_active, ActEntry* act,
                                    int* n_tg, int* tg_expert, int* tg_begin, int* pair_tok,
                                    int* pair_pick, int* out_row) {
  pdl_wait();
  pdl_trigger();
  const int ng = (T + kTokGroup - 1) / kTokGroup;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *n_active = 1;
    *n_tg = ng;
    ActEntry en;
    en.ptr = ptr;
    en.off = 0;
    en.cnt = T;
    en.kind = 0;
    en.tg0 = 0;
    en.pad0 = en.pad1 = 0;
    act[0] = en;
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < T; i += gridDim.x * blockDim.x) {
    pair_tok[i] = i;
    pair_pick[i] = 0;
    out_row[i] = i;
    if (i < ng) {
      tg_expert[i] = 0;
      tg_begin[i] = i * kTokGroup;
    }
  }
}

template <typename K, typename... Args>
cudaError_t launch_pdl(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
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

int grid_for(size_t n, int threads) {
  size_t b = (n + threads - 1) / threads;
  if (b > 148 * 64) b = 148 * 64;
  if (b < 1) b = 1;
  return (int)b;
}

}  // namespace

cudaError_t launch_frag_prep(const float* x, int rows, int K, uint4* frag, float* fsum8,
                             cudaStream_t s, uint64_t* launches) {
  const size_t n = (size_t)rows * (K >> 3);
  const cudaError_t e =
      launch_pdl(frag_prep_kernel, dim3(grid_for(n, 256)), dim3(256), 0, s, x, rows, K, frag, fsum8);
  if (launches) *launches += 1;
  return e;
}

cudaError_t launch_proj(const ProjArgs& a, ProjKind kind, int max_rows, int max_tg, int grid_cap,
                        int max_tokens_chunk, cudaStream_t s, uint64_t* launches) {
  cudaError_t err = cudaSuccess;
  auto go = [&](auto kernel, int rows_per_cta, int K, int ctas_per_sm) {
    const int tiles = (max_rows + rows_per_cta - 1) / rows_per_cta;
    const int tc = max_tokens_chunk < 8 ? (max_tokens_chunk < 1 ? 1 : max_tokens_chunk) : 8;
    const size_t smem = (size_t)tc * ((K >> 3) * 2 + 1) * sizeof(uint4);
    // resident CTAs: registers allow ctas_per_sm, shared memory (227 KB) may allow fewer
    int per_sm = ctas_per_sm;
    const int by_smem = (int)((227u * 1024u) / (smem + 8192));
    if (by_smem < per_sm) per_sm = by_smem < 1 ? 1 : by_smem;
    const int cap = grid_cap / 4 * per_sm;
    long long items = (long long)tiles * max_tg;
    int grid = (int)(items < cap ? items : cap);
    if (grid < 1) grid = 1;
    err = launch_pdl(kernel, dim3(grid), dim3(kWarps * 32), smem, s, a, tiles);
  };
  const int Kmax = a.sec.K[0] > a.sec.K[1] ? a.sec.K[0] : a.sec.K[1];
  switch (kind) {
    case ProjKind::kGateUp:  // 8 intermediate rows per CTA tile, input split over 4 warps
      go(proj_kernel<true, 4, 8>, 8, Kmax, 5);
      break;
    case ProjKind::kDown:    // 64 output rows per CTA tile, one warp per 16 rows (K <= 512)
      go(proj_kernel<false, 1, 8>, 64, Kmax, 4);
      break;
    case ProjKind::kDown12:  // the same for K <= 768
      go(proj_kernel<false, 1, 12>, 64, Kmax, 4);
      break;
    case ProjKind::kSingle:  // 16 rows per CTA tile, input split over 4 warps (K <= 2048)
      go(proj_kernel<false, 4, 8>, 16, Kmax, 4);
      break;
  }
  if (launches) *launches += 1;
  return err;
}

cudaError_t init_expert_attributes(int max_smem) {
  const auto attr = cudaFuncAttributeMaxDynamicSharedMemorySize;
  cudaError_t e = cudaFuncSetAttribute(proj_kernel<true, 4, 8>, attr, max_smem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(proj_kernel<false, 1, 8>, attr, max_smem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(proj_kernel<false, 1, 12>, attr, max_smem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(proj_kernel<false, 4, 8>, attr, max_smem);
  return e;
}

cudaError_t launch_setup_single(int T, const uint8_t* ptr, int* n_active, ActEntry* act, int* n_tg,
                                int* tg_expert, int* tg_begin, int* pair_tok, int* pair_pick,
                                int* out_row, cudaStream_t s, uint64_t* launches) {
  const cudaError_t e =
      launch_pdl(setup_single_kernel, dim3(grid_for((size_t)T, 256)), dim3(256), 0, s, T, ptr,
                 n_active, act, n_tg, tg_expert, tg_begin, pair_tok, pair_pick, out_row);
  if (launches) *launches += 1;
  return e;
}

}  // namespace osm
