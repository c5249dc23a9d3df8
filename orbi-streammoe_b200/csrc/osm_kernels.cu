// osm_kernels.cu -- sm_100a element-wise kernels of the routed-MoE sublayer
// (the router is in osm_router.cu, the expert projections in osm_experts.cu):
//   combine_kernel   out = sum over picks in pick order of w*y, then the shared
//                    expert s*y, then the residual (src/model/routed_moe.cpp:
//                    13-92, :396-404; src/model/checkpoint_moe_sublayer.cpp:21-33)
//   rmsnorm_kernel   reference_ops.cpp:96-128, sequential (bit-exact) or block
//                    reduction
//   dequant_kernel   reference_ops.cpp:11-67 bit for bit (multiply, then add)
//   swiglu / waccum  shaders/swiglu.comp, shaders/weighted_accumulate.comp
//   gen_*            seeded synthetic weights, quantised like
//                    src/conversion/single_expert_pilot.cpp:276-346
//   router_pack      the router weight layout of osm_kernels.cuh
//   host_copy        a plan's input / output copy through pinned host memory
//                    mapped into the GPU (loads and stores by the SMs)
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "osm_common.cuh"
#include "osm_kernels.cuh"

namespace osm {

namespace {


// ----------------------------------------------------------------------------
// Combine, RMSNorm, element-wise ops
// ----------------------------------------------------------------------------
__global__ void combine_kernel(CombineArgs a) {
  pdl_wait();
  const int b = blockIdx.x;  // rows in x: more than 65535 of them are allowed
  const int i = blockIdx.y * blockDim.x + threadIdx.x;
  if (i >= a.H) return;
  const int kp1 = a.k + 1;
  const float* P = a.partial + (size_t)b * kp1 * a.H + i;
  float acc = 0.0f;
  for (int j = 0; j < a.k; ++j)
    acc = __fadd_rn(acc, __fmul_rn(a.weights[(size_t)b * a.k + j], P[(size_t)j * a.H]));
  if (a.sgate) acc = __fadd_rn(acc, __fmul_rn(a.sgate[b], P[(size_t)a.k * a.H]));
  if (a.residual) acc = __fadd_rn(a.residual[(size_t)b * a.H + i], acc);
  a.out[(size_t)b * a.H + i] = acc;
}

// in == out is allowed (osm_rms_norm normalises in place): no __restrict__
// on them; each element is read before its own write
__global__ void rmsnorm_kernel(const float* in, float* out, int dim, const float* __restrict__ w,
                               float eps, int exact) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  __shared__ float s_sum;
  const float* v = in + (size_t)blockIdx.x * dim;
  float* o = out + (size_t)blockIdx.x * dim;
  float sum;
  if (exact) {
    if (threadIdx.x == 0) {
      float s = 0.0f;
      for (int i = 0; i < dim; ++i) s = __fadd_rn(s, __fmul_rn(v[i], v[i]));
      s_sum = s;
    }
    __syncthreads();
    sum = s_sum;
  } else {
    float s = 0.0f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) s = fmaf(v[i], v[i], s);
    sum = block_reduce_sum(s, red);
  }
  const float scale =
      __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)dim), eps)));
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float ww = w ? w[i] : 1.0f;
    o[i] = __fmul_rn(v[i], __fmul_rn(scale, ww));
  }
}

// Affine metadata element i: bf16 bits (the slot format) or fp32.
__device__ __forceinline__ float meta_at(const uint16_t* p, size_t i) {
  return bf16_bits_to_f32(p[i]);
}
__device__ __forceinline__ float meta_at(const float* p, size_t i) { return p[i]; }

template <typename M>
__global__ void dequant_kernel(const uint32_t* __restrict__ packed, const M* __restrict__ sc,
                               const M* __restrict__ bi, int rows, int K, int group,
                               float* __restrict__ out) {
  const size_t total = (size_t)rows * K;
  const int G = K / group;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t row = i / K;
    const int col = (int)(i - row * K);
    const uint32_t q = (packed[row * (K >> 3) + (col >> 3)] >> ((col & 7) * 4)) & 0xFu;
    const float s = meta_at(sc, row * G + col / group);
    const float b = meta_at(bi, row * G + col / group);
    out[i] = __fadd_rn(__fmul_rn(s, (float)q), b);
  }
}

// Any-geometry affine Q4 GEMV (group dividing K, K a multiple of 8): one warp
// per (token, row), each lane a strided run of packed words, the dequantised
// weight formed as in dequant_kernel.  Serves the small and odd shapes the
// row-tiled projection kernels do not take (group sizes other than 64, K not
// a multiple of 64, fp32 metadata); not a hot path.
template <typename M>
__global__ void gemv_any_kernel(const uint32_t* __restrict__ packed, const M* __restrict__ sc,
                                const M* __restrict__ bi, int rows, int K, int group,
                                const float* __restrict__ x, int tokens, float* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const size_t warps = ((size_t)gridDim.x * blockDim.x) >> 5;
  const int W = K >> 3, G = K / group;
  for (size_t w = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5; w < (size_t)rows * tokens;
       w += warps) {
    const int t = (int)(w / rows), r = (int)(w - (size_t)t * rows);
    const uint32_t* pr = packed + (size_t)r * W;
    const float* xt = x + (size_t)t * K;
    float acc = 0.0f;
    for (int word = lane; word < W; word += 32) {
      const uint32_t p = pr[word];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = word * 8 + j, g = c / group;
        const float s = meta_at(sc, (size_t)r * G + g);
        const float b = meta_at(bi, (size_t)r * G + g);
        acc = fmaf(__fadd_rn(__fmul_rn(s, (float)((p >> (4 * j)) & 0xFu)), b), xt[c], acc);
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) y[(size_t)t * rows + r] = acc;
  }
}

__global__ void swiglu_kernel(const float* g, const float* u, float* o, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    o[i] = __fmul_rn(ref_silu(g[i]), u[i]);
}

__global__ void waccum_kernel(const float* src, float w, float* acc, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    acc[i] = __fadd_rn(acc[i], __fmul_rn(w, src[i]));
}

// ----------------------------------------------------------------------------
// Synthetic data
// ----------------------------------------------------------------------------
__device__ __forceinline__ float gen_one(uint64_t base, uint64_t idx, float sigma) {
  const uint64_t h1 = splitmix64(base + idx);
  const uint64_t h2 = splitmix64(h1);
  const double u1 = (double)((h1 >> 11) + 1) * 0x1.0p-53;
  const double u2 = (double)(h2 >> 11) * 0x1.0p-53;
  const double r = sqrt(-2.0 * log(u1));
  const double v = r * cos(6.283185307179586 * u2);
  return __fmul_rn((float)v, sigma);
}

__global__ void gen_normal_kernel(uint64_t base, float sigma, float* out, size_t n, size_t first) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    out[i] = gen_one(base, first + i, sigma);
}

// One thread per (row, group of 64): single_expert_pilot.cpp:276-346.
__global__ void gen_quant_kernel(uint64_t base, float sigma, int rows, int cols,
                                 uint32_t* __restrict__ packed, uint16_t* __restrict__ sc,
                                 uint16_t* __restrict__ bi) {
  const int G = cols >> 6;
  const size_t total = (size_t)rows * G;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t row = i / G;
    const int g = (int)(i - row * G);
    const uint64_t first = row * (uint64_t)cols + (uint64_t)g * 64;
    float v[64];
    float mn = INFINITY, mx = -INFINITY;
#pragma unroll 8
    for (int q = 0; q < 64; ++q) {
      v[q] = gen_one(base, first + q, sigma);
      if (v[q] < mn) mn = v[q];
      if (mx < v[q]) mx = v[q];
    }
    const float range = __fsub_rn(mx, mn);
    const float scale = range > 0.0f ? __fdiv_rn(range, 15.0f) : 1.0f;
    const float bias = mn;
    uint32_t* pw = packed + row * (size_t)(cols >> 3) + g * 8;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      uint32_t word = 0;
#pragma unroll
      for (int l = 0; l < 8; ++l) {
        const float nrm = __fdiv_rn(__fsub_rn(v[w * 8 + l], bias), scale);
        long r = lroundf(nrm);
        r = r < 0 ? 0 : (r > 15 ? 15 : r);
        word |= (uint32_t)r << (4 * l);
      }
      pw[w] = word;
    }
    sc[i] = (uint16_t)f32_to_bf16_rne(scale);
    bi[i] = (uint16_t)f32_to_bf16_rne(bias);
  }
}

__global__ void router_pack_kernel(const float* __restrict__ w, RouterGeom g,
                                   void* __restrict__ wp) {
  const size_t total = (size_t)g.E * g.Hp;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t e = i / g.Hp;
    const int h = (int)(i - e * g.Hp);
    const float v = h < g.H ? w[e * g.H + h] : 0.0f;
    const int l = h / g.c, o = h - l * g.c;
    const size_t idx = ((e * g.nvec + (o >> 3)) * 32 + l) * 8 + (o & 7);
    if (g.f32w) reinterpret_cast<float*>(wp)[idx] = v;
    else reinterpret_cast<uint16_t*>(wp)[idx] = (uint16_t)f32_to_bf16_rne(v);
  }
}

__global__ void router_tile_kernel(const float* __restrict__ w, RouterGeom g,
                                   unsigned char* __restrict__ wx) {
  const int esz = g.f32w ? 4 : 2, hpt = 128 / esz, epc = 16 / esz;
  const int nht = g.H / hpt;
  const int Ep = (g.E + 127) & ~127;
  const size_t total = (size_t)Ep * g.H;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int e = (int)(i / g.H), h = (int)(i - (size_t)e * g.H);
    const float v = e < g.E ? w[(size_t)e * g.H + h] : 0.0f;
    const int eb = e >> 7, r = e & 127, ht = h / hpt, hh = h - ht * hpt;
    const int c = hh / epc, p = hh - c * epc;
    const size_t off = (((size_t)eb * nht + ht) * 128 + r) * 128 + (size_t)((c ^ (r & 7)) * 16) + (size_t)p * esz;
    if (g.f32w) *reinterpret_cast<float*>(wx + off) = v;
    else *reinterpret_cast<uint16_t*>(wx + off) = (uint16_t)f32_to_bf16_rne(v);
  }
}

// q8 router layouts, from the byte matrix q [E][H]: the lane-chunk vectors of
// router_pack_kernel with one byte per element, and 16 KB tiles of 128
// experts x 128 bytes (128 values of h) with the same 16-byte chunk swizzle.
__global__ void router_pack_q8_kernel(const uint8_t* __restrict__ q, RouterGeom g,
                                      uint8_t* __restrict__ wp) {
  const size_t total = (size_t)g.E * g.Hp;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t e = i / g.Hp;
    const int h = (int)(i - e * g.Hp);
    const int l = h / g.c, o = h - l * g.c;
    wp[((e * g.nvec + (o >> 3)) * 32 + l) * 8 + (o & 7)] = h < g.H ? q[e * g.H + h] : 0;
  }
}

__global__ void router_tile_q8_kernel(const uint8_t* __restrict__ q, RouterGeom g,
                                      unsigned char* __restrict__ wx) {
  const int nht = g.H / 128;
  const int Ep = (g.E + 127) & ~127;
  const size_t total = (size_t)Ep * g.H;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int e = (int)(i / g.H), h = (int)(i - (size_t)e * g.H);
    const int eb = e >> 7, r = e & 127, ht = h >> 7, hh = h & 127;
    const int c = hh >> 4, p = hh & 15;
    wx[(((size_t)eb * nht + ht) * 128 + r) * 128 + (size_t)((c ^ (r & 7)) * 16) + p] =
        e < g.E ? q[(size_t)e * g.H + h] : 0;
  }
}

inline int grid_for(size_t n, int threads) {
  size_t b = (n + threads - 1) / threads;
  if (b > 148 * 64) b = 148 * 64;
  if (b < 1) b = 1;
  return (int)b;
}

}  // namespace

__global__ void slot_updates_kernel(const SlotUpdates u) {
  // in order: a later write to the same entry wins
  if (threadIdx.x == 0)
    for (int i = 0; i < u.n; ++i) *u.ptr[i] = u.val[i];
}

// Copies n16 16-byte words between this GPU's memory and pinned host memory
// that the GPU maps (unified addressing: the host pointer is the device
// pointer).  One word per thread per pass; each warp's 512 bytes go over PCIe
// as full-line reads or posted writes.  after_pdl: the kernel was launched as
// a programmatic dependent and waits for its predecessor before it reads.
__global__ void __launch_bounds__(256) host_copy_kernel(const uint4* __restrict__ src,
                                                        uint4* __restrict__ dst, size_t n16,
                                                        int after_pdl) {
  if (after_pdl) pdl_wait();
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n16; i += stride)
    dst[i] = src[i];
}

cudaError_t launch_host_copy(void* dst, const void* src, size_t bytes, bool after_pdl, int num_sms,
                             cudaStream_t s, uint64_t* launches) {
  const size_t n16 = bytes / 16;
  if (n16 == 0) return cudaSuccess;
  size_t blocks = (n16 + 255) / 256;
  const size_t cap = (size_t)2 * (num_sms > 0 ? num_sms : 148);
  if (blocks > cap) blocks = cap;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = after_pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, host_copy_kernel, static_cast<const uint4*>(src),
                                           static_cast<uint4*>(dst), n16, after_pdl ? 1 : 0);
  if (e == cudaSuccess && launches) *launches += 1;
  return e;
}

void launch_slot_updates(const SlotUpdates& u, cudaStream_t s, uint64_t* launches) {
  if (u.n <= 0) return;
  slot_updates_kernel<<<1, 32, 0, s>>>(u);
  if (launches) *launches += 1;
}

void launch_combine(const CombineArgs& a, cudaStream_t s, uint64_t* launches) {
  const dim3 grid(a.B, (a.H + 255) / 256);
  combine_kernel<<<grid, 256, 0, s>>>(a);
  if (launches) *launches += 1;
}

void launch_rmsnorm(const float* in, float* out, int rows, int dim, const float* w, float eps,
                    bool exact, cudaStream_t s, uint64_t* launches) {
  rmsnorm_kernel<<<rows, 256, 0, s>>>(in, out, dim, w, eps, exact ? 1 : 0);
  if (launches) *launches += 1;
}

void launch_dequant(const uint32_t* packed, const void* sc, const void* bi, bool f32_meta,
                    int rows, int K, int group, float* out, cudaStream_t s, uint64_t* launches) {
  const int grid = grid_for((size_t)rows * K, 256);
  if (f32_meta)
    dequant_kernel<float><<<grid, 256, 0, s>>>(packed, static_cast<const float*>(sc),
                                               static_cast<const float*>(bi), rows, K, group, out);
  else
    dequant_kernel<uint16_t><<<grid, 256, 0, s>>>(packed, static_cast<const uint16_t*>(sc),
                                                  static_cast<const uint16_t*>(bi), rows, K, group,
                                                  out);
  if (launches) *launches += 1;
}

void launch_gemv_any(const uint32_t* packed, const void* sc, const void* bi, bool f32_meta,
                     int rows, int K, int group, const float* x, int tokens, float* y,
                     cudaStream_t s, uint64_t* launches) {
  const int grid = grid_for((size_t)rows * tokens * 32, 256);
  if (f32_meta)
    gemv_any_kernel<float><<<grid, 256, 0, s>>>(packed, static_cast<const float*>(sc),
                                                static_cast<const float*>(bi), rows, K, group, x,
                                                tokens, y);
  else
    gemv_any_kernel<uint16_t><<<grid, 256, 0, s>>>(packed, static_cast<const uint16_t*>(sc),
                                                   static_cast<const uint16_t*>(bi), rows, K, group,
                                                   x, tokens, y);
  if (launches) *launches += 1;
}

void launch_swiglu(const float* g, const float* u, float* out, size_t n, cudaStream_t s,
                   uint64_t* launches) {
  swiglu_kernel<<<grid_for(n, 256), 256, 0, s>>>(g, u, out, n);
  if (launches) *launches += 1;
}

void launch_waccum(const float* src, float w, float* acc, size_t n, cudaStream_t s,
                   uint64_t* launches) {
  waccum_kernel<<<grid_for(n, 256), 256, 0, s>>>(src, w, acc, n);
  if (launches) *launches += 1;
}

static uint64_t stream_base(uint64_t seed, uint64_t tensor) {
  auto sm = [](uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  };
  return sm(seed ^ sm(tensor));
}

void launch_gen_normal(uint64_t seed, uint64_t tensor, float sigma, float* out, size_t n,
                       size_t first, cudaStream_t s, uint64_t* launches) {
  gen_normal_kernel<<<grid_for(n, 256), 256, 0, s>>>(stream_base(seed, tensor), sigma, out, n,
                                                       first);
  if (launches) *launches += 1;
}

void launch_gen_quant(uint64_t seed, uint64_t tensor, float sigma, int rows, int cols,
                      uint32_t* packed, uint16_t* sc, uint16_t* bi, cudaStream_t s,
                      uint64_t* launches) {
  const size_t n = (size_t)rows * (cols >> 6);
  gen_quant_kernel<<<grid_for(n, 128), 128, 0, s>>>(stream_base(seed, tensor), sigma, rows, cols,
                                                     packed, sc, bi);
  if (launches) *launches += 1;
}

size_t router_tile_bytes(const RouterGeom& g) {
  return (size_t)((g.E + 127) & ~127) * g.H * (g.q8 ? 1 : g.f32w ? 4 : 2);
}

void launch_router_pack_q8(const uint8_t* q, const RouterGeom& g, void* wp, cudaStream_t s,
                           uint64_t* launches) {
  router_pack_q8_kernel<<<grid_for((size_t)g.E * g.Hp, 256), 256, 0, s>>>(q, g,
                                                                          static_cast<uint8_t*>(wp));
  if (launches) *launches += 1;
}

void launch_router_tile_q8(const uint8_t* q, const RouterGeom& g, void* wx, cudaStream_t s,
                           uint64_t* launches) {
  router_tile_q8_kernel<<<grid_for((size_t)((g.E + 127) & ~127) * g.H, 256), 256, 0, s>>>(
      q, g, static_cast<unsigned char*>(wx));
  if (launches) *launches += 1;
}

void launch_router_tile(const float* w, const RouterGeom& g, void* wx, cudaStream_t s,
                        uint64_t* launches) {
  router_tile_kernel<<<grid_for((size_t)((g.E + 127) & ~127) * g.H, 256), 256, 0, s>>>(
      w, g, static_cast<unsigned char*>(wx));
  if (launches) *launches += 1;
}

void launch_router_pack(const float* w, const RouterGeom& g, void* wp, cudaStream_t s,
                        uint64_t* launches) {
  router_pack_kernel<<<grid_for((size_t)g.E * g.Hp, 256), 256, 0, s>>>(w, g, wp);
  if (launches) *launches += 1;
}

}  // namespace osm
