// osm_ep.cu -- expert parallelism over NVLink peer memory.
//
// Every rank owns one EP block (osm_ep_layout): a receive region per source
// rank ((token, pick) rows in fp16 with their owner-local expert id, routing
// weight and the source's pair index), one more region for its own tokens'
// shared-expert rows, a back buffer that owners fill with the weighted
// results of this rank's pairs, and the barrier flags.  The blocks of the
// other ranks are mapped through CUDA IPC, so the kernels below store straight
// into a peer's memory (plain st.global over NVLink; no multicast, no TMA).
//
//   ep_dispatch_kernel  one warp per (token, pick): claims the next slot of
//                       its region in the owner's block, converts x to fp16
//                       into it and writes the slot's id, weight and pair
//                       index; then the shared-expert rows into the own block
//   ep_barrier_kernel   signals every rank (release, system scope) and waits
//                       for every rank's signal of the same epoch, bounded in
//                       time (status bit 7 when a rank does not arrive)
//   ep_return_kernel    on the owner, after its experts ran over all regions:
//                       each filled slot's fp16 result row times its routing
//                       weight (rounded to fp16 once), stored into the source
//                       rank's back buffer at the pair's index; the slot's id
//                       goes back to "empty" for the next call
//   ep_combine_kernel   on the source: each token's back rows summed in pick
//                       order in fp32, then its shared-expert row -- the
//                       accumulation order of run_qwen_sparse_moe_vulkan_accum
//                       (src/model/routed_moe.cpp:396-404)
//
// A slot's place inside its region is claimed with an atomic and is
// therefore not deterministic, but no result depends on it: every pair's
// expert output is computed on its own row, and the sums run in pick order
// on the source.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "osm_common.cuh"
#include "osm_kernels.cuh"

namespace osm {
namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ep_now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// eight fp32 values -> eight fp16 values (round to nearest), with a flag when
// one of them is beyond the fp16 range
__device__ __forceinline__ uint4 to_f16x8(float4 p, float4 q, bool& over) {
  over |= fabsf(p.x) >= 65504.0f || fabsf(p.y) >= 65504.0f || fabsf(p.z) >= 65504.0f ||
          fabsf(p.w) >= 65504.0f || fabsf(q.x) >= 65504.0f || fabsf(q.y) >= 65504.0f ||
          fabsf(q.z) >= 65504.0f || fabsf(q.w) >= 65504.0f;
  const __half2 a = __floats2half2_rn(p.x, p.y), b = __floats2half2_rn(p.z, p.w);
  const __half2 c = __floats2half2_rn(q.x, q.y), d = __floats2half2_rn(q.z, q.w);
  return make_uint4(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b),
                    *reinterpret_cast<const uint32_t*>(&c), *reinterpret_cast<const uint32_t*>(&d));
}

constexpr int kDispWarps = 8;

__global__ void __launch_bounds__(kDispWarps * 32) ep_dispatch_kernel(EpArgs a) {
  const EpLayout& L = a.lay;
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kDispWarps + (threadIdx.x >> 5);
  const int nw = gridDim.x * kDispWarps;
  const int nk = a.T * L.k;
  const int total = nk + (L.shared ? a.T : 0);
  const int nch = L.H >> 3;  // 8-value chunks of a row
  bool over = false;
  for (int p = gw; p < total; p += nw) {
    int t, region, pos;
    uint32_t le;
    float wgt;
    int32_t src;
    unsigned char* dst;
    if (p < nk) {
      t = p / L.k;
      const uint32_t id = a.ids[p];
      const uint32_t o = id / (uint32_t)L.e_local;
      if (o >= (uint32_t)L.world) {
        if (lane == 0) atomicOr(a.status, kStatusBadSlot);
        continue;
      }
      le = id - o * (uint32_t)L.e_local;
      wgt = a.w[p];
      src = p;
      region = L.rank;
      int claimed = 0;
      if (lane == 0) claimed = atomicAdd(a.send_cnt + o, 1);
      pos = __shfl_sync(0xFFFFFFFFu, claimed, 0);
      if (pos >= L.cap) {  // cannot happen: a source sends at most T_r * k pairs
        if (lane == 0) atomicOr(a.status, kStatusBadSlot);
        continue;
      }
      dst = a.peer[o];
    } else {
      t = p - nk;
      le = (uint32_t)L.e_local;  // the shared expert's local id
      wgt = a.sgate[t];
      src = L.T_r * L.k + t;
      region = L.world;
      pos = t;
      dst = a.peer[L.rank];
    }
    const size_t slot = (size_t)region * L.cap + pos;
    const float4* xr = reinterpret_cast<const float4*>(a.x + (size_t)t * L.H);
    uint4* rr = reinterpret_cast<uint4*>(dst + L.o_rows + slot * (size_t)L.H * 2);
    for (int c0 = 0; c0 < nch; c0 += 4 * 32) {  // a lane's loads before its stores
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = c0 + u * 32 + lane;
        v[2 * u] = c < nch ? xr[2 * c] : make_float4(0.f, 0.f, 0.f, 0.f);
        v[2 * u + 1] = c < nch ? xr[2 * c + 1] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < nch) rr[c] = to_f16x8(v[2 * u], v[2 * u + 1], over);
      }
    }
    if (lane == 0) {
      reinterpret_cast<uint32_t*>(dst + L.o_ids)[slot] = le;
      reinterpret_cast<float*>(dst + L.o_wts)[slot] = wgt;
      reinterpret_cast<int32_t*>(dst + L.o_src)[slot] = src;
    }
  }
  if (__any_sync(0xFFFFFFFFu, over) && lane == 0) atomicOr(a.status, kStatusF16Range);
  __threadfence_system();
}

__global__ void ep_barrier_kernel(EpArgs a, uint32_t epoch, unsigned long long timeout_ns) {
  const EpLayout& L = a.lay;
  const int i = threadIdx.x;
  __threadfence_system();
  __syncthreads();
  if (i < L.world) st_release_sys(reinterpret_cast<uint32_t*>(a.peer[i] + L.o_flags) + L.rank, epoch);
  if (i < L.world) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(a.peer[L.rank] + L.o_flags) + i;
    const unsigned long long t0 = ep_now_ns();
    while ((int32_t)(ld_acquire_sys(f) - epoch) < 0) {
      if (ep_now_ns() - t0 > timeout_ns) {
        atomicOr(a.status, kStatusPeerTimeout);
        break;
      }
      __nanosleep(200);
    }
  }
  __syncthreads();
}

// One warp per receive slot (grid-stride over all regions): a filled slot's
// result row (fp16, H / 8 chunks of 16 bytes, all of a lane's loads issued
// before its stores) times the slot's weight, to the source's back rows.
constexpr int kRetWarps = 8;
__global__ void __launch_bounds__(kRetWarps * 32) ep_return_kernel(EpArgs a, const uint16_t* __restrict__ pb,
                                                              const int* __restrict__ tp_pos) {
  const EpLayout& L = a.lay;
  const int lane = threadIdx.x & 31;
  const size_t nslots = (size_t)(L.world + 1) * L.cap;
  const int nch = L.H >> 3;  // <= 1024: at most 32 chunks per lane
  unsigned char* own = a.peer[L.rank];
  uint32_t* ids = reinterpret_cast<uint32_t*>(own + L.o_ids);
  bool over = false, bad = false;
  for (size_t slot = (size_t)blockIdx.x * kRetWarps + (threadIdx.x >> 5); slot < nslots;
       slot += (size_t)gridDim.x * kRetWarps) {
    const uint32_t id = ids[slot];
    if (id == kEpEmpty) continue;
    __syncwarp();
    if (lane == 0) ids[slot] = kEpEmpty;  // empty again for the next call
    if (id >= (uint32_t)(L.e_local + L.shared)) {  // never written by ep_dispatch_kernel
      bad = true;
      continue;
    }
    const int region = (int)(slot / L.cap);
    const float wgt = reinterpret_cast<const float*>(own + L.o_wts)[slot];
    const int32_t src = reinterpret_cast<const int32_t*>(own + L.o_src)[slot];
    const uint4* in = reinterpret_cast<const uint4*>(pb + (size_t)tp_pos[slot] * L.H);
    unsigned char* dst = region < L.world ? a.peer[region] : own;
    uint4* outp = reinterpret_cast<uint4*>(dst + L.o_back + (size_t)src * L.H * 2);
    for (int c0 = 0; c0 < nch; c0 += 8 * 32) {
      uint4 q[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + u * 32 + lane;
        q[u] = c < nch ? in[c] : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c >= nch) break;
        const uint32_t qq[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
        float v[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&qq[j]));
          v[2 * j] = __fmul_rn(wgt, f.x);
          v[2 * j + 1] = __fmul_rn(wgt, f.y);
        }
        outp[c] = to_f16x8(make_float4(v[0], v[1], v[2], v[3]), make_float4(v[4], v[5], v[6], v[7]),
                           over);
      }
    }
  }
  if (__any_sync(0xFFFFFFFFu, over) && lane == 0) atomicOr(a.status, kStatusF16Range);
  if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) atomicOr(a.status, kStatusBadSlot);
  __threadfence_system();
}

// grid (T, ceil(H / 8 / 256)), 256 threads
__global__ void __launch_bounds__(256) ep_combine_kernel(EpArgs a, float* __restrict__ out) {
  const EpLayout& L = a.lay;
  const int t = blockIdx.x;
  const int i = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (i >= L.H) return;
  const uint16_t* back = reinterpret_cast<const uint16_t*>(a.peer[L.rank] + L.o_back);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  auto add_row = [&](size_t r) {
    const uint4 q = *reinterpret_cast<const uint4*>(back + r * L.H + i);
    const uint32_t qq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&qq[u]));
      acc[2 * u] = __fadd_rn(acc[2 * u], v.x);
      acc[2 * u + 1] = __fadd_rn(acc[2 * u + 1], v.y);
    }
  };
  for (int j = 0; j < L.k; ++j) add_row((size_t)t * L.k + j);
  if (L.shared) add_row((size_t)L.T_r * L.k + t);
  float* op = out + (size_t)t * L.H + i;
  *reinterpret_cast<float4*>(op) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  *reinterpret_cast<float4*>(op + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
}

// The empty-slot marker over every id of the block's regions.
__global__ void ep_clear_ids_kernel(uint32_t* ids, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    ids[i] = kEpEmpty;
}

}  // namespace

EpLayout ep_layout(int world, int rank, int T_r, int k, int H, int e_local, int shared) {
  auto up = [](size_t v) { return (v + 255) & ~(size_t)255; };
  EpLayout L{};
  L.world = world;
  L.rank = rank;
  L.T_r = T_r;
  L.k = k;
  L.H = H;
  L.e_local = e_local;
  L.shared = shared;
  L.cap = T_r * k > T_r ? T_r * k : T_r;
  const size_t slots = (size_t)(world + 1) * L.cap;
  size_t o = 0;
  L.o_rows = o;  o = up(o + slots * (size_t)H * 2);
  L.o_ids = o;   o = up(o + slots * 4);
  L.o_wts = o;   o = up(o + slots * 4);
  L.o_src = o;   o = up(o + slots * 4);
  L.o_back = o;  o = up(o + ((size_t)T_r * k + T_r) * (size_t)H * 2);
  L.o_flags = o; o = up(o + 4 * 64);
  L.o_cnt = o;   o = up(o + 4 * 64);
  L.total = o;
  return L;
}

void launch_ep_clear_ids(const EpLayout& L, unsigned char* own, cudaStream_t s, uint64_t* launches) {
  const size_t n = (size_t)(L.world + 1) * L.cap;
  ep_clear_ids_kernel<<<(unsigned)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096), 256, 0, s>>>(
      reinterpret_cast<uint32_t*>(own + L.o_ids), n);
  if (launches) *launches += 1;
}

void launch_ep_dispatch(const EpArgs& a, int num_sms, cudaStream_t s, uint64_t* launches) {
  const int total = a.T * a.lay.k + (a.lay.shared ? a.T : 0);
  int blocks = (total + kDispWarps - 1) / kDispWarps;
  if (blocks > num_sms * 8) blocks = num_sms * 8;
  if (blocks < 1) blocks = 1;
  ep_dispatch_kernel<<<blocks, kDispWarps * 32, 0, s>>>(a);
  if (launches) *launches += 1;
}

void launch_ep_barrier(const EpArgs& a, uint32_t epoch, uint64_t timeout_ns, cudaStream_t s,
                       uint64_t* launches) {
  ep_barrier_kernel<<<1, 32, 0, s>>>(a, epoch, (unsigned long long)timeout_ns);
  if (launches) *launches += 1;
}

void launch_ep_return(const EpArgs& a, const uint16_t* pb, const int* tp_pos, int num_sms,
                      cudaStream_t s, uint64_t* launches) {
  const size_t nslots = (size_t)(a.lay.world + 1) * a.lay.cap;
  size_t blocks = (nslots + kRetWarps - 1) / kRetWarps;
  if (blocks > (size_t)num_sms * 8) blocks = (size_t)num_sms * 8;
  ep_return_kernel<<<(unsigned)blocks, kRetWarps * 32, 0, s>>>(a, pb, tp_pos);
  if (launches) *launches += 1;
}

void launch_ep_combine(const EpArgs& a, float* out, cudaStream_t s, uint64_t* launches) {
  const dim3 grid((unsigned)a.T, (unsigned)((a.lay.H / 8 + 255) / 256));
  ep_combine_kernel<<<grid, 256, 0, s>>>(a, out);
  if (launches) *launches += 1;
}

}  // namespace osm
