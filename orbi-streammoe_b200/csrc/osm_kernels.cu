// osm_kernels.cu -- sm_100a kernels of the routed-MoE sublayer.
//
// Router (replaces route_qwen_top_k_cpu, src/model/qwen_router.cpp:11-94):
//   router_logits_kernel  fp32 CUDA-core logits, each with a rigorous bound on
//                         its distance to the reference's sequential fp32 sum
//                         (src/cpu/reference_ops.cpp:85-91).
//   router_select_kernel  one block per token: top-(k+1) by (logit desc, id
//                         asc); if every adjacent gap of the top k+1 exceeds
//                         twice the largest bound, the order provably equals
//                         the reference's, else the token is routed on an exact
//                         path that repeats the reference's arithmetic (sequential
//                         fp32 logits, softmax, stable top-k,
//                         reference_ops.cpp:130-212).  Also the shared-expert
//                         scalar gate, the activation fragments, and (last
//                         block) the grouping of (token, pick) pairs by expert.
// Experts (replace q4_gemv.comp / swiglu.comp / weighted_accumulate.comp):
//   proj_kernel<PAIRED>   Q4 projections on mma.sync m16n8k16: nibbles are
//                         exact integers in bf16 (A), activations are split
//                         into bf16 hi + lo (B, 16 significant bits), groups of
//                         64 are scaled in fp32: acc += s*sum(q x) + b*sum(x)
//                         (the group identity of shaders/q4_gemv.comp:44-60).
//                         PAIRED: gate row r and up row r share a thread, so
//                         SwiGLU is applied in registers.
//   combine_kernel        out = sum over picks in pick order of w*y, then the
//                         shared expert s*y, then the residual
//                         (src/model/routed_moe.cpp:13-92, :396-404;
//                         src/model/checkpoint_moe_sublayer.cpp:21-33).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "osm_common.cuh"
#include "osm_kernels.cuh"

namespace osm {

namespace {

constexpr float kU = 5.9604644775390625e-8f;  // 2^-24, unit roundoff of fp32

// ----------------------------------------------------------------------------
// Router: logits + error bounds
// ----------------------------------------------------------------------------
constexpr int kRtExp = 4;   // experts per warp
constexpr int kRtTok = 4;   // tokens per block
constexpr int kRtWarps = 4;

// Eight consecutive weights of lane chunk vector (e, m, lane): one uint4 of
// bf16 or two float4 of fp32, depending on the router storage.
__device__ __forceinline__ void load8(const RouterArgs& a, int e, int m, int lane, float w[8]) {
  const size_t v = ((size_t)e * a.g.nvec + m) * 32 + lane;
  if (a.g.f32w) {
    const float4* p = reinterpret_cast<const float4*>(a.wp) + 2 * v;
    const float4 x0 = __ldg(p), x1 = __ldg(p + 1);
    w[0] = x0.x; w[1] = x0.y; w[2] = x0.z; w[3] = x0.w;
    w[4] = x1.x; w[5] = x1.y; w[6] = x1.z; w[7] = x1.w;
  } else {
    const uint4 q = __ldg(a.wp + v);
    const uint32_t ww[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int jj = 0; jj < 8; ++jj)
      w[jj] = bf16_bits_to_f32((ww[jj >> 1] >> ((jj & 1) * 16)) & 0xFFFFu);
  }
}

__global__ void __launch_bounds__(kRtWarps * 32)
router_logits_kernel(RouterArgs a) {
  extern __shared__ float4 smem4[];
  float* xs = reinterpret_cast<float*>(smem4);
  const RouterGeom g = a.g;
  const int t0 = blockIdx.y * kRtTok;
  // Stage x for kRtTok tokens in the lane-chunk layout of the weights.
  for (int i = threadIdx.x; i < kRtTok * g.Hp; i += blockDim.x) {
    const int t = i / g.Hp, h = i - t * g.Hp;
    float v = 0.0f;
    if (h < g.H && t0 + t < a.B) v = a.x[(size_t)(t0 + t) * g.H + h];
    const int l = h / g.c, o = h - l * g.c;
    xs[(((t * g.nvec + (o >> 3)) * 32 + l) << 3) + (o & 7)] = v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e0 = (blockIdx.x * kRtWarps + warp) * kRtExp;
  if (e0 >= g.E) return;
  float tacc[kRtExp][kRtTok], aacc[kRtExp][kRtTok], sacc[kRtExp][kRtTok];
#pragma unroll
  for (int q = 0; q < kRtExp; ++q)
#pragma unroll
    for (int t = 0; t < kRtTok; ++t) tacc[q][t] = aacc[q][t] = sacc[q][t] = 0.0f;

  for (int m = 0; m < g.nvec; ++m) {
    float wv[kRtExp][8];
#pragma unroll
    for (int q = 0; q < kRtExp; ++q) {
      const int e = e0 + q;
      if (e < g.E) {
        load8(a, e, m, lane, wv[q]);
      } else {
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) wv[q][jj] = 0.0f;
      }
    }
#pragma unroll
    for (int t = 0; t < kRtTok; ++t) {
      const float4* xp = reinterpret_cast<const float4*>(xs + (((t * g.nvec + m) * 32 + lane) << 3));
      const float4 xa = xp[0], xb = xp[1];
      const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
      for (int q = 0; q < kRtExp; ++q) {
        // |partial sum| at the start of this 8-element block: the partial
        // sums inside the block are bounded by it plus the block's |w x|.
        sacc[q][t] += fabsf(tacc[q][t]);
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const float w = wv[q][jj];
          tacc[q][t] = fmaf(w, xv[jj], tacc[q][t]);
          aacc[q][t] = fmaf(fabsf(w), fabsf(xv[jj]), aacc[q][t]);
        }
      }
    }
  }
  // n*gamma_n with n = Hp (gamma_n = n u / (1 - n u)).
  const float n = (float)g.Hp;
  const float gam = n * kU / (1.0f - n * kU);
#pragma unroll
  for (int q = 0; q < kRtExp; ++q) {
#pragma unroll
    for (int t = 0; t < kRtTok; ++t) {
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
      // |fast - exact| + |reference sequential - exact| (running error
      // bounds; chunk prefix P_l and in-chunk partials t_{l,o} bound every
      // partial sum of the sequential order: |s_i| <= |P_l| + |t_{l,o}|).
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
}

// ----------------------------------------------------------------------------
// Router: selection (fast certified path / exact path), scalar gate,
// fragments, grouping
// ----------------------------------------------------------------------------
constexpr int kSelThreads = 512;

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// Select the best n (<= E) of lane-strided values (index i*32 + lane) by
// (value desc, index asc).  Every lane receives the winners in order.
__device__ void warp_select(const float (&v)[32], int E, int n, int* sel_id, float* sel_v) {
  const int lane = threadIdx.x & 31;
  uint32_t taken = 0;
  for (int r = 0; r < n; ++r) {
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int id = i * 32 + lane;
      if (id < E && !((taken >> i) & 1u) && better(v[i], id, bv, bi)) {
        bv = v[i];
        bi = id;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
      const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
      if (better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    sel_id[r] = bi;
    sel_v[r] = bv;
  }
}

__device__ float block_reduce_sum(float v, float* red) {
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

__device__ float block_reduce_max(float v, float* red) {
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

// Block-wide exclusive scan of n (<= 4*blockDim) ints in smem `v`, in place;
// returns the total.
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

__device__ void group_pairs(const RouterArgs& a, int* sm_cnt, int* sm_cur, int* sm_flag,
                            int* red) {
  const int E = a.g.E, k = a.g.k, B = a.B;
  const int has_sh = a.shared_slot != nullptr;
  const int NE = E + has_sh;
  for (int i = threadIdx.x; i < NE; i += blockDim.x) {
    sm_cnt[i] = 0;
    sm_cur[i] = 0;
  }
  __syncthreads();
  for (int p = threadIdx.x; p < B * k; p += blockDim.x) {
    const uint32_t e = __ldcg(a.ids + p);
    if (e < (uint32_t)E) atomicAdd(&sm_cnt[e], 1);
    else atomicOr(a.status, kStatusBadSlot);
  }
  if (has_sh && threadIdx.x == 0) sm_cnt[E] = B;
  __syncthreads();
  for (int i = threadIdx.x; i < NE; i += blockDim.x) sm_flag[i] = sm_cnt[i] > 0 ? 1 : 0;
  __syncthreads();
  // sm_flag -> active index, sm_cnt kept; offsets into sm_cur (copy, scan)
  const int n_active = block_exclusive_scan(sm_flag, NE, red);
  for (int i = threadIdx.x; i < NE; i += blockDim.x) sm_cur[i] = sm_cnt[i];
  __syncthreads();
  block_exclusive_scan(sm_cur, NE, red);  // sm_cur = offsets
  for (int e = threadIdx.x; e < NE; e += blockDim.x) {
    if (sm_cnt[e] == 0) continue;
    const int j = sm_flag[e];
    a.act_off[j] = sm_cur[e];
    a.act_cnt[j] = sm_cnt[e];
    if (e == E) {
      a.act_kind[j] = 1;
      a.act_ptr[j] = a.shared_slot;
    } else {
      a.act_kind[j] = 0;
      const int slot = a.slot_of[e];
      if (slot < 0) {
        atomicOr(a.status, kStatusNotResident);
        a.act_ptr[j] = nullptr;
      } else {
        a.act_ptr[j] = a.slab + (size_t)slot * a.slab_stride;
      }
    }
  }
  __syncthreads();
  // scatter: reuse sm_cnt as per-expert cursors
  for (int i = threadIdx.x; i < NE; i += blockDim.x) sm_cnt[i] = 0;
  __syncthreads();
  for (int p = threadIdx.x; p < B * k; p += blockDim.x) {
    const uint32_t e = __ldcg(a.ids + p);
    if (e >= (uint32_t)E) continue;
    const int pos = sm_cur[e] + atomicAdd(&sm_cnt[e], 1);
    a.pair_tok[pos] = p / k;
    a.pair_pick[pos] = p % k;
  }
  if (has_sh)
    for (int t = threadIdx.x; t < B; t += blockDim.x) {
      a.pair_tok[sm_cur[E] + t] = t;
      a.pair_pick[sm_cur[E] + t] = k;
    }
  if (threadIdx.x == 0) *a.n_active = n_active;
}

__global__ void __launch_bounds__(kSelThreads) router_select_kernel(RouterArgs a) {
  extern __shared__ float4 smem4[];
  float* xs = reinterpret_cast<float*>(smem4);   // [H]
  float* lex = xs + a.g.H;                        // [E] exact logits / exps
  float* pex = lex + a.g.E;                       // [E] exact probabilities
  __shared__ float red[32];
  __shared__ int sel_id[kMaxTopK + 1];
  __shared__ float sel_v[kMaxTopK + 1];
  __shared__ int s_flag;
  __shared__ float s_bcast;
  const RouterGeom g = a.g;
  const int tok = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* x = a.x + (size_t)tok * g.H;
  int nonfinite = 0;
  for (int h = tid; h < g.H; h += blockDim.x) {
    const float v = x[h];
    xs[h] = v;
    if (!isfinite(v)) nonfinite = 1;
  }
  nonfinite = __syncthreads_or(nonfinite);
  if (tid == 0) s_flag = 0;
  __syncthreads();
  if (nonfinite) {
    if (tid == 0) atomicOr(a.status, kStatusNonFinite);
  }
  const int k = g.k;
  // ---- fast path: certified top-k over the fast logits ----
  if (warp == 0 && !nonfinite && !a.skip_route) {
    float v[32];
    float bm = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int id = i * 32 + lane;
      v[i] = id < g.E ? a.logits[(size_t)tok * g.E + id] : -INFINITY;
      if (id < g.E) bm = fmaxf(bm, a.bounds[(size_t)tok * g.E + id]);
    }
    bm = warp_max(bm);
    const int nsel = k + 1 <= g.E ? k + 1 : k;
    warp_select(v, g.E, nsel, sel_id, sel_v);
    bool ok = !a.force_exact;
    // Certified when each adjacent gap exceeds twice the largest bound plus
    // a floor that keeps distinct logits at distinct probabilities after
    // exp and the division (|d| = distance to the max logit).
    const float mx0 = sel_v[0];
    for (int j = 0; j + 1 < nsel; ++j) {
      const float need = 2.0f * bm * 1.0001f + 1e-6f +
                         3e-7f * (fabsf(sel_v[j] - mx0) + fabsf(sel_v[j + 1] - mx0));
      if (!(__fsub_rd(sel_v[j], sel_v[j + 1]) > need)) ok = false;
    }
    if (!isfinite(sel_v[0])) ok = false;
    if (ok) {
      const float mx = sel_v[0];
      float s = 0.0f;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i * 32 + lane < g.E) s += expf(__fsub_rn(v[i], mx));
      s = warp_sum(s);
      if (lane == 0) {
        float p[kMaxTopK];
        float mass = 0.0f;
        for (int j = 0; j < k; ++j) {
          p[j] = __fdiv_rn(expf(__fsub_rn(sel_v[j], mx)), s);
          mass = __fadd_rn(mass, p[j]);
        }
        if (!(mass > 0.0f) || !isfinite(mass) || !(s > 0.0f) || !isfinite(s))
          atomicOr(a.status, kStatusBadMass);
        for (int j = 0; j < k; ++j) {
          const float w = a.norm ? __fdiv_rn(p[j], mass) : p[j];
          a.ids[(size_t)tok * k + j] = (uint32_t)sel_id[j];
          a.weights[(size_t)tok * k + j] = w;
        }
        a.mass[tok] = mass;
      }
    } else if (lane == 0) {
      s_flag = 1;
    }
  }
  __syncthreads();
  // ---- exact path: the reference's arithmetic, operation by operation ----
  if (s_flag && !nonfinite) {
    if (tid == 0) atomicAdd(a.exact_count, 1ull);
    for (int e = tid; e < g.E; e += blockDim.x) {
      float acc = 0.0f;
      for (int h8 = 0; h8 < g.H; h8 += 8) {
        const int l = h8 / g.c, o = h8 - l * g.c;
        float w8[8];
        load8(a, e, o >> 3, l, w8);
#pragma unroll
        for (int jj = 0; jj < 8; ++jj)
          if (h8 + jj < g.H) acc = __fadd_rn(acc, __fmul_rn(w8[jj], xs[h8 + jj]));
      }
      if (a.bias != nullptr) acc = __fadd_rn(acc, a.bias[e]);
      lex[e] = acc;
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
    for (int e = tid; e < g.E; e += blockDim.x) pex[e] = __fdiv_rn(lex[e], sum);
    __syncthreads();
    if (warp == 0) {
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int id = i * 32 + lane;
        v[i] = id < g.E ? pex[id] : -INFINITY;
      }
      warp_select(v, g.E, k, sel_id, sel_v);
      if (lane == 0) {
        float mass = 0.0f;
        for (int j = 0; j < k; ++j) mass = __fadd_rn(mass, sel_v[j]);
        if (!(mass > 0.0f) || !isfinite(mass)) atomicOr(a.status, kStatusBadMass);
        for (int j = 0; j < k; ++j) {
          a.ids[(size_t)tok * k + j] = (uint32_t)sel_id[j];
          a.weights[(size_t)tok * k + j] = a.norm ? __fdiv_rn(sel_v[j], mass) : sel_v[j];
        }
        a.mass[tok] = mass;
      }
    }
  }
  if (nonfinite && tid == 0 && !a.skip_route) {
    for (int j = 0; j < k; ++j) {
      a.ids[(size_t)tok * k + j] = 0;
      a.weights[(size_t)tok * k + j] = 0.0f;
    }
    a.mass[tok] = 0.0f;
  }
  __syncthreads();
  // user copies of the routing
  if (tid < k && !a.skip_route) {
    if (a.ids_out) a.ids_out[(size_t)tok * k + tid] = a.ids[(size_t)tok * k + tid];
    if (a.weights_out) a.weights_out[(size_t)tok * k + tid] = a.weights[(size_t)tok * k + tid];
  }
  if (tid == 0 && a.mass_out && !a.skip_route) a.mass_out[tok] = a.mass[tok];
  // ---- shared expert scalar gate: sigmoid(g . x) ----
  if (a.sgate_w != nullptr) {
    float d = 0.0f;
    for (int h = tid; h < g.H; h += blockDim.x) d = fmaf(a.sgate_w[h], xs[h], d);
    const float dot = block_reduce_sum(d, red);
    if (tid == 0) {
      const float s = ref_sigmoid(dot);
      a.sgate[tok] = s;
      if (a.sgate_out) a.sgate_out[tok] = s;
    }
  } else if (tid == 0) {
    if (a.sgate) a.sgate[tok] = 0.0f;
    if (a.sgate_out) a.sgate_out[tok] = 0.0f;
  }
  // ---- activation fragments for the expert kernels ----
  if (a.xfrag != nullptr) {
    const int nch = g.H >> 3;
    for (int c = tid; c < nch; c += blockDim.x) {
      const float* xc = xs + c * 8;
      uint32_t hi[8], lo[8];
      float fs = xc[0];
#pragma unroll
      for (int q = 0; q < 8; ++q) split_bf16(xc[q], hi[q], lo[q]);
#pragma unroll
      for (int q = 1; q < 8; ++q) fs = __fadd_rn(fs, xc[q]);
      uint4* dst = a.xfrag + ((size_t)tok * nch + c) * 2;
      dst[0] = make_uint4(pack2(hi[0], hi[4]), pack2(hi[1], hi[5]), pack2(hi[2], hi[6]),
                          pack2(hi[3], hi[7]));
      dst[1] = make_uint4(pack2(lo[0], lo[4]), pack2(lo[1], lo[5]), pack2(lo[2], lo[6]),
                          pack2(lo[3], lo[7]));
      a.xfsum8[(size_t)tok * nch + c] = fs;
    }
  }
  // ---- last block groups (token, pick) pairs by expert ----
  if (!a.do_group) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned int prev = atomicAdd(a.ticket, 1u);
    s_flag = (prev == gridDim.x - 1) ? 2 : 0;
  }
  __syncthreads();
  if (s_flag != 2) return;
  __threadfence();
  int* sm = reinterpret_cast<int*>(smem4);
  const int NE = g.E + 1;
  group_pairs(a, sm, sm + NE, sm + 2 * NE, reinterpret_cast<int*>(red));
  if (tid == 0) *a.ticket = 0u;
}

__global__ void __launch_bounds__(kSelThreads) group_kernel(RouterArgs a) {
  extern __shared__ float4 smem4[];
  __shared__ int red[32];
  int* sm = reinterpret_cast<int*>(smem4);
  const int NE = a.g.E + 1;
  group_pairs(a, sm, sm + NE, sm + 2 * NE, red);
}

// ----------------------------------------------------------------------------
// Activation fragments
// ----------------------------------------------------------------------------
__global__ void frag_prep_kernel(const float* __restrict__ x, int rows, int K,
                                 uint4* __restrict__ frag, float* __restrict__ fsum8) {
  const int nch = K >> 3;
  const size_t total = (size_t)rows * nch;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const float* xc = x + i * 8;
    float v[8];
    const float4 p = *reinterpret_cast<const float4*>(xc);
    const float4 q = *reinterpret_cast<const float4*>(xc + 4);
    v[0] = p.x; v[1] = p.y; v[2] = p.z; v[3] = p.w;
    v[4] = q.x; v[5] = q.y; v[6] = q.z; v[7] = q.w;
    uint32_t hi[8], lo[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) split_bf16(v[j], hi[j], lo[j]);
    float fs = v[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) fs = __fadd_rn(fs, v[j]);
    frag[i * 2] = make_uint4(pack2(hi[0], hi[4]), pack2(hi[1], hi[5]), pack2(hi[2], hi[6]),
                             pack2(hi[3], hi[7]));
    frag[i * 2 + 1] = make_uint4(pack2(lo[0], lo[4]), pack2(lo[1], lo[5]),
                                 pack2(lo[2], lo[6]), pack2(lo[3], lo[7]));
    fsum8[i] = fs;
  }
}

// ----------------------------------------------------------------------------
// Q4 projection tiles on mma.sync
// ----------------------------------------------------------------------------
constexpr int kProjWarps = 4;
constexpr int kMaxGPerWarp = 8;   // K <= 2048

// One 64-wide group for one tile: 2 words per row and thread, 4 k16 steps,
// hi and lo activation pieces.
__device__ __forceinline__ void mma_group(float d[4], uint2 wl, uint2 wh, uint4 xh0, uint4 xl0,
                                          uint4 xh1, uint4 xl1) {
#pragma unroll
  for (int jj = 0; jj < 2; ++jj) {
    const uint32_t wlo = jj ? wl.y : wl.x;
    const uint32_t whi = jj ? wh.y : wh.x;
    const uint4 xh = jj ? xh1 : xh0;
    const uint4 xl = jj ? xl1 : xl0;
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

template <bool PAIRED>
__global__ void __launch_bounds__(kProjWarps * 32) proj_kernel(ProjArgs a) {
  const int j = blockIdx.y;
  if (j >= *a.n_active) return;
  const uint8_t* base = a.act_ptr[j];
  const int kind = a.act_kind[j];
  if (base == nullptr && !a.raw) return;  // non-resident expert
  const int rows = a.sec.rows[kind], K = a.sec.K[kind];
  constexpr int kTileRows = PAIRED ? 8 : 16;
  const int r0 = blockIdx.x * kTileRows;
  if (r0 >= rows) return;
  const int G = K >> 6, KW = K >> 3;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, t = lane & 3;

  // base + offset as integers: in raw mode base is null and the offsets are
  // the projection's absolute addresses.
  const uintptr_t ub = reinterpret_cast<uintptr_t>(base);
  const uint32_t* Wlo = reinterpret_cast<const uint32_t*>(ub + a.sec.w[kind]);
  const uint16_t* Slo = reinterpret_cast<const uint16_t*>(ub + a.sec.s[kind]);
  const uint16_t* Blo = reinterpret_cast<const uint16_t*>(ub + a.sec.b[kind]);
  const uint32_t* Whi = PAIRED ? reinterpret_cast<const uint32_t*>(ub + a.sec.w2[kind]) : Wlo;
  const uint16_t* Shi = PAIRED ? reinterpret_cast<const uint16_t*>(ub + a.sec.s2[kind]) : Slo;
  const uint16_t* Bhi = PAIRED ? reinterpret_cast<const uint16_t*>(ub + a.sec.b2[kind]) : Blo;
  const int row_lo = r0 + gid;
  const int row_hi = PAIRED ? r0 + gid : r0 + 8 + gid;

  // Weights and metadata of this warp's groups stay in registers for every
  // token chunk of the expert.
  uint2 wl[kMaxGPerWarp], wh[kMaxGPerWarp];
  float sl[kMaxGPerWarp], bl[kMaxGPerWarp], sh[kMaxGPerWarp], bh[kMaxGPerWarp];
#pragma unroll
  for (int i = 0; i < kMaxGPerWarp; ++i) {
    const int g = warp + kProjWarps * i;
    if (g < G) {
      wl[i] = __ldg(reinterpret_cast<const uint2*>(Wlo + (size_t)row_lo * KW + g * 8 + 2 * t));
      wh[i] = __ldg(reinterpret_cast<const uint2*>(Whi + (size_t)row_hi * KW + g * 8 + 2 * t));
      sl[i] = bf16_bits_to_f32(__ldg(Slo + (size_t)row_lo * G + g));
      bl[i] = bf16_bits_to_f32(__ldg(Blo + (size_t)row_lo * G + g));
      sh[i] = bf16_bits_to_f32(__ldg(Shi + (size_t)row_hi * G + g));
      bh[i] = bf16_bits_to_f32(__ldg(Bhi + (size_t)row_hi * G + g));
    } else {
      wl[i] = wh[i] = make_uint2(0u, 0u);
      sl[i] = bl[i] = sh[i] = bh[i] = 0.0f;
    }
  }

  __shared__ float fsg[8][33];
  __shared__ float red[kProjWarps][32][4];
  __shared__ float hs[8][9];
  const int off = a.act_off[j], cnt = a.act_cnt[j];
  for (int c0 = 0; c0 < cnt; c0 += 8) {
    const int nv = min(8, cnt - c0);
    for (int i = threadIdx.x; i < 8 * G; i += blockDim.x) {
      const int n = i / G, g = i - n * G;
      float s = 0.0f;
      if (n < nv) {
        const int p = off + c0 + n;
        const int rr = a.frag_by_pair ? p : a.pair_tok[p];
        const float* f = a.fsum8 + (size_t)rr * a.frag_stride + g * 8;
        s = f[0];
#pragma unroll
        for (int q = 1; q < 8; ++q) s = __fadd_rn(s, f[q]);
      }
      fsg[n][g] = s;
    }
    __syncthreads();
    const bool has_tok = gid < nv;
    int my_row = 0;
    if (has_tok) {
      const int p = off + c0 + gid;
      my_row = a.frag_by_pair ? p : a.pair_tok[p];
    }
    const uint4* xf = a.frag + (size_t)my_row * a.frag_stride * 2;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int i = 0; i < kMaxGPerWarp; ++i) {
      const int g = warp + kProjWarps * i;
      if (g < G) {
        uint4 xh0 = make_uint4(0u, 0u, 0u, 0u), xl0 = xh0, xh1 = xh0, xl1 = xh0;
        if (has_tok) {
          const int c = 8 * g + 2 * t;
          xh0 = __ldg(xf + 2 * c);
          xl0 = __ldg(xf + 2 * c + 1);
          xh1 = __ldg(xf + 2 * c + 2);
          xl1 = __ldg(xf + 2 * c + 3);
        }
        float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        mma_group(d, wl[i], wh[i], xh0, xl0, xh1, xl1);
        const float f0 = fsg[2 * t][g], f1 = fsg[2 * t + 1][g];
        acc[0] = fmaf(bl[i], f0, fmaf(sl[i], d[0], acc[0]));
        acc[1] = fmaf(bl[i], f1, fmaf(sl[i], d[1], acc[1]));
        acc[2] = fmaf(bh[i], f0, fmaf(sh[i], d[2], acc[2]));
        acc[3] = fmaf(bh[i], f1, fmaf(sh[i], d[3], acc[3]));
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) red[warp][lane][q] = acc[q];
    __syncthreads();
    if (warp == 0) {
      float tot[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float s = red[0][lane][q];
#pragma unroll
        for (int w = 1; w < kProjWarps; ++w) s = __fadd_rn(s, red[w][lane][q]);
        tot[q] = s;
      }
      if (PAIRED) {
        // thread (gid, t): gate/up of intermediate row r0+gid, tokens 2t, 2t+1
        hs[gid][2 * t] = __fmul_rn(ref_silu(tot[0]), tot[2]);
        hs[gid][2 * t + 1] = __fmul_rn(ref_silu(tot[1]), tot[3]);
        __syncwarp();
        if (lane < nv) {
          const int p = off + c0 + lane;
          const int hch = a.hK >> 3;
          uint32_t hi[8], lo[8];
          float fs = hs[0][lane];
#pragma unroll
          for (int r = 0; r < 8; ++r) split_bf16(hs[r][lane], hi[r], lo[r]);
#pragma unroll
          for (int r = 1; r < 8; ++r) fs = __fadd_rn(fs, hs[r][lane]);
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
            const int p = off + c0 + n;
            const int orow = a.out_row ? a.out_row[p] : a.pair_tok[p] * a.kp1 + a.pair_pick[p];
            float* o = a.out + (size_t)orow * a.ostride;
            o[row_lo] = tot[q];
            o[row_hi] = tot[2 + q];
          }
        }
      }
    }
    __syncthreads();
  }
}

// ----------------------------------------------------------------------------
// Combine, RMSNorm, element-wise ops
// ----------------------------------------------------------------------------
__global__ void combine_kernel(CombineArgs a) {
  const int b = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
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

__global__ void rmsnorm_kernel(const float* __restrict__ in, float* __restrict__ out, int dim,
                               const float* __restrict__ w, float eps, int exact) {
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

__global__ void dequant_kernel(const uint32_t* __restrict__ packed, const uint16_t* __restrict__ sc,
                               const uint16_t* __restrict__ bi, int rows, int K,
                               float* __restrict__ out) {
  const size_t total = (size_t)rows * K;
  const int G = K >> 6;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t row = i / K;
    const int col = (int)(i - row * K);
    const uint32_t q = (packed[row * (K >> 3) + (col >> 3)] >> ((col & 7) * 4)) & 0xFu;
    const float s = bf16_bits_to_f32(sc[row * G + (col >> 6)]);
    const float b = bf16_bits_to_f32(bi[row * G + (col >> 6)]);
    out[i] = __fadd_rn(__fmul_rn(s, (float)q), b);
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

// Expert list for a single expert over `T` tokens (standalone projections).
__global__ void setup_single_kernel(int T, const uint8_t* ptr, int* n_active, int* act_kind,
                                    const uint8_t** act_ptr, int* act_off, int* act_cnt,
                                    int* pair_tok, int* pair_pick, int* out_row) {
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *n_active = 1;
    act_kind[0] = 0;
    act_ptr[0] = ptr;
    act_off[0] = 0;
    act_cnt[0] = T;
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < T; i += gridDim.x * blockDim.x) {
    pair_tok[i] = i;
    pair_pick[i] = 0;
    out_row[i] = i;
  }
}

inline int grid_for(size_t n, int threads) {
  size_t b = (n + threads - 1) / threads;
  if (b > 148 * 64) b = 148 * 64;
  if (b < 1) b = 1;
  return (int)b;
}

}  // namespace

void launch_router_logits(const RouterArgs& a, cudaStream_t s, uint64_t* launches) {
  const RouterGeom& g = a.g;
  const dim3 grid1((g.E + kRtExp * kRtWarps - 1) / (kRtExp * kRtWarps),
                   (a.B + kRtTok - 1) / kRtTok);
  const size_t sm1 = (size_t)kRtTok * g.Hp * sizeof(float);
  if (sm1 > 48 * 1024)
    cudaFuncSetAttribute(router_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)sm1);
  router_logits_kernel<<<grid1, kRtWarps * 32, sm1, s>>>(a);
  if (launches) *launches += 1;
}

void launch_router_select(const RouterArgs& a, cudaStream_t s, uint64_t* launches) {
  const RouterGeom& g = a.g;
  const size_t sm_tok = (size_t)(g.H + 2 * g.E) * sizeof(float);
  const size_t sm_grp = (size_t)3 * (g.E + 1) * sizeof(int);
  const size_t sm2 = sm_tok > sm_grp ? sm_tok : sm_grp;
  if (sm2 > 48 * 1024)
    cudaFuncSetAttribute(router_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)sm2);
  router_select_kernel<<<a.B, kSelThreads, sm2, s>>>(a);
  if (launches) *launches += 1;
}

void launch_group(const RouterArgs& a, cudaStream_t s, uint64_t* launches) {
  const size_t sm = (size_t)3 * (a.g.E + 1) * sizeof(int);
  group_kernel<<<1, kSelThreads, sm, s>>>(a);
  if (launches) *launches += 1;
}

void launch_frag_prep(const float* x, int rows, int K, uint4* frag, float* fsum8, cudaStream_t s,
                      uint64_t* launches) {
  const size_t n = (size_t)rows * (K >> 3);
  frag_prep_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, rows, K, frag, fsum8);
  if (launches) *launches += 1;
}

void launch_proj(const ProjArgs& a, bool paired, int max_rows, int max_active, cudaStream_t s,
                 uint64_t* launches) {
  const int tile = paired ? 8 : 16;
  const dim3 grid((max_rows + tile - 1) / tile, max_active);
  if (paired) proj_kernel<true><<<grid, kProjWarps * 32, 0, s>>>(a);
  else proj_kernel<false><<<grid, kProjWarps * 32, 0, s>>>(a);
  if (launches) *launches += 1;
}

void launch_combine(const CombineArgs& a, cudaStream_t s, uint64_t* launches) {
  const dim3 grid((a.H + 255) / 256, a.B);
  combine_kernel<<<grid, 256, 0, s>>>(a);
  if (launches) *launches += 1;
}

void launch_rmsnorm(const float* in, float* out, int rows, int dim, const float* w, float eps,
                    bool exact, cudaStream_t s, uint64_t* launches) {
  rmsnorm_kernel<<<rows, 256, 0, s>>>(in, out, dim, w, eps, exact ? 1 : 0);
  if (launches) *launches += 1;
}

void launch_dequant(const uint32_t* packed, const uint16_t* sc, const uint16_t* bi, int rows,
                    int K, float* out, cudaStream_t s, uint64_t* launches) {
  dequant_kernel<<<grid_for((size_t)rows * K, 256), 256, 0, s>>>(packed, sc, bi, rows, K, out);
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

void launch_router_pack(const float* w, const RouterGeom& g, void* wp, cudaStream_t s,
                        uint64_t* launches) {
  router_pack_kernel<<<grid_for((size_t)g.E * g.Hp, 256), 256, 0, s>>>(w, g, wp);
  if (launches) *launches += 1;
}

void launch_setup_single(int T, const uint8_t* ptr, int* n_active, int* act_kind,
                         const uint8_t** act_ptr, int* act_off, int* act_cnt, int* pair_tok,
                         int* pair_pick, int* out_row, cudaStream_t s, uint64_t* launches) {
  setup_single_kernel<<<grid_for((size_t)T, 256), 256, 0, s>>>(
      T, ptr, n_active, act_kind, act_ptr, act_off, act_cnt, pair_tok, pair_pick, out_row);
  if (launches) *launches += 1;
}

}  // namespace osm
