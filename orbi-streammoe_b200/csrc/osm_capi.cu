// osm_capi.cu -- the extern "C" boundary (include/osm_b200.h) over the sm_100a
// kernels: contexts with their stream and scratch, the HBM expert slab, MoE
// layers, and every entry point.  No exception crosses the boundary.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <new>
#include <string>
#include <thread>
#include <tuple>
#include <unordered_map>
#include <vector>

#include "../../include/osm_b200.h"
#include "osm_common.cuh"
#include "osm_kernels.cuh"

namespace {

constexpr size_t kAlign = 256;
constexpr uint32_t kGemvMaxTokens = 2;  // calls with at most this many tokens use osm_gemv.cu

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Device scratch of one context, carved from a single allocation.  Sized for
// (tokens T, hidden H, experts E, top-k k, intermediate I, projection K).
struct Scratch {
  size_t T = 0, H = 0, E = 0, k = 0, I = 0, K = 0;
  void* base = nullptr;
  size_t bytes = 0;
  float* logits = nullptr;
  float* bounds = nullptr;
  uint32_t* ids = nullptr;
  float* weights = nullptr;
  float* mass = nullptr;
  float* sgate = nullptr;
  uint4* xfrag = nullptr;
  float* xfsum8 = nullptr;
  uint16_t* xbf = nullptr;      // bf16 copy of x (prefill path)
  unsigned int* ticket = nullptr;
  int* counts = nullptr;
  int* n_active = nullptr;
  osm::ActEntry* act = nullptr;
  int* n_tg = nullptr;
  int* tg_expert = nullptr;
  int* tg_begin = nullptr;
  int* n_ch = nullptr;
  int2* chunks = nullptr;
  int* pair_tok = nullptr;
  int* pair_pick = nullptr;
  int* tp_pos = nullptr;
  int* cursor = nullptr;
  int* out_row = nullptr;
  uint4* hfrag = nullptr;
  float* hfsum8 = nullptr;
  float* partial = nullptr;
  float* normalized = nullptr;
  uint8_t* xd = nullptr;        // digit planes of each pair's x row / of h (osm_tcd.cu)
  float2* xq = nullptr;
  uint8_t* hd = nullptr;
  float2* hq = nullptr;
  uint32_t* status = nullptr;
  uint32_t* range_status = nullptr;  // status of one checked prefill call
  uint32_t* early_status = nullptr;  // status of a cached call's early expert run
  unsigned long long* exact_count = nullptr;
  const uint8_t** pick_ptr = nullptr;
};

}  // namespace

namespace {
enum KernelKind {
  kKRouterLogits = 0,
  kKRouterSelect,
  kKGateUp,
  kKDown,
  kKCombine,
  kKRmsNorm,
  kKPrep,
  kKOther,
};
const char* const kKindNames[OSM_KERNEL_KINDS] = {
    "router_logits", "router_select", "proj_gate_up", "proj_down",
    "combine",       "rmsnorm",       "prep",         "other"};

struct ProfRec {
  int kind;
  cudaEvent_t a, b;
};
}  // namespace

struct osm_context {
  int device = 0;
  uint32_t max_tokens = 0;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  std::string err;
  uint64_t launches = 0;
  Scratch sc;
  int grid_cap = 148 * 4;       // resident CTAs of the projection kernels
  int num_sms = 148;
  int max_smem = 0;             // dynamic shared memory limit of the decode kernels
  bool prof_on = false;
  const float* cur_x = nullptr;  // activations of the call in flight (expert kernels)
  std::vector<cudaEvent_t> ev_pool;
  std::vector<ProfRec> recs;
  void* status_blk = nullptr;       // status words + exact-route counter: never moves
  int plans_alive = 0;              // captured graphs hold scratch pointers
  std::vector<void*> retired;       // scratch blocks a live plan may still use
  uint32_t* picks_host = nullptr;   // mapped pinned: the picks a cached call reads back
  uint32_t* picks_dev = nullptr;    // the same memory as the kernels address it
  size_t picks_cap = 0;
  cudaEvent_t picks_ev = nullptr;
  uint32_t pending_status = 0;      // status bits read by checked calls, reported next
  bool tc_enabled = true;           // tensor-core expert kernels (OSM_DISABLE_TC=1: off)
  bool tc_decode = false;           // also for fp32 calls of 3+ tokens (OSM_TC_DECODE=1)
  bool dg_decode = true;            // int8 digit-plane tensor-core kernels for fp32 calls
                                    // (OSM_DG_DECODE=0: the mma.sync kernels throughout)
  uint32_t dg_min_tokens = 96;      // ... of at least this many tokens (OSM_DG_MIN_TOKENS;
                                    // below it the mma.sync grouped kernels are faster)
};

struct osm_slab {
  osm_context* ctx = nullptr;
  osm_expert_layout layout{};
  uint32_t slots = 0;
  uint8_t* base = nullptr;
  cudaStream_t side = nullptr;
  cudaEvent_t ev = nullptr;
  uint64_t h2d_bytes = 0;
  // TMA tensor maps over the gate, up and down weight sections of every slot
  // (the tensor-core expert kernels); tc_ok false: the layout does not suit them
  alignas(64) unsigned char tc_maps[3][128];
  bool tc_ok = false;
};

// One rank's expert-parallel block and the peers' blocks as mapped here.
struct osm_ep {
  osm_context* ctx = nullptr;
  osm::EpLayout lay{};
  unsigned char* own = nullptr;
  unsigned char* peer[osm::kEpMaxWorld] = {};
  bool opened = false;
  float* sgate = nullptr;  // [T_r] shared-expert gates of this rank's tokens
  uint32_t epoch = 0;
  uint64_t timeout_ns = 2000000000ull;
};

// Expert residency over one slab: LFU + recency entries keyed (layer, expert).
struct osm_cache {
  osm_slab* slab = nullptr;             // null: policy only (no copies)
  uint64_t budget = 0, accounted = 0;
  osm_cache_source_fn source = nullptr;
  void* user = nullptr;
  struct Node {
    int32_t slot = -1;
    uint64_t frequency = 0, last_use = 0, epoch = 0;
  };
  using Rank = std::tuple<uint64_t, uint64_t, uint64_t>;  // (frequency, last use, key)
  std::unordered_map<uint64_t, Node> entries;
  std::set<Rank> order;                 // eviction order of the resident entries
  std::unordered_map<uint64_t, uint64_t> frequency_history;  // survives evictions
  std::unordered_map<uint32_t, osm_layer*> layers;
  std::vector<int32_t> free_slots;
  // one acquire's copies (slot, host source) and slot-table writes, issued
  // together when the acquire ends
  std::vector<std::pair<uint32_t, const void*>> fills;
  std::vector<std::pair<int32_t*, int32_t>> table_writes;
  uint64_t tick = 0, epoch = 0, resident_bytes = 0;
  uint64_t hits = 0, misses = 0, loads = 0, evictions = 0;
  // exposed-copy timing: event pairs on the compute stream around each
  // acquire's copies (issue to landing), read and released by
  // osm_cache_exposed_read
  bool time_copies = false;
  int device = 0;                       // the slab's device
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> copy_waits, spare_events;
  std::string err;
};

struct osm_plan {
  osm_layer* layer = nullptr;
  cudaGraphExec_t exec = nullptr;
  std::vector<ProfRec> recs;
  uint32_t kernels = 0;
};

struct osm_layer {
  osm_context* ctx = nullptr;
  osm::RouterGeom g{};
  uint32_t norm = 0;
  void* wp = nullptr;          // permuted router
  void* wx = nullptr;          // router tiles of the exact logits
  uint32_t* qmeta = nullptr;   // 8-bit router: scale | bias << 16 per (expert, 64-group)
  float* bias = nullptr;
  float* sgate_w = nullptr;
  uint8_t* shared_slot = nullptr;
  osm_expert_layout shared_layout{};
  float* norm_w = nullptr;
  float norm_eps = 1e-6f;
  int* slot_of = nullptr;
  std::vector<int32_t> slot_host;
  osm_slab* slab = nullptr;
  // TMA tensor maps over the shared expert's weight sections
  alignas(64) unsigned char tc_shared[3][128];
  bool tc_shared_ok = false;
};

namespace {

int fail(osm_context* ctx, int code, const std::string& msg) {
  if (ctx) ctx->err = msg;
  return code;
}

int cuda_fail(osm_context* ctx, cudaError_t e, const char* what) {
  return fail(ctx, OSM_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define OSM_CUDA(ctx, call)                                   \
  do {                                                        \
    cudaError_t e_ = (call);                                  \
    if (e_ != cudaSuccess) return cuda_fail((ctx), e_, #call); \
  } while (0)

int check_launch(osm_context* ctx, const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(ctx, e, what);
  return OSM_OK;
}

cudaEvent_t pool_event(osm_context* ctx) {
  if (!ctx->ev_pool.empty()) {
    cudaEvent_t e = ctx->ev_pool.back();
    ctx->ev_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

// Bracket one launch with events on the context stream when profiling.
struct Prof {
  osm_context* ctx;
  int idx = -1;
  Prof(osm_context* c, int kind) : ctx(c) {
    if (!ctx->prof_on) return;
    ProfRec r{kind, pool_event(ctx), pool_event(ctx)};
    cudaEventRecord(r.a, ctx->stream);
    ctx->recs.push_back(r);
    idx = (int)ctx->recs.size() - 1;
  }
  ~Prof() {
    if (idx >= 0) cudaEventRecord(ctx->recs[idx].b, ctx->stream);
  }
};

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// Grow the scratch to cover the request (no shrink).
int ensure_scratch(osm_context* ctx, size_t T, size_t H, size_t E, size_t k, size_t I,
                   size_t K) {
  Scratch& s = ctx->sc;
  T = std::max<size_t>(T, 1);
  if (s.base && T <= s.T && H <= s.H && E <= s.E && k <= s.k && I <= s.I && K <= s.K)
    return OSM_OK;
  T = std::max(T, s.T);
  H = std::max(H, s.H);
  E = std::max(E, s.E);
  k = std::max(k, s.k);
  I = std::max(I, s.I);
  K = std::max(K, s.K);
  const size_t kp1 = k + 1;
  const size_t P = T * kp1;
  const size_t Kx = std::max(H, K);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, kAlign);
    return o;
  };
  const size_t o_logits = take(T * E * 4), o_bounds = take(T * E * 4);
  const size_t o_ids = take(T * k * 4), o_w = take(T * k * 4), o_mass = take(T * 4);
  const size_t o_sg = take(T * 4);
  const size_t o_xf = take(T * (Kx / 8) * 32), o_xs = take(T * (Kx / 8) * 4);
  const size_t o_xbf = take(T * H * 2);
  const size_t o_ticket = take(4), o_counts = take((E + 1) * 4), o_nact = take(4);
  const size_t o_act = take((E + 1) * sizeof(osm::ActEntry)), o_ntg = take(4);
  const size_t max_tg = P / osm::kTokGroup + E + 2;
  const size_t o_tge = take(max_tg * 4), o_tgb = take(max_tg * 4);
  const size_t max_ch = P / 8 + E + 2;
  const size_t o_nch = take(4), o_ch = take(max_ch * 8);
  const size_t o_ptok = take(P * 4), o_ppick = take(P * 4), o_cursor = take((E + 1) * 4);
  const size_t o_tpp = take(P * 4);
  const size_t o_orow = take(P * 4);
  const size_t o_hf = take(P * (I / 8) * 32), o_hs = take(P * (I / 8) * 4);
  const size_t o_part = take(P * H * 4), o_norm = take(T * H * 4);
  const size_t o_pptr = take(T * k * sizeof(void*));
  const size_t o_xd = take(P * 3 * Kx), o_xq = take(P * (Kx / 64) * 8);
  const size_t o_hd = take(P * 3 * I), o_hq = take(P * (I / 64) * 8);
  void* base = nullptr;
  cudaError_t e = cudaMalloc(&base, off);
  if (e != cudaSuccess) return fail(ctx, OSM_ENOMEM, "scratch allocation failed");
  if (s.base) {
    // a captured plan replays on the block it was captured with: keep it
    // until the context goes; otherwise free it once queued work is done
    if (ctx->plans_alive > 0) {
      ctx->retired.push_back(s.base);
    } else {
      cudaStreamSynchronize(ctx->stream);
      cudaFree(s.base);
    }
  }
  cudaMemset(base, 0, off);
  char* b = static_cast<char*>(base);
  s.base = base;
  s.bytes = off;
  s.T = T; s.H = H; s.E = E; s.k = k; s.I = I; s.K = K;
  s.logits = reinterpret_cast<float*>(b + o_logits);
  s.bounds = reinterpret_cast<float*>(b + o_bounds);
  s.ids = reinterpret_cast<uint32_t*>(b + o_ids);
  s.weights = reinterpret_cast<float*>(b + o_w);
  s.mass = reinterpret_cast<float*>(b + o_mass);
  s.sgate = reinterpret_cast<float*>(b + o_sg);
  s.xfrag = reinterpret_cast<uint4*>(b + o_xf);
  s.xfsum8 = reinterpret_cast<float*>(b + o_xs);
  s.xbf = reinterpret_cast<uint16_t*>(b + o_xbf);
  s.ticket = reinterpret_cast<unsigned int*>(b + o_ticket);
  s.counts = reinterpret_cast<int*>(b + o_counts);
  s.n_active = reinterpret_cast<int*>(b + o_nact);
  s.act = reinterpret_cast<osm::ActEntry*>(b + o_act);
  s.n_tg = reinterpret_cast<int*>(b + o_ntg);
  s.tg_expert = reinterpret_cast<int*>(b + o_tge);
  s.tg_begin = reinterpret_cast<int*>(b + o_tgb);
  s.n_ch = reinterpret_cast<int*>(b + o_nch);
  s.chunks = reinterpret_cast<int2*>(b + o_ch);
  s.pair_tok = reinterpret_cast<int*>(b + o_ptok);
  s.pair_pick = reinterpret_cast<int*>(b + o_ppick);
  s.tp_pos = reinterpret_cast<int*>(b + o_tpp);
  s.cursor = reinterpret_cast<int*>(b + o_cursor);
  s.out_row = reinterpret_cast<int*>(b + o_orow);
  s.hfrag = reinterpret_cast<uint4*>(b + o_hf);
  s.hfsum8 = reinterpret_cast<float*>(b + o_hs);
  s.partial = reinterpret_cast<float*>(b + o_part);
  s.normalized = reinterpret_cast<float*>(b + o_norm);
  s.pick_ptr = reinterpret_cast<const uint8_t**>(b + o_pptr);
  s.xd = reinterpret_cast<uint8_t*>(b + o_xd);
  s.xq = reinterpret_cast<float2*>(b + o_xq);
  s.hd = reinterpret_cast<uint8_t*>(b + o_hd);
  s.hq = reinterpret_cast<float2*>(b + o_hq);
  return OSM_OK;
}

bool layout_ok(const osm_expert_layout* L) {
  if (!L || L->group != 64 || L->hidden == 0 || L->inter == 0) return false;
  if (L->hidden % 64 || L->inter % 64) return false;
  if (L->hidden > 2048 || L->inter > 768) return false;  // gate/up K <= 2048, down K <= 768
  if (L->hidden % 16 || L->inter % 8) return false;
  const uint64_t H = L->hidden, I = L->inter;
  const uint64_t gu_w = I * H / 2, gu_m = I * (H / 64) * 2, dn_w = H * I / 2,
                 dn_m = H * (I / 64) * 2;
  auto in = [&](uint64_t o, uint64_t n) { return o % 4 == 0 && o + n <= L->stride; };
  return in(L->gate_w, gu_w) && in(L->up_w, gu_w) && in(L->down_w, dn_w) && in(L->gate_s, gu_m) &&
         in(L->gate_b, gu_m) && in(L->up_s, gu_m) && in(L->up_b, gu_m) && in(L->down_s, dn_m) &&
         in(L->down_b, dn_m) && (L->gate_w % 8 == 0) && (L->up_w % 8 == 0) &&
         (L->down_w % 8 == 0);
}

void fill_sections(osm::ProjSections& s, const osm_expert_layout& r, const osm_expert_layout& sh,
                   bool gate_up) {
  const osm_expert_layout* L[2] = {&r, &sh};
  for (int i = 0; i < 2; ++i) {
    if (gate_up) {
      s.w[i] = L[i]->gate_w; s.s[i] = L[i]->gate_s; s.b[i] = L[i]->gate_b;
      s.w2[i] = L[i]->up_w; s.s2[i] = L[i]->up_s; s.b2[i] = L[i]->up_b;
      s.rows[i] = (int)L[i]->inter;
      s.K[i] = (int)L[i]->hidden;
    } else {
      s.w[i] = L[i]->down_w; s.s[i] = L[i]->down_s; s.b[i] = L[i]->down_b;
      s.w2[i] = s.w[i]; s.s2[i] = s.s[i]; s.b2[i] = s.b[i];
      s.rows[i] = (int)L[i]->hidden;
      s.K[i] = (int)L[i]->inter;
    }
  }
}

// Router args common to route / forward / experts.
osm::RouterArgs router_args(osm_layer* L, const float* x, uint32_t T) {
  osm_context* ctx = L->ctx;
  Scratch& s = ctx->sc;
  osm::RouterArgs a{};
  a.g = L->g;
  a.wp = static_cast<const uint4*>(L->wp);
  a.wx = L->wx;
  a.qmeta = L->qmeta;
  a.bias = L->bias;
  a.x = x;
  a.B = (int)T;
  a.norm = (int)L->norm;
  a.logits = s.logits;
  a.bounds = s.bounds;
  a.ids = s.ids;
  a.weights = s.weights;
  a.mass = s.mass;
  a.sgate_w = L->shared_slot ? L->sgate_w : nullptr;
  a.sgate = s.sgate;
  a.xfrag = s.xfrag;
  a.xfsum8 = s.xfsum8;
  a.xbf = nullptr;
  a.chunk_pairs = 8;
  a.slot_of = L->slot_of;
  a.slab = L->slab ? L->slab->base : nullptr;
  a.slab_stride = L->slab ? L->slab->layout.stride : 0;
  a.shared_slot = L->shared_slot;
  a.ticket = s.ticket;
  a.counts = s.counts;
  a.n_active = s.n_active;
  a.act = s.act;
  a.n_tg = s.n_tg;
  a.tg_expert = s.tg_expert;
  a.tg_begin = s.tg_begin;
  a.pair_tok = s.pair_tok;
  a.pair_pick = s.pair_pick;
  a.tp_pos = s.tp_pos;
  a.n_ch = s.n_ch;
  a.chunks = s.chunks;
  a.cursor = s.cursor;
  a.defer_scatter = (size_t)T * (L->g.k + 1) > 8192 ? 1 : 0;  // grid-wide pair scatter
  a.status = s.status;
  a.exact_count = s.exact_count;
  a.pick_ptr = L->slab ? s.pick_ptr : nullptr;
  return a;
}

void launch_router_pair(osm_context* ctx, const osm::RouterArgs& a) {
  if (!a.skip_route) {
    Prof p(ctx, kKRouterLogits);
    osm::launch_router_logits(a, ctx->stream, &ctx->launches);
  }
  Prof p(ctx, kKRouterSelect);
  osm::launch_router_select(a, ctx->stream, &ctx->launches);
}

// The decode kernels (osm_gemv.cu) serve calls of 1-2 tokens whose shapes fit
// their shared-memory plan; fills the call-independent fields of g.
bool gemv_path(osm_layer* L, uint32_t T, osm::GemvArgs* g, osm::GemvLaunch* gl) {
  if (T > kGemvMaxTokens || !L->slab) return false;
  osm_context* ctx = L->ctx;
  const osm_expert_layout& R = L->slab->layout;
  const osm_expert_layout& S = L->shared_slot ? L->shared_layout : R;
  const int max_active = (int)std::min<size_t>(L->g.E, (size_t)T * L->g.k) + (L->shared_slot ? 1 : 0);
  *g = osm::GemvArgs{};
  fill_sections(g->gu, R, S, true);
  fill_sections(g->dn, R, S, false);
  g->B = (int)T;
  g->H = L->g.H;
  g->Imax = (int)std::max(R.inter, L->shared_slot ? S.inter : 0u);
  g->k = L->g.k;
  g->E = L->g.E;
  g->has_shared = L->shared_slot ? 1 : 0;
  g->slab = L->slab->base;
  g->slab_stride = R.stride;
  g->shared_ptr = L->shared_slot;
  return osm::gemv_configure(*g, max_active, ctx->num_sms, ctx->max_smem, gl);
}

// The grouped kernels (osm_gemv.cu) serve calls of 3+ tokens whose layouts
// suit them; fills the call-independent fields of a.
bool grouped_path(osm_layer* L, osm::GrpArgs* a, size_t* smem_gu, size_t* smem_dn) {
  if (!L->slab) return false;
  osm_context* ctx = L->ctx;
  const osm_expert_layout& R = L->slab->layout;
  const osm_expert_layout& S = L->shared_slot ? L->shared_layout : R;
  *a = osm::GrpArgs{};
  fill_sections(a->gu, R, S, true);
  fill_sections(a->dn, R, S, false);
  a->H = L->g.H;
  a->Imax = (int)std::max(R.inter, L->shared_slot ? S.inter : 0u);
  a->kp1 = (int)L->g.k + 1;
  a->has_shared = L->shared_slot ? 1 : 0;
  a->slab_stride = R.stride;
  return osm::grouped_configure(*a, ctx->max_smem, smem_gu, smem_dn);
}

// TMA tensor maps over the weight sections of an expert layout at `base`.
bool encode_expert_maps(unsigned char (*dst)[128], const uint8_t* base, const osm_expert_layout& L,
                        uint32_t slots) {
  const uint64_t off[3] = {L.gate_w, L.up_w, L.down_w};
  const int rows[3] = {(int)L.inter, (int)L.inter, (int)L.hidden};
  const int words[3] = {(int)L.hidden / 8, (int)L.hidden / 8, (int)L.inter / 8};
  return osm::tc_encode_maps(dst, base, off, rows, words, (int)slots, L.stride);
}

// The tensor-core expert kernels (osm_tc.cu): fills the call-independent
// fields of ta and the tensor maps; false when the layer's shapes or
// alignment do not suit them (the older kernels run instead).
bool tc_path(osm_layer* L, osm::TcArgs* ta, osm::TcMaps* maps) {
  osm_context* ctx = L->ctx;
  if (!ctx->tc_enabled || !L->slab || !L->slab->tc_ok) return false;
  if (L->shared_slot && !L->tc_shared_ok) return false;
  const osm_expert_layout& R = L->slab->layout;
  const osm_expert_layout& S = L->shared_slot ? L->shared_layout : R;
  *ta = osm::TcArgs{};
  fill_sections(ta->gu, R, S, true);
  fill_sections(ta->dn, R, S, false);
  ta->H = L->g.H;
  ta->Imax = (int)std::max(R.inter, L->shared_slot ? S.inter : 0u);
  ta->kp1 = (int)L->g.k + 1;
  ta->slab = L->slab->base;
  ta->slab_stride = R.stride;
  if (!osm::tc_configure(*ta, L->shared_slot ? 1 : 0, ctx->max_smem)) return false;
  std::memcpy(maps->m[0], L->slab->tc_maps, sizeof(L->slab->tc_maps));
  if (L->shared_slot) std::memcpy(maps->m[1], L->tc_shared, sizeof(L->tc_shared));
  else std::memcpy(maps->m[1], L->slab->tc_maps, sizeof(L->slab->tc_maps));
  return true;
}

// Whether a call runs its experts on the tensor-core kernels of osm_tc.cu:
// every prefill call whose shapes they take (the older prefill kernel of
// osm_prefill.cu otherwise, or with OSM_DISABLE_TC=1); fp32 calls of 3+
// tokens only when the context enables it (OSM_TC_DECODE=1; the grouped
// decode kernels are faster at the decode batch sizes measured so far).
bool tc_use(osm_layer* L, uint32_t T, bool prefill, osm::TcArgs* ta, osm::TcMaps* maps) {
  osm_context* ctx = L->ctx;
  if (!prefill && !ctx->tc_decode) {
    return false;
  }
  return tc_path(L, ta, maps);
}

// Whether an fp32 call of T tokens runs its experts on the int8 digit-plane
// tensor-core kernels of osm_tcd.cu: from dg_min_tokens tokens (96 by default,
// where they overtake the mma.sync grouped kernels of osm_gemv.cu on the
// Qwen3-Next sublayer; OSM_DG_MIN_TOKENS moves the threshold, OSM_DG_DECODE=0
// turns them off).  The shapes are those of the 16-bit tensor-core
// kernels (same tensor maps, same item geometry); scale and bias rows arrive
// by bulk copies, so their sections must be 16-byte aligned.
bool dg_use(osm_layer* L, uint32_t T, osm::TcArgs* ta, osm::TcMaps* maps) {
  osm_context* ctx = L->ctx;
  if (!ctx->dg_decode || T < 3 || T < ctx->dg_min_tokens || !osm::dg_fits(ctx->max_smem)) return false;
  if (!tc_path(L, ta, maps)) return false;
  for (int kd = 0; kd < 2; ++kd) {
    const uint64_t o[6] = {ta->gu.s[kd], ta->gu.b[kd], ta->gu.s2[kd], ta->gu.b2[kd], ta->dn.s[kd], ta->dn.b[kd]};
    for (uint64_t v : o)
      if (v % 16) return false;
  }
  return ta->H % 128 == 0 && ta->Imax % 128 == 0;
}

// Pairs per chunk of the grouping for a call of T tokens: the tensor-core
// kernels take 32 (fp32 calls) or 96 (prefill), the older grouped kernels 8
// and the older prefill kernel 128.
int chunk_pairs_for(osm_layer* L, uint32_t T, bool prefill) {
  osm::TcArgs ta;
  osm::TcMaps maps;
  if (!prefill && dg_use(L, T, &ta, &maps)) return osm::kDgChunk;
  const bool tc = tc_use(L, T, prefill, &ta, &maps);
  if (prefill) return tc ? osm::kTcChunkFast : 128;
  return tc ? osm::kTcChunkPrecise : 8;
}

// Runs the tensor-core gate/up and down kernels, then the combine.
int run_tc(osm_layer* L, uint32_t T, float* out, const float* residual, osm::TcArgs ta,
           const osm::TcMaps& maps, bool precise, const uint16_t* xb, bool f16_out,
           bool combine = true) {
  osm_context* ctx = L->ctx;
  Scratch& s = ctx->sc;
  ta.x = ctx->cur_x;
  ta.xb = xb;
  ta.h = reinterpret_cast<float*>(s.hfrag);
  ta.hb = reinterpret_cast<uint16_t*>(s.hfrag);
  ta.partial = s.partial;
  ta.pb = reinterpret_cast<uint16_t*>(s.partial);
  ta.n_ch = s.n_ch;
  ta.chunks = s.chunks;
  ta.act = s.act;
  ta.pair_tok = s.pair_tok;
  ta.pair_pick = s.pair_pick;
  ta.status = s.status;
  {
    Prof p(ctx, kKGateUp);
    const cudaError_t e = osm::launch_tc_gateup(ta, maps, precise, ctx->num_sms, ctx->stream, &ctx->launches);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "tensor-core gate/up");
  }
  {
    Prof p(ctx, kKDown);
    const cudaError_t e = osm::launch_tc_down(ta, maps, precise, ctx->num_sms, ctx->stream, &ctx->launches);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "tensor-core down");
  }
  if (!combine) return OSM_OK;  // the caller reads the pair rows (expert parallelism)
  if (precise) {
    osm::CombineArgs c{};
    c.partial = s.partial;
    c.weights = s.weights;
    c.sgate = L->shared_slot ? s.sgate : nullptr;
    c.residual = residual;
    c.out = out;
    c.B = (int)T;
    c.H = L->g.H;
    c.k = L->g.k;
    {
      Prof p(ctx, kKCombine);
      osm::launch_combine(c, ctx->stream, &ctx->launches);
    }
    return check_launch(ctx, "combine");
  }
  if ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(residual)) & 15)
    return fail(ctx, OSM_EINVAL, "prefill: out and residual must be 16-byte aligned");
  {
    Prof p(ctx, kKCombine);
    osm::launch_combine_bf16(ta.pb, s.tp_pos, s.weights, L->shared_slot ? s.sgate : nullptr, residual,
                             out, f16_out, s.status, (int)T, L->g.H, L->g.k, ctx->stream,
                             &ctx->launches);
  }
  return check_launch(ctx, "prefill combine");
}

// The digit-plane tensor-core path: digit planes of each pair's x row,
// gate/up (+ SwiGLU), digit planes of h, down, then the pick-order combine.
int run_dg(osm_layer* L, uint32_t T, float* out, const float* residual, const osm::TcArgs& ta0,
           const osm::TcMaps& maps) {
  osm_context* ctx = L->ctx;
  Scratch& s = ctx->sc;
  osm::DgArgs d{};
  d.t = ta0;
  osm::TcArgs& ta = d.t;
  ta.x = ctx->cur_x;
  ta.h = reinterpret_cast<float*>(s.hfrag);
  ta.partial = s.partial;
  ta.n_ch = s.n_ch;
  ta.chunks = s.chunks;
  ta.act = s.act;
  ta.pair_tok = s.pair_tok;
  ta.pair_pick = s.pair_pick;
  ta.status = s.status;
  d.xq = s.xq;
  d.hq = s.hq;
  const int H = L->g.H, Imax = ta.Imax;
  // pair positions of the call: k per token, plus the shared expert's
  const int P = (int)T * (int)L->g.k + (L->shared_slot ? (int)T : 0);
  osm::DgMaps dm;
  std::memcpy(&dm.q, &maps, sizeof(maps));
  for (int i = 0; i < 3; ++i)
    if (!osm::tc_encode_u8_rows(dm.xd[i], s.xd, (uint64_t)P * 3, (uint64_t)H, 16 * (i + 1)) ||
        !osm::tc_encode_u8_rows(dm.hd[i], s.hd, (uint64_t)P * 3, (uint64_t)Imax, 16 * (i + 1)))
      return fail(ctx, OSM_ECUDA, "digit-plane tensor maps");
  {
    Prof p(ctx, kKGateUp);
    osm::launch_digits(ctx->cur_x, s.pair_tok, (int)T, P, H, H, s.xd, s.xq, ctx->stream, &ctx->launches);
    const cudaError_t e = osm::launch_dg_gateup(d, dm, ctx->num_sms, ctx->stream, &ctx->launches);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "digit-plane gate/up");
  }
  {
    Prof p(ctx, kKDown);
    osm::launch_digits(ta.h, nullptr, P, P, Imax, Imax, s.hd, s.hq, ctx->stream, &ctx->launches);
    const cudaError_t e = osm::launch_dg_down(d, dm, ctx->num_sms, ctx->stream, &ctx->launches);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "digit-plane down");
  }
  osm::CombineArgs c{};
  c.partial = s.partial;
  c.weights = s.weights;
  c.sgate = L->shared_slot ? s.sgate : nullptr;
  c.residual = residual;
  c.out = out;
  c.B = (int)T;
  c.H = H;
  c.k = L->g.k;
  {
    Prof p(ctx, kKCombine);
    osm::launch_combine(c, ctx->stream, &ctx->launches);
  }
  return check_launch(ctx, "combine");
}

// picks_from_ids: one token whose picks the decode kernels resolve through
// the slot table themselves (no binding step ran)
// status: where the decode kernels report (the context's status word when
// null)
int run_experts(osm_layer* L, uint32_t T, float* out, const float* residual,
                bool picks_from_ids = false, uint32_t* status = nullptr) {
  osm_context* ctx = L->ctx;
  Scratch& s = ctx->sc;
  const osm_expert_layout& R = L->slab->layout;
  const osm_expert_layout& S = L->shared_slot ? L->shared_layout : R;
  const int Imax = (int)std::max(R.inter, L->shared_slot ? S.inter : 0u);
  const int max_active = (int)std::min<size_t>(L->g.E, (size_t)T * L->g.k) + (L->shared_slot ? 1 : 0);
  osm::GemvArgs g;
  osm::GemvLaunch gl;
  if (gemv_path(L, T, &g, &gl)) {
    // 1-2 tokens: bulk-copy decode kernels, combine fused into the down kernel
    g.x = ctx->cur_x;
    g.n_active = s.n_active;
    g.act = s.act;
    g.pair_tok = s.pair_tok;
    g.tp_pos = s.tp_pos;
    g.direct = 1;  // the picks of each token in order, no grouping needed
    g.ids = s.ids;
    g.pick_ptr = picks_from_ids ? nullptr : s.pick_ptr;
    g.mass = s.mass;
    g.slot_of = L->slot_of;
    g.status = status ? status : s.status;
    g.h = s.partial;
    g.weights = s.weights;
    g.sgate = s.sgate;
    g.residual = residual;
    g.out = out;
    {
      Prof p(ctx, kKGateUp);
      osm::launch_gemv_gateup(g, gl, ctx->stream, &ctx->launches);
    }
    int rc = check_launch(ctx, "gate/up gemv");
    if (rc) return rc;
    {
      Prof p(ctx, kKDown);
      osm::launch_gemv_down(g, gl, ctx->stream, &ctx->launches);
    }
    return check_launch(ctx, "down gemv + combine");
  }
  {
    // dg_min_tokens+ tokens: the int8 digit-plane tensor-core kernels over 16-pair chunks
    osm::TcArgs ta;
    osm::TcMaps maps;
    if (dg_use(L, T, &ta, &maps)) return run_dg(L, T, out, residual, ta, maps);
  }
  {
    // 3+ tokens: the 16-bit tensor-core kernels over 32-pair chunks of each expert
    osm::TcArgs ta;
    osm::TcMaps maps;
    if (tc_use(L, T, false, &ta, &maps)) return run_tc(L, T, out, residual, ta, maps, true, nullptr, false);
  }
  {
    // 3+ tokens: grouped projections over 8-token chunks of each expert
    osm::GrpArgs ga;
    size_t smem_gu = 0, smem_dn = 0;
    if (grouped_path(L, &ga, &smem_gu, &smem_dn)) {
      ga.x = ctx->cur_x;
      ga.n_ch = s.n_ch;
      ga.chunks = s.chunks;
      ga.act = s.act;
      ga.pair_tok = s.pair_tok;
      ga.pair_pick = s.pair_pick;
      ga.h = reinterpret_cast<float*>(s.hfrag);
      ga.partial = s.partial;
      ga.status = s.status;
      {
        Prof p(ctx, kKGateUp);
        osm::launch_grouped_gateup(ga, ctx->num_sms, smem_gu, ctx->stream, &ctx->launches);
      }
      int rc = check_launch(ctx, "grouped gate/up");
      if (rc) return rc;
      {
        Prof p(ctx, kKDown);
        osm::launch_grouped_down(ga, ctx->num_sms, smem_dn, ctx->stream, &ctx->launches);
      }
      rc = check_launch(ctx, "grouped down");
      if (rc) return rc;
      osm::CombineArgs c{};
      c.partial = s.partial;
      c.weights = s.weights;
      c.sgate = L->shared_slot ? s.sgate : nullptr;
      c.residual = residual;
      c.out = out;
      c.B = (int)T;
      c.H = L->g.H;
      c.k = L->g.k;
      {
        Prof p(ctx, kKCombine);
        osm::launch_combine(c, ctx->stream, &ctx->launches);
      }
      return check_launch(ctx, "combine");
    }
  }
  const int max_tg = (int)((size_t)T * (L->g.k + 1) / osm::kTokGroup) + max_active + 1;
  const int tchunk = (int)std::min<uint32_t>(T, 8);
  osm::ProjArgs gu{};
  fill_sections(gu.sec, R, S, true);
  gu.n_tg = s.n_tg;
  gu.act = s.act;
  gu.tg_expert = s.tg_expert;
  gu.tg_begin = s.tg_begin;
  gu.pair_tok = s.pair_tok;
  gu.frag_by_pair = 0;
  gu.raw = 0;
  gu.shared_first = L->shared_slot ? 1 : 0;
  gu.shared_ptr = L->shared_slot;
  gu.frag_stride = L->g.H / 8;
  gu.frag = s.xfrag;
  gu.fsum8 = s.xfsum8;
  gu.hfrag = s.hfrag;
  gu.hfsum8 = s.hfsum8;
  gu.hK = Imax;
  {
    Prof p(ctx, kKGateUp);
    osm::launch_proj(gu, osm::ProjKind::kGateUp, Imax, max_tg, ctx->grid_cap, tchunk, ctx->stream,
                     &ctx->launches);
  }
  int rc = check_launch(ctx, "gate/up projection");
  if (rc) return rc;
  osm::ProjArgs dn = gu;
  fill_sections(dn.sec, R, S, false);
  dn.frag_by_pair = 1;
  dn.frag_stride = Imax / 8;
  dn.frag = s.hfrag;
  dn.fsum8 = s.hfsum8;
  dn.hfrag = nullptr;
  dn.hfsum8 = nullptr;
  dn.out = s.partial;
  dn.out_row = nullptr;
  dn.pair_pick = s.pair_pick;
  dn.kp1 = (int)L->g.k + 1;
  dn.ostride = L->g.H;
  {
    Prof p(ctx, kKDown);
    osm::launch_proj(dn, Imax <= 512 ? osm::ProjKind::kDown : osm::ProjKind::kDown12, L->g.H,
                     max_tg, ctx->grid_cap, tchunk, ctx->stream, &ctx->launches);
  }
  rc = check_launch(ctx, "down projection");
  if (rc) return rc;
  osm::CombineArgs c{};
  c.partial = s.partial;
  c.weights = s.weights;
  c.sgate = L->shared_slot ? s.sgate : nullptr;
  c.residual = residual;
  c.out = out;
  c.B = (int)T;
  c.H = L->g.H;
  c.k = L->g.k;
  {
    Prof p(ctx, kKCombine);
    osm::launch_combine(c, ctx->stream, &ctx->launches);
  }
  return check_launch(ctx, "combine");
}

// The bf16 tensor-core path (osm_prefill.cu) for prefill-sized batches; fills
// the call-independent fields of pa.
bool prefill_path(osm_layer* L, osm::PfArgs* pa, size_t* smem) {
  if (!L->slab) return false;
  osm_context* ctx = L->ctx;
  const osm_expert_layout& R = L->slab->layout;
  const osm_expert_layout& S = L->shared_slot ? L->shared_layout : R;
  *pa = osm::PfArgs{};
  fill_sections(pa->gu, R, S, true);
  fill_sections(pa->dn, R, S, false);
  pa->H = L->g.H;
  pa->Imax = (int)std::max(R.inter, L->shared_slot ? S.inter : 0u);
  const int rmax = std::max(pa->gu.rows[0], L->shared_slot ? pa->gu.rows[1] : 0);
  pa->nmt_gu = (rmax + 127) / 128;
  pa->nmt_dn = (L->g.H + 127) / 128;
  return osm::prefill_configure(*pa, L->shared_slot ? 1 : 0, ctx->max_smem, smem);
}

int run_prefill(osm_layer* L, uint32_t T, float* out, const float* residual, osm::PfArgs pa,
                size_t smem, bool x_given = false, bool f16_out = false, bool combine = true) {
  osm_context* ctx = L->ctx;
  Scratch& s = ctx->sc;
  if ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(residual)) & 15)
    return fail(ctx, OSM_EINVAL, "prefill: out and residual must be 16-byte aligned");
  {
    osm::TcArgs ta;
    osm::TcMaps maps;
    if (tc_use(L, T, true, &ta, &maps))
      return run_tc(L, T, out, residual, ta, maps, false, x_given ? pa.xb : s.xbf, f16_out,
                    combine);
  }
  if (!x_given) pa.xb = s.xbf;
  pa.hb = reinterpret_cast<uint16_t*>(s.hfrag);
  pa.pb = reinterpret_cast<uint16_t*>(s.partial);
  pa.n_ch = s.n_ch;
  pa.chunks = s.chunks;
  pa.act = s.act;
  pa.pair_tok = s.pair_tok;
  pa.status = s.status;
  {
    Prof p(ctx, kKGateUp);
    osm::launch_prefill_gateup(pa, ctx->num_sms, smem, ctx->stream, &ctx->launches);
  }
  int rc = check_launch(ctx, "prefill gate/up");
  if (rc) return rc;
  {
    Prof p(ctx, kKDown);
    osm::launch_prefill_down(pa, ctx->num_sms, smem, ctx->stream, &ctx->launches);
  }
  rc = check_launch(ctx, "prefill down");
  if (rc || !combine) return rc;
  {
    Prof p(ctx, kKCombine);
    osm::launch_combine_bf16(pa.pb, s.tp_pos, s.weights, L->shared_slot ? s.sgate : nullptr, residual,
                             out, f16_out, s.status, (int)T, L->g.H, L->g.k, ctx->stream,
                             &ctx->launches);
  }
  return check_launch(ctx, "prefill combine");
}

// An 8-bit router's exact logits stream x by bulk copies: x must be 16-byte
// aligned.
int router_x_ok(osm_layer* L, const float* x) {
  if (L->g.q8 && (reinterpret_cast<uintptr_t>(x) & 15))
    return fail(L->ctx, OSM_EINVAL, "8-bit router: x must be 16-byte aligned");
  return OSM_OK;
}

int layer_ready(osm_layer* L, uint32_t T, bool need_slab) {
  if (!L || !L->ctx) return OSM_EINVAL;
  osm_context* ctx = L->ctx;
  if (T == 0) return fail(ctx, OSM_EINVAL, "token count must be non-zero");
  if (T > ctx->max_tokens) return fail(ctx, OSM_EINVAL, "token count exceeds context max_tokens");
  if (need_slab && !L->slab) return fail(ctx, OSM_EINVAL, "layer has no expert slab bound");
  const size_t I = std::max<size_t>(L->slab ? L->slab->layout.inter : 64,
                                    L->shared_slot ? L->shared_layout.inter : 0);
  return ensure_scratch(ctx, T, L->g.H, L->g.E, L->g.k, I, L->g.H);
}

}  // namespace

extern "C" {

int osm_expert_layout_packed(uint32_t hidden, uint32_t inter, uint32_t group,
                             osm_expert_layout* out) {
  if (!out || group == 0 || hidden % group || inter % group || hidden % 8 || inter % 8)
    return OSM_EINVAL;
  const uint64_t H = hidden, I = inter;
  const uint64_t gu_w = I * H / 2, gu_m = I * (H / group) * 2, dn_w = H * I / 2,
                 dn_m = H * (I / group) * 2;
  osm_expert_layout L{};
  L.hidden = hidden;
  L.inter = inter;
  L.group = group;
  L.gate_w = 0;
  L.gate_s = L.gate_w + gu_w;
  L.gate_b = L.gate_s + gu_m;
  L.up_w = L.gate_b + gu_m;
  L.up_s = L.up_w + gu_w;
  L.up_b = L.up_s + gu_m;
  L.down_w = L.up_b + gu_m;
  L.down_s = L.down_w + dn_w;
  L.down_b = L.down_s + dn_m;
  L.stride = L.down_b + dn_m;
  *out = L;
  return OSM_OK;
}

int osm_context_create(int device, uint32_t max_tokens, osm_context** out) {
  if (!out) return OSM_EINVAL;
  *out = nullptr;
  if (max_tokens == 0) return OSM_EINVAL;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return OSM_ECUDA;
  DeviceGuard dg(device);
  auto* ctx = new (std::nothrow) osm_context();
  if (!ctx) return OSM_ENOMEM;
  ctx->device = device;
  ctx->max_tokens = max_tokens;
  if (cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete ctx;
    return OSM_ECUDA;
  }
  ctx->stream = ctx->own_stream;
  if (cudaMalloc(&ctx->status_blk, 32) != cudaSuccess || cudaMemset(ctx->status_blk, 0, 32) != cudaSuccess) {
    if (ctx->status_blk) cudaFree(ctx->status_blk);
    cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return OSM_ENOMEM;
  }
  ctx->sc.status = static_cast<uint32_t*>(ctx->status_blk);
  ctx->sc.range_status = static_cast<uint32_t*>(ctx->status_blk) + 1;
  ctx->sc.exact_count = reinterpret_cast<unsigned long long*>(static_cast<char*>(ctx->status_blk) + 8);
  ctx->sc.early_status = static_cast<uint32_t*>(ctx->status_blk) + 4;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) == cudaSuccess && sms > 0) {
    ctx->grid_cap = sms * 4;
    ctx->num_sms = sms;
  }
  int optin = 0;
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  // dynamic limit = opt-in maximum minus room for each kernel's static smem
  // (the decode kernels have none)
  const int max_smem = optin > 64 * 1024 ? optin - 16 * 1024 : 48 * 1024;
  ctx->max_smem = optin > 64 * 1024 ? optin : 48 * 1024;
  osm::init_router_attributes(max_smem);
  osm::init_expert_attributes(max_smem);
  osm::init_gemv_attributes(ctx->max_smem);
  osm::init_grouped_attributes(ctx->max_smem);
  osm::init_prefill_attributes(ctx->max_smem);
  osm::init_tc_attributes(ctx->max_smem);
  osm::init_dg_attributes(ctx->max_smem);
  {
    const char* v = std::getenv("OSM_DISABLE_TC");
    ctx->tc_enabled = !(v && v[0] && v[0] != '0');
    const char* d = std::getenv("OSM_TC_DECODE");
    ctx->tc_decode = d && d[0] && d[0] != '0';
    const char* g = std::getenv("OSM_DG_DECODE");
    ctx->dg_decode = !(g && g[0] == '0');
    const char* gm = std::getenv("OSM_DG_MIN_TOKENS");
    if (gm && gm[0]) ctx->dg_min_tokens = (uint32_t)std::strtoul(gm, nullptr, 10);
  }
  const cudaError_t ae = cudaGetLastError();
  if (ae != cudaSuccess) {
    cudaFree(ctx->status_blk);
    cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return OSM_ECUDA;
  }
  *out = ctx;
  return OSM_OK;
}

int osm_device_info(int device, char* name, size_t name_bytes, uint32_t* sms,
                    uint32_t* runtime_version) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return OSM_ECUDA;
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return OSM_ECUDA;
  if (name && name_bytes) {
    std::strncpy(name, prop.name, name_bytes - 1);
    name[name_bytes - 1] = '\0';
  }
  if (sms) *sms = (uint32_t)prop.multiProcessorCount;
  int rv = 0;
  cudaRuntimeGetVersion(&rv);
  if (runtime_version) *runtime_version = (uint32_t)rv;
  return OSM_OK;
}

int osm_context_destroy(osm_context* ctx) {
  if (!ctx) return OSM_EINVAL;
  DeviceGuard dg(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->sc.base) cudaFree(ctx->sc.base);
  for (void* p : ctx->retired) cudaFree(p);
  if (ctx->status_blk) cudaFree(ctx->status_blk);
  for (const ProfRec& r : ctx->recs) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  for (cudaEvent_t e : ctx->ev_pool) cudaEventDestroy(e);
  if (ctx->picks_host) cudaFreeHost(ctx->picks_host);
  if (ctx->picks_ev) cudaEventDestroy(ctx->picks_ev);
  if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
  delete ctx;
  return OSM_OK;
}

const char* osm_last_error(const osm_context* ctx) { return ctx ? ctx->err.c_str() : "null context"; }
int osm_context_device(const osm_context* ctx) { return ctx ? ctx->device : -1; }
void* osm_context_stream(const osm_context* ctx) { return ctx ? (void*)ctx->stream : nullptr; }
uint64_t osm_context_launches(const osm_context* ctx) { return ctx ? ctx->launches : 0; }

int osm_context_profile(osm_context* ctx, int enable) {
  if (!ctx) return OSM_EINVAL;
  ctx->prof_on = enable != 0;
  return OSM_OK;
}

int osm_context_profile_read(osm_context* ctx, double* ms, uint64_t* launches) {
  if (!ctx) return OSM_EINVAL;
  DeviceGuard dg(ctx->device);
  OSM_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  for (const ProfRec& r : ctx->recs) {
    float t = 0.0f;
    if (cudaEventElapsedTime(&t, r.a, r.b) == cudaSuccess && r.kind >= 0 &&
        r.kind < OSM_KERNEL_KINDS) {
      if (ms) ms[r.kind] += t;
      if (launches) launches[r.kind] += 1;
    } else {
      cudaGetLastError();  // an unrecorded pair is skipped, not a sticky error
    }
    ctx->ev_pool.push_back(r.a);
    ctx->ev_pool.push_back(r.b);
  }
  ctx->recs.clear();
  return OSM_OK;
}

const char* osm_kernel_kind_name(int kind) {
  return (kind >= 0 && kind < OSM_KERNEL_KINDS) ? kKindNames[kind] : "unknown";
}

int osm_context_set_stream(osm_context* ctx, void* stream) {
  if (!ctx) return OSM_EINVAL;
  ctx->stream = static_cast<cudaStream_t>(stream);
  return OSM_OK;
}

int osm_context_reset_stream(osm_context* ctx) {
  if (!ctx) return OSM_EINVAL;
  ctx->stream = ctx->own_stream;
  return OSM_OK;
}

int osm_context_synchronize(osm_context* ctx) {
  if (!ctx) return OSM_EINVAL;
  DeviceGuard dg(ctx->device);
  OSM_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return OSM_OK;
}

int osm_context_status(osm_context* ctx, uint32_t* status, uint64_t* exact_tokens) {
  if (!ctx) return OSM_EINVAL;
  DeviceGuard dg(ctx->device);
  uint32_t st = 0;
  unsigned long long ex = 0;
  OSM_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  OSM_CUDA(ctx, cudaMemcpy(&st, ctx->sc.status, 4, cudaMemcpyDeviceToHost));
  OSM_CUDA(ctx, cudaMemcpy(&ex, ctx->sc.exact_count, 8, cudaMemcpyDeviceToHost));
  OSM_CUDA(ctx, cudaMemset(ctx->sc.status, 0, 4));
  OSM_CUDA(ctx, cudaMemset(ctx->sc.exact_count, 0, 8));
  st |= ctx->pending_status;
  ctx->pending_status = 0;
  if (status) *status = st;
  if (exact_tokens) *exact_tokens = ex;
  return OSM_OK;
}

int osm_test_set_copy_wait_polls(int device, uint32_t polls) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return OSM_EINVAL;
  DeviceGuard dg(device);
  const uint32_t v = polls == UINT32_MAX ? osm::kCopyPolls : polls;
  if (osm::set_first_wait_polls_gemv(v) != cudaSuccess ||
      osm::set_first_wait_polls_prefill(v) != cudaSuccess ||
      osm::set_first_wait_polls_router(v) != cudaSuccess)
    return OSM_ECUDA;
  return OSM_OK;
}

int osm_device_alloc(osm_context* ctx, size_t bytes, void** dev) {
  if (!ctx || !dev) return OSM_EINVAL;
  DeviceGuard dg(ctx->device);
  if (cudaMalloc(dev, std::max<size_t>(bytes, 1)) != cudaSuccess)
    return fail(ctx, OSM_ENOMEM, "device allocation failed");
  return OSM_OK;
}

int osm_device_free(osm_context* ctx, void* dev) {
  if (!ctx) return OSM_EINVAL;
  DeviceGuard dg(ctx->device);
  OSM_CUDA(ctx, cudaFree(dev));
  return OSM_OK;
}

int osm_upload(osm_context* ctx, void* dev, const void* host, size_t bytes) {
  if (!ctx || (!dev && bytes) || (!host && bytes)) return OSM_EINVAL;
  DeviceGuard dg(ctx->device);
  OSM_CUDA(ctx, cudaMemcpyAsync(dev, host, bytes, cudaMemcpyHostToDevice, ctx->stream));
  OSM_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return OSM_OK;
}

int osm_download(osm_context* ctx, void* host, const void* dev, size_t bytes) {
  if (!ctx || (!dev && bytes) || (!host && bytes)) return OSM_EINVAL;
  DeviceGuard dg(ctx->device);
  OSM_CUDA(ctx, cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  OSM_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return OSM_OK;
}

int osm_host_alloc_pinned(size_t bytes, void** host) {
  if (!host) return OSM_EINVAL;
  if (cudaHostAlloc(host, std::max<size_t>(bytes, 1), cudaHostAllocDefault) != cudaSuccess)
    return OSM_ENOMEM;
  return OSM_OK;
}

int osm_host_free_pinned(void* host) {
  return cudaFreeHost(host) == cudaSuccess ? OSM_OK : OSM_ECUDA;
}

namespace {

// The Q4 geometry every dequant / GEMV entry accepts.
int check_q4(osm_context* ctx, const char* what, const void* packed, const void* sc,
             const void* bi, uint32_t rows, uint32_t in_dim, uint32_t group) {
  if (group == 0 || in_dim == 0 || in_dim % 8 || in_dim % group || rows == 0 || !packed || !sc ||
      !bi)
    return fail(ctx, OSM_EINVAL,
                std::string(what) +
                    ": in_dim must be a non-zero multiple of 8 and of the group size");
  if ((uint64_t)rows * in_dim > (uint64_t)INT32_MAX * 8)
    return fail(ctx, OSM_EINVAL, std::string(what) + ": matrix too large");
  return OSM_OK;
}

int q4_dequant_any(osm_context* ctx, const uint32_t* packed, const void* sc, const void* bi,
                   bool f32, uint32_t rows, uint32_t in_dim, uint32_t group, float* out) {
  if (!ctx) return OSM_EINVAL;
  if (int rc = check_q4(ctx, "q4 dequant", packed, sc, bi, rows, in_dim, group)) return rc;
  if (!out) return fail(ctx, OSM_EINVAL, "q4 dequant: null output");
  DeviceGuard dg(ctx->device);
  osm::launch_dequant(packed, sc, bi, f32, (int)rows, (int)in_dim, (int)group, out, ctx->stream,
                      &ctx->launches);
  return check_launch(ctx, "q4 dequant");
}

int q4_gemv_any(osm_context* ctx, const uint32_t* packed, const void* sc, const void* bi, bool f32,
                uint32_t out_dim, uint32_t in_dim, uint32_t group, const float* x,
                uint32_t tokens, float* y) {
  if ((uint64_t)out_dim * tokens > (uint64_t)INT32_MAX / 32)
    return fail(ctx, OSM_EINVAL, "q4 gemv: out_dim * tokens too large");
  DeviceGuard dg(ctx->device);
  osm::launch_gemv_any(packed, sc, bi, f32, (int)out_dim, (int)in_dim, (int)group, x, (int)tokens,
                       y, ctx->stream, &ctx->launches);
  return check_launch(ctx, "q4 gemv");
}

}  // namespace

int osm_q4_dequant(osm_context* ctx, const uint32_t* packed, const uint16_t* sc,
                   const uint16_t* bi, uint32_t rows, uint32_t in_dim, uint32_t group,
                   float* out) {
  return q4_dequant_any(ctx, packed, sc, bi, false, rows, in_dim, group, out);
}

int osm_q4_dequant_f32(osm_context* ctx, const uint32_t* packed, const float* sc, const float* bi,
                       uint32_t rows, uint32_t in_dim, uint32_t group, float* out) {
  return q4_dequant_any(ctx, packed, sc, bi, true, rows, in_dim, group, out);
}

int osm_q4_gemv_f32(osm_context* ctx, const uint32_t* packed, const float* sc, const float* bi,
                    uint32_t out_dim, uint32_t in_dim, uint32_t group, const float* x,
                    uint32_t tokens, float* y) {
  if (!ctx) return OSM_EINVAL;
  if (int rc = check_q4(ctx, "q4 gemv", packed, sc, bi, out_dim, in_dim, group)) return rc;
  if (!x || !y || tokens == 0) return fail(ctx, OSM_EINVAL, "q4 gemv: null vector or no tokens");
  return q4_gemv_any(ctx, packed, sc, bi, true, out_dim, in_dim, group, x, tokens, y);
}

int osm_q4_gemv(osm_context* ctx, const uint32_t* packed, const uint16_t* sc,
                const uint16_t* bi, uint32_t out_dim, uint32_t in_dim, uint32_t group,
                const float* x, uint32_t tokens, float* y) {
  if (!ctx) return OSM_EINVAL;
  if (int rc = check_q4(ctx, "q4 gemv", packed, sc, bi, out_dim, in_dim, group)) return rc;
  if (!x || !y || tokens == 0) return fail(ctx, OSM_EINVAL, "q4 gemv: null vector or no tokens");
  if (group != 64 || in_dim % 64 || in_dim > 2048 || out_dim % 16 || tokens > ctx->max_tokens)
    return q4_gemv_any(ctx, packed, sc, bi, false, out_dim, in_dim, group, x, tokens, y);
  DeviceGuard dg(ctx->device);
  int rc = ensure_scratch(ctx, tokens, 0, 1, 1, 64, in_dim);
  if (rc) return rc;
  Scratch& s = ctx->sc;
  osm::launch_frag_prep(x, (int)tokens, (int)in_dim, s.xfrag, s.xfsum8, ctx->stream, &ctx->launches);
  osm::launch_setup_single((int)tokens, nullptr, s.n_active, s.act, s.n_tg, s.tg_expert,
                           s.tg_begin, s.pair_tok, s.pair_pick, s.out_row, ctx->stream,
                           &ctx->launches);
  osm::ProjArgs a{};
  for (int i = 0; i < 2; ++i) {
    a.sec.w[i] = a.sec.w2[i] = (uint64_t)(uintptr_t)packed;
    a.sec.s[i] = a.sec.s2[i] = (uint64_t)(uintptr_t)sc;
    a.sec.b[i] = a.sec.b2[i] = (uint64_t)(uintptr_t)bi;
    a.sec.rows[i] = (int)out_dim;
    a.sec.K[i] = (int)in_dim;
  }
  a.n_tg = s.n_tg;
  a.act = s.act;
  a.tg_expert = s.tg_expert;
  a.tg_begin = s.tg_begin;
  a.pair_tok = s.pair_tok;
  a.frag_by_pair = 0;
  a.raw = 1;
  a.frag_stride = (int)in_dim / 8;
  a.frag = s.xfrag;
  a.fsum8 = s.xfsum8;
  a.out = y;
  a.out_row = s.out_row;
  a.pair_pick = s.pair_pick;
  a.kp1 = 1;
  a.ostride = (int)out_dim;
  osm::launch_proj(a, osm::ProjKind::kSingle, (int)out_dim,
                   (int)((tokens + osm::kTokGroup - 1) / osm::kTokGroup), ctx->grid_cap,
                   (int)std::min<uint32_t>(tokens, 8), ctx->stream, &ctx->launches);
  return check_launch(ctx, "q4 gemv");
}

int osm_swiglu(osm_context* ctx, const float* g, const float* u, float* out, size_t n) {
  if (!ctx || (n && (!g || !u || !out))) return OSM_EINVAL;
  DeviceGuard dg(ctx->device);
  if (n == 0) return OSM_OK;
  osm::launch_swiglu(g, u, out, n, ctx->stream, &ctx->launches);
  return check_launch(ctx, "swiglu");
}

int osm_weighted_accumulate(osm_context* ctx, const float* src, float w, float* acc, size_t n) {
  if (!ctx || (n && (!src || !acc))) return OSM_EINVAL;
  if (!std::isfinite(w)) return fail(ctx, OSM_EINVAL, "weighted accumulate: non-finite weight");
  DeviceGuard dg(ctx->device);
  if (n == 0) return OSM_OK;
  osm::launch_waccum(src, w, acc, n, ctx->stream, &ctx->launches);
  return check_launch(ctx, "weighted accumulate");
}

int osm_rms_norm(osm_context* ctx, float* values, uint32_t rows, uint32_t dim, const float* w,
                 float eps, uint32_t flags) {
  if (!ctx) return OSM_EINVAL;
  if (rows == 0 || dim == 0 || !values) return fail(ctx, OSM_EINVAL, "rms_norm: invalid shape");
  if (!(eps >= 0.0f)) return fail(ctx, OSM_EINVAL, "rms_norm: eps must be non-negative");
  DeviceGuard dg(ctx->device);
  osm::launch_rmsnorm(values, values, (int)rows, (int)dim, w, eps, (flags & OSM_RMSNORM_EXACT) != 0,
                      ctx->stream, &ctx->launches);
  return check_launch(ctx, "rms_norm");
}

int osm_expert_forward(osm_context* ctx, const void* slot, const osm_expert_layout* layout,
                       const float* x, uint32_t tokens, float* out) {
  if (!ctx) return OSM_EINVAL;
  if (!slot || !x || !out || tokens == 0 || !layout_ok(layout))
    return fail(ctx, OSM_EINVAL, "expert forward: invalid arguments or unsupported layout");
  if (tokens > ctx->max_tokens) return fail(ctx, OSM_EINVAL, "expert forward: tokens > max_tokens");
  DeviceGuard dg(ctx->device);
  const osm_expert_layout& L = *layout;
  int rc = ensure_scratch(ctx, tokens, L.hidden, 1, 1, L.inter, L.hidden);
  if (rc) return rc;
  Scratch& s = ctx->sc;
  osm::launch_frag_prep(x, (int)tokens, (int)L.hidden, s.xfrag, s.xfsum8, ctx->stream,
                        &ctx->launches);
  osm::launch_setup_single((int)tokens, static_cast<const uint8_t*>(slot), s.n_active, s.act,
                           s.n_tg, s.tg_expert, s.tg_begin, s.pair_tok, s.pair_pick, s.out_row,
                           ctx->stream, &ctx->launches);
  osm::ProjArgs gu{};
  fill_sections(gu.sec, L, L, true);
  gu.n_tg = s.n_tg;
  gu.act = s.act;
  gu.tg_expert = s.tg_expert;
  gu.tg_begin = s.tg_begin;
  gu.pair_tok = s.pair_tok;
  gu.frag_stride = (int)L.hidden / 8;
  gu.frag = s.xfrag;
  gu.fsum8 = s.xfsum8;
  gu.hfrag = s.hfrag;
  gu.hfsum8 = s.hfsum8;
  gu.hK = (int)L.inter;
  const int ntg1 = (int)((tokens + osm::kTokGroup - 1) / osm::kTokGroup);
  const int tch1 = (int)std::min<uint32_t>(tokens, 8);
  osm::launch_proj(gu, osm::ProjKind::kGateUp, (int)L.inter, ntg1, ctx->grid_cap, tch1, ctx->stream,
                   &ctx->launches);
  rc = check_launch(ctx, "expert gate/up");
  if (rc) return rc;
  osm::ProjArgs dn = gu;
  fill_sections(dn.sec, L, L, false);
  dn.frag_by_pair = 1;
  dn.frag_stride = (int)L.inter / 8;
  dn.frag = s.hfrag;
  dn.fsum8 = s.hfsum8;
  dn.out = out;
  dn.out_row = s.out_row;
  dn.pair_pick = s.pair_pick;
  dn.kp1 = 1;
  dn.ostride = (int)L.hidden;
  osm::launch_proj(dn, L.inter <= 512 ? osm::ProjKind::kDown : osm::ProjKind::kDown12,
                   (int)L.hidden, ntg1, ctx->grid_cap, tch1, ctx->stream, &ctx->launches);
  return check_launch(ctx, "expert down");
}

int osm_slab_create(osm_context* ctx, const osm_expert_layout* layout, uint32_t slots,
                    osm_slab** out) {
  if (!ctx || !out) return OSM_EINVAL;
  *out = nullptr;
  if (slots == 0 || !layout_ok(layout))
    return fail(ctx, OSM_EINVAL, "slab: zero slots or unsupported expert layout");
  DeviceGuard dg(ctx->device);
  auto* s = new (std::nothrow) osm_slab();
  if (!s) return OSM_ENOMEM;
  s->ctx = ctx;
  s->layout = *layout;
  s->slots = slots;
  if (cudaMalloc(&s->base, (size_t)slots * layout->stride) != cudaSuccess) {
    delete s;
    return fail(ctx, OSM_ENOMEM, "slab: device allocation failed");
  }
  if (cudaStreamCreateWithFlags(&s->side, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&s->ev, cudaEventDisableTiming) != cudaSuccess) {
    cudaFree(s->base);
    delete s;
    return fail(ctx, OSM_ECUDA, "slab: stream/event creation failed");
  }
  s->tc_ok = encode_expert_maps(s->tc_maps, s->base, s->layout, slots);
  *out = s;
  return OSM_OK;
}

int osm_slab_destroy(osm_slab* s) {
  if (!s) return OSM_EINVAL;
  DeviceGuard dg(s->ctx->device);
  cudaStreamSynchronize(s->side);
  cudaStreamSynchronize(s->ctx->stream);
  cudaFree(s->base);
  cudaEventDestroy(s->ev);
  cudaStreamDestroy(s->side);
  delete s;
  return OSM_OK;
}

uint32_t osm_slab_slots(const osm_slab* s) { return s ? s->slots : 0; }

int osm_slab_layout(const osm_slab* s, osm_expert_layout* out) {
  if (!s || !out) return OSM_EINVAL;
  *out = s->layout;
  return OSM_OK;
}

void* osm_slab_slot_ptr(const osm_slab* s, uint32_t slot) {
  if (!s || slot >= s->slots) return nullptr;
  return s->base + (size_t)slot * s->layout.stride;
}

uint64_t osm_slab_h2d_bytes(const osm_slab* s) { return s ? s->h2d_bytes : 0; }

int osm_slab_fill_async(osm_slab* s, uint32_t slot, const void* host) {
  if (!s || !host) return OSM_EINVAL;
  osm_context* ctx = s->ctx;
  if (slot >= s->slots) return fail(ctx, OSM_EINVAL, "slab fill: slot out of range");
  DeviceGuard dg(ctx->device);
  // A fill must not overwrite a slot that queued kernels still read.
  OSM_CUDA(ctx, cudaEventRecord(s->ev, ctx->stream));
  OSM_CUDA(ctx, cudaStreamWaitEvent(s->side, s->ev, 0));
  OSM_CUDA(ctx, cudaMemcpyAsync(s->base + (size_t)slot * s->layout.stride, host, s->layout.stride,
                                cudaMemcpyHostToDevice, s->side));
  OSM_CUDA(ctx, cudaEventRecord(s->ev, s->side));
  OSM_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, s->ev, 0));
  s->h2d_bytes += s->layout.stride;
  return OSM_OK;
}

int osm_slab_fill_wait(osm_slab* s, uint32_t timeout_ms) {
  if (!s) return OSM_EINVAL;
  osm_context* ctx = s->ctx;
  DeviceGuard dg(ctx->device);
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t e = cudaEventQuery(s->ev);
    if (e == cudaSuccess) return OSM_OK;
    if (e != cudaErrorNotReady) return cuda_fail(ctx, e, "slab fill wait");
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                        std::chrono::steady_clock::now() - t0).count();
    if (ms >= (long long)timeout_ms)
      return fail(ctx, OSM_ETIMEOUT, "slab fill wait: timed out");
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

int osm_layer_create(osm_context* ctx, const osm_layer_desc* d, osm_layer** out) {
  if (!ctx || !d || !out) return OSM_EINVAL;
  *out = nullptr;
  if (d->hidden == 0 || d->experts == 0 || d->top_k == 0)
    return fail(ctx, OSM_EINVAL, "qwen router: dimensions and top_k must be non-zero");
  if (d->top_k > d->experts) return fail(ctx, OSM_EINVAL, "qwen router: top_k cannot exceed expert_count");
  if (d->experts > (uint32_t)osm::kMaxExperts - 1 || d->top_k > (uint32_t)osm::kMaxTopK)
    return fail(ctx, OSM_EINVAL, "router: at most 1023 experts and top_k 32 are supported");
  if (d->hidden > 8192) return fail(ctx, OSM_EINVAL, "router: hidden must be <= 8192");
  if (!d->router_weight_host) return fail(ctx, OSM_EINVAL, "router weight missing");
  const size_t EH = (size_t)d->experts * d->hidden;
  bool bf16_exact = true;
  for (size_t i = 0; i < EH; ++i) {
    const float v = d->router_weight_host[i];
    if (!std::isfinite(v))
      return fail(ctx, OSM_EINVAL, "qwen router: router weight contains non-finite value");
    uint32_t u;
    std::memcpy(&u, &v, 4);
    if (u & 0xFFFFu) bf16_exact = false;
  }
  if (d->shared_slot_host) {
    if (!layout_ok(&d->shared_layout) || d->shared_layout.hidden != d->hidden)
      return fail(ctx, OSM_EINVAL, "shared expert layout unsupported or hidden mismatch");
    if (!d->shared_gate_host) return fail(ctx, OSM_EINVAL, "shared expert scalar gate missing");
  }
  DeviceGuard dg(ctx->device);
  auto* L = new (std::nothrow) osm_layer();
  if (!L) return OSM_ENOMEM;
  L->ctx = ctx;
  osm::RouterGeom g{};
  g.H = (int)d->hidden;
  g.Hp = (int)align_up(d->hidden, 256);
  g.c = g.Hp / 32;
  g.nvec = g.c / 8;
  g.E = (int)d->experts;
  g.k = (int)d->top_k;
  g.f32w = bf16_exact ? 0 : 1;
  L->g = g;
  L->norm = d->norm_topk_prob ? 1 : 0;
  L->norm_eps = d->norm_eps;
  auto cleanup = [&](int code, const char* msg) {
    osm_layer_destroy(L);
    return fail(ctx, code, msg);
  };
  float* tmp = nullptr;
  if (cudaMalloc(&L->wp, (size_t)g.E * g.Hp * (g.f32w ? 4 : 2)) != cudaSuccess ||
      cudaMalloc(&L->wx, osm::router_tile_bytes(g)) != cudaSuccess ||
      cudaMalloc(&tmp, EH * 4) != cudaSuccess)
    return cleanup(OSM_ENOMEM, "layer: router allocation failed");
  cudaMemcpyAsync(tmp, d->router_weight_host, EH * 4, cudaMemcpyHostToDevice, ctx->stream);
  osm::launch_router_pack(tmp, g, L->wp, ctx->stream, &ctx->launches);
  osm::launch_router_tile(tmp, g, L->wx, ctx->stream, &ctx->launches);
  cudaStreamSynchronize(ctx->stream);
  cudaFree(tmp);
  if (d->logit_bias_host) {
    for (uint32_t e = 0; e < d->experts; ++e)
      if (!std::isfinite(d->logit_bias_host[e])) return cleanup(OSM_EINVAL, "logit bias non-finite");
    if (cudaMalloc(&L->bias, d->experts * 4) != cudaSuccess)
      return cleanup(OSM_ENOMEM, "layer: bias allocation failed");
    cudaMemcpy(L->bias, d->logit_bias_host, d->experts * 4, cudaMemcpyHostToDevice);
  }
  if (d->shared_slot_host) {
    L->shared_layout = d->shared_layout;
    if (cudaMalloc(&L->shared_slot, d->shared_layout.stride) != cudaSuccess ||
        cudaMalloc(&L->sgate_w, d->hidden * 4) != cudaSuccess)
      return cleanup(OSM_ENOMEM, "layer: shared expert allocation failed");
    cudaMemcpy(L->shared_slot, d->shared_slot_host, d->shared_layout.stride, cudaMemcpyHostToDevice);
    cudaMemcpy(L->sgate_w, d->shared_gate_host, d->hidden * 4, cudaMemcpyHostToDevice);
    L->tc_shared_ok = encode_expert_maps(L->tc_shared, L->shared_slot, L->shared_layout, 1);
  }
  if (d->norm_weight_host) {
    if (cudaMalloc(&L->norm_w, d->hidden * 4) != cudaSuccess)
      return cleanup(OSM_ENOMEM, "layer: norm weight allocation failed");
    cudaMemcpy(L->norm_w, d->norm_weight_host, d->hidden * 4, cudaMemcpyHostToDevice);
  }
  if (cudaMalloc(&L->slot_of, d->experts * 4) != cudaSuccess)
    return cleanup(OSM_ENOMEM, "layer: slot table allocation failed");
  L->slot_host.assign(d->experts, -1);
  cudaMemcpy(L->slot_of, L->slot_host.data(), d->experts * 4, cudaMemcpyHostToDevice);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cleanup(OSM_ECUDA, cudaGetErrorString(e));
  *out = L;
  return OSM_OK;
}

int osm_layer_destroy(osm_layer* L) {
  if (!L) return OSM_EINVAL;
  DeviceGuard dg(L->ctx->device);
  cudaStreamSynchronize(L->ctx->stream);
  cudaFree(L->wp);
  cudaFree(L->wx);
  cudaFree(L->qmeta);
  cudaFree(L->bias);
  cudaFree(L->sgate_w);
  cudaFree(L->shared_slot);
  cudaFree(L->norm_w);
  cudaFree(L->slot_of);
  delete L;
  return OSM_OK;
}

int osm_layer_set_router_q8(osm_layer* L, const uint32_t* packed, const uint16_t* scales_bf16,
                            const uint16_t* biases_bf16, uint32_t group) {
  if (!L || !packed || !scales_bf16 || !biases_bf16) return OSM_EINVAL;
  osm_context* ctx = L->ctx;
  if (group != 64) return fail(ctx, OSM_EINVAL, "8-bit router: group must be 64");
  if (L->g.H % 256 || L->g.E % 32)
    return fail(ctx, OSM_EINVAL, "8-bit router: hidden must be a multiple of 256, experts of 32");
  if (ctx->plans_alive > 0) return fail(ctx, OSM_EINVAL, "8-bit router: set it before creating plans");
  const size_t E = (size_t)L->g.E, H = (size_t)L->g.H, G = H / 64;
  std::vector<uint32_t> meta(E * G);
  for (size_t i = 0; i < E * G; ++i) {
    const uint32_t sb = scales_bf16[i], bb = biases_bf16[i];
    if ((sb & 0x7F80u) == 0x7F80u || (bb & 0x7F80u) == 0x7F80u)
      return fail(ctx, OSM_EINVAL, "8-bit router: non-finite scale or bias");
    meta[i] = sb | (bb << 16);
  }
  DeviceGuard dg(ctx->device);
  osm::RouterGeom g = L->g;
  g.q8 = 1;
  g.f32w = 0;
  void *wp = nullptr, *wx = nullptr, *qm = nullptr, *tmp = nullptr;
  if (cudaMalloc(&wp, E * g.Hp) != cudaSuccess || cudaMalloc(&wx, osm::router_tile_bytes(g)) != cudaSuccess ||
      cudaMalloc(&qm, E * G * 4) != cudaSuccess || cudaMalloc(&tmp, E * H) != cudaSuccess) {
    cudaFree(wp);
    cudaFree(wx);
    cudaFree(qm);
    cudaFree(tmp);
    return fail(ctx, OSM_ENOMEM, "8-bit router: allocation failed");
  }
  cudaStreamSynchronize(ctx->stream);  // no queued call still reads the old router
  cudaMemcpy(tmp, packed, E * H, cudaMemcpyHostToDevice);  // the words' bytes, element order
  cudaMemcpy(qm, meta.data(), E * G * 4, cudaMemcpyHostToDevice);
  osm::launch_router_pack_q8(static_cast<const uint8_t*>(tmp), g, wp, ctx->stream, &ctx->launches);
  osm::launch_router_tile_q8(static_cast<const uint8_t*>(tmp), g, wx, ctx->stream, &ctx->launches);
  const cudaError_t e = cudaStreamSynchronize(ctx->stream);
  cudaFree(tmp);
  if (e != cudaSuccess) {
    cudaFree(wp);
    cudaFree(wx);
    cudaFree(qm);
    return cuda_fail(ctx, e, "8-bit router: layout kernels");
  }
  cudaFree(L->wp);
  cudaFree(L->wx);
  cudaFree(L->qmeta);
  L->wp = wp;
  L->wx = wx;
  L->qmeta = static_cast<uint32_t*>(qm);
  L->g = g;
  return OSM_OK;
}

int osm_layer_bind_slab(osm_layer* L, osm_slab* slab, const int32_t* slot_of) {
  if (!L || !slab || !slot_of) return OSM_EINVAL;
  osm_context* ctx = L->ctx;
  if (slab->ctx != ctx) return fail(ctx, OSM_EINVAL, "slab belongs to another context");
  if (slab->layout.hidden != (uint32_t)L->g.H)
    return fail(ctx, OSM_EINVAL, "slab expert geometry does not match the router hidden size");
  for (int e = 0; e < L->g.E; ++e)
    if (slot_of[e] >= (int32_t)slab->slots) return fail(ctx, OSM_EINVAL, "slot index out of range");
  DeviceGuard dg(ctx->device);
  L->slab = slab;
  L->slot_host.assign(slot_of, slot_of + L->g.E);
  OSM_CUDA(ctx, cudaMemcpyAsync(L->slot_of, L->slot_host.data(), L->g.E * 4,
                                cudaMemcpyHostToDevice, ctx->stream));
  OSM_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return OSM_OK;
}

int osm_layer_set_slot(osm_layer* L, uint32_t expert, int32_t slot) {
  if (!L) return OSM_EINVAL;
  osm_context* ctx = L->ctx;
  if (expert >= (uint32_t)L->g.E) return fail(ctx, OSM_EINVAL, "expert out of range");
  if (L->slab && slot >= (int32_t)L->slab->slots) return fail(ctx, OSM_EINVAL, "slot out of range");
  DeviceGuard dg(ctx->device);
  L->slot_host[expert] = slot;
  // pageable-source copy: the value is staged before the call returns
  OSM_CUDA(ctx, cudaMemcpyAsync(L->slot_of + expert, &L->slot_host[expert], 4,
                                cudaMemcpyHostToDevice, ctx->stream));
  return OSM_OK;
}

int osm_moe_route(osm_layer* L, const float* x, uint32_t T, uint32_t* ids, float* w, float* mass,
                  uint32_t flags) {
  int rc = layer_ready(L, T, false);
  if (rc) return rc;
  if (!x) return fail(L->ctx, OSM_EINVAL, "route: null input");
  if (int e = router_x_ok(L, x)) return e;
  osm_context* ctx = L->ctx;
  DeviceGuard dg(ctx->device);
  osm::RouterArgs a = router_args(L, x, T);
  a.force_exact = (flags & OSM_ROUTE_EXACT) ? 1 : 0;
  a.ids_out = ids;
  a.weights_out = w;
  a.mass_out = mass;
  a.do_group = 0;
  a.xfrag = nullptr;
  a.sgate_w = nullptr;
  a.pick_ptr = nullptr;  // routing only: residency is the caller's next step
  launch_router_pair(ctx, a);
  return check_launch(ctx, "router");
}

int osm_moe_route_logits(osm_layer* L, const float* x, uint32_t T, float* logits, uint32_t* ids,
                         float* w, float* mass) {
  int rc = layer_ready(L, T, false);
  if (rc) return rc;
  if (!x || !logits) return fail(L->ctx, OSM_EINVAL, "route: null input/logits");
  if (int e = router_x_ok(L, x)) return e;
  osm_context* ctx = L->ctx;
  DeviceGuard dg(ctx->device);
  osm::RouterArgs a = router_args(L, x, T);
  a.force_exact = 1;  // every token on the reference's arithmetic: its logits are the reference's
  a.ids_out = ids;
  a.weights_out = w;
  a.mass_out = mass;
  a.logits_out = logits;
  a.do_group = 0;
  a.xfrag = nullptr;
  a.sgate_w = nullptr;
  a.pick_ptr = nullptr;
  launch_router_pair(ctx, a);
  return check_launch(ctx, "router");
}

int osm_moe_forward(osm_layer* L, const float* x, uint32_t T, float* out, uint32_t* ids, float* w,
                    float* mass, float* sgate, const float* residual, uint32_t flags) {
  int rc = layer_ready(L, T, true);
  if (rc) return rc;
  osm_context* ctx = L->ctx;
  if (!x || !out) return fail(ctx, OSM_EINVAL, "forward: null input/output");
  if (int e = router_x_ok(L, x)) return e;
  if ((flags & OSM_ADD_RESIDUAL) && !residual) return fail(ctx, OSM_EINVAL, "forward: residual missing");
  DeviceGuard dg(ctx->device);
  osm::RouterArgs a = router_args(L, x, T);
  a.force_exact = (flags & OSM_ROUTE_EXACT) ? 1 : 0;
  a.ids_out = ids;
  a.weights_out = w;
  a.mass_out = mass;
  a.sgate_out = sgate;
  if (flags & OSM_PREFILL_BF16) {
    osm::PfArgs pa;
    size_t psm = 0;
    if (!prefill_path(L, &pa, &psm)) return fail(ctx, OSM_EINVAL, "prefill: layer shapes not supported");
    // Checked (the default outside stream capture): this call's status bits
    // go to a word of their own, read back when the call ends; if a value
    // left the fp16 range the call runs again on the fp32 path.
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    OSM_CUDA(ctx, cudaStreamIsCapturing(ctx->stream, &cap));
    const bool checked = !(flags & OSM_PREFILL_NO_CHECK) && cap == cudaStreamCaptureStatusNone;
    Scratch& sc = ctx->sc;
    uint32_t* const main_status = sc.status;
    if (checked) {
      OSM_CUDA(ctx, cudaMemsetAsync(sc.range_status, 0, 4, ctx->stream));
      sc.status = sc.range_status;
    }
    a.status = sc.status;
    a.do_group = 1;
    a.xfrag = nullptr;
    a.xbf = sc.xbf;
    a.chunk_pairs = chunk_pairs_for(L, T, true);
    ctx->cur_x = x;
    launch_router_pair(ctx, a);
    rc = check_launch(ctx, "router");
    if (!rc) rc = run_prefill(L, T, out, (flags & OSM_ADD_RESIDUAL) ? residual : nullptr, pa, psm);
    sc.status = main_status;
    if (rc || !checked) return rc;
    uint32_t st = 0;
    OSM_CUDA(ctx, cudaMemcpyAsync(&st, sc.range_status, 4, cudaMemcpyDeviceToHost, ctx->stream));
    OSM_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    if (!(st & osm::kStatusF16Range)) {
      ctx->pending_status |= st;
      return OSM_OK;
    }
    ctx->pending_status |= (st & ~osm::kStatusF16Range) | osm::kStatusPrefillFallback;
    flags &= ~(OSM_PREFILL_BF16 | OSM_PREFILL_NO_CHECK);
    return osm_moe_forward(L, x, T, out, ids, w, mass, sgate, residual, flags);
  }
  // one or two tokens: the expert kernels read the picks directly (no
  // grouping, no tensor-core fragments)
  osm::GemvArgs g;
  osm::GemvLaunch gl;
  const bool dec = gemv_path(L, T, &g, &gl);
  a.do_group = dec ? 0 : 1;
  osm::GrpArgs ga;
  size_t sgu = 0, sdn = 0;
  if (dec || grouped_path(L, &ga, &sgu, &sdn)) a.xfrag = nullptr;  // only the older kernels read it
  a.chunk_pairs = chunk_pairs_for(L, T, false);
  ctx->cur_x = x;
  launch_router_pair(ctx, a);
  rc = check_launch(ctx, "router");
  if (rc) return rc;
  return run_experts(L, T, out, (flags & OSM_ADD_RESIDUAL) ? residual : nullptr);
}

}  // extern "C"

namespace {

// The expert half of a call whose routing is in device memory: `ids`/`w`
// are copied into the context's routing scratch first, or, with both null,
// are already there (a cached call routed into it).
int experts_impl(osm_layer* L, const float* x, uint32_t T, const uint32_t* ids, const float* w,
                 float* out, float* sgate, const float* residual, uint32_t flags) {
  osm_context* ctx = L->ctx;
  DeviceGuard dg(ctx->device);
  Scratch& s = ctx->sc;
  int rc = OSM_OK;
  const size_t nk = (size_t)T * L->g.k;
  if (ids) {
    OSM_CUDA(ctx, cudaMemcpyAsync(s.ids, ids, nk * 4, cudaMemcpyDeviceToDevice, ctx->stream));
    OSM_CUDA(ctx, cudaMemcpyAsync(s.weights, w, nk * 4, cudaMemcpyDeviceToDevice, ctx->stream));
  }
  osm::RouterArgs a = router_args(L, x, T);
  a.skip_route = 1;
  a.sgate_out = sgate;
  a.do_group = 1;
  osm::PfArgs pa;
  size_t psm = 0;
  const bool prefill = (flags & OSM_PREFILL_BF16) != 0;
  const bool f16 = (flags & OSM_INPUT_F16) != 0;
  const bool f16_out = (flags & OSM_OUTPUT_F16) != 0;
  if (f16 && (!prefill || L->shared_slot))
    return fail(ctx, OSM_EINVAL, "experts: fp16 rows need OSM_PREFILL_BF16 and no shared expert");
  if (f16_out && !prefill) return fail(ctx, OSM_EINVAL, "experts: fp16 output needs OSM_PREFILL_BF16");
  if (prefill) {
    if (!prefill_path(L, &pa, &psm)) return fail(ctx, OSM_EINVAL, "prefill: layer shapes not supported");
    a.xfrag = nullptr;
    a.xbf = s.xbf;
  }
  a.chunk_pairs = chunk_pairs_for(L, T, prefill);
  ctx->cur_x = x;
  if (f16) {
    // the rows are the GEMM's operand already: only the grouping runs first
    Prof p(ctx, kKRouterSelect);
    a.pick_ptr = nullptr;  // the grouped entries carry the slot bases
    osm::launch_group(a, ctx->stream, &ctx->launches);
  } else {
    launch_router_pair(ctx, a);
  }
  rc = check_launch(ctx, "expert grouping");
  if (rc) return rc;
  if (prefill) {
    const float* res = (flags & OSM_ADD_RESIDUAL) ? residual : nullptr;
    if (f16) {
      osm::PfArgs pf = pa;
      pf.xb = reinterpret_cast<const uint16_t*>(x);
      return run_prefill(L, T, out, res, pf, psm, true, f16_out);
    }
    return run_prefill(L, T, out, res, pa, psm, false, f16_out);
  }
  return run_experts(L, T, out, (flags & OSM_ADD_RESIDUAL) ? residual : nullptr);
}

// The owner's experts over every slot of its EP block (fp16 rows, one pick
// each, empty slots skipped by the grouping): gate/up and down on the
// tensor-core prefill path, leaving each pair's fp16 result row in the
// context's pair rows for ep_return_kernel.
int ep_experts(osm_ep* ep, osm_layer* X) {
  osm_context* ctx = ep->ctx;
  Scratch& s = ctx->sc;
  const osm::EpLayout& Ly = ep->lay;
  const uint32_t R = (uint32_t)((Ly.world + 1) * Ly.cap);
  const size_t nk = R;
  OSM_CUDA(ctx, cudaMemcpyAsync(s.ids, ep->own + Ly.o_ids, nk * 4, cudaMemcpyDeviceToDevice, ctx->stream));
  OSM_CUDA(ctx, cudaMemcpyAsync(s.weights, ep->own + Ly.o_wts, nk * 4, cudaMemcpyDeviceToDevice,
                                ctx->stream));
  const float* rows = reinterpret_cast<const float*>(ep->own + Ly.o_rows);
  osm::RouterArgs a = router_args(X, rows, R);
  a.skip_route = 1;
  a.sgate_out = nullptr;
  a.do_group = 1;
  a.pick_ptr = nullptr;
  osm::PfArgs pa;
  size_t psm = 0;
  if (!prefill_path(X, &pa, &psm)) return fail(ctx, OSM_EINVAL, "expert parallel: expert shapes not supported");
  a.xfrag = nullptr;
  a.xbf = s.xbf;
  a.chunk_pairs = chunk_pairs_for(X, R, true);
  ctx->cur_x = rows;
  {
    Prof p(ctx, kKRouterSelect);
    osm::launch_group(a, ctx->stream, &ctx->launches);
  }
  int rc = check_launch(ctx, "expert parallel grouping");
  if (!rc) {
    osm::PfArgs pf = pa;
    pf.xb = reinterpret_cast<const uint16_t*>(rows);
    rc = run_prefill(X, R, nullptr, nullptr, pf, psm, true, true, false);
  }
  return rc;
}

osm::EpArgs ep_args(const osm_ep* ep) {
  osm::EpArgs e{};
  e.lay = ep->lay;
  for (int i = 0; i < osm::kEpMaxWorld; ++i) e.peer[i] = ep->peer[i];
  e.send_cnt = reinterpret_cast<int*>(ep->own + ep->lay.o_cnt);
  e.status = ep->ctx->sc.status;
  return e;
}

}  // namespace

extern "C" {

int osm_moe_experts(osm_layer* L, const float* x, uint32_t T, const uint32_t* ids, const float* w,
                    float* out, float* sgate, const float* residual, uint32_t flags) {
  int rc = layer_ready(L, T, true);
  if (rc) return rc;
  osm_context* ctx = L->ctx;
  if (!x || !out || !ids || !w) return fail(ctx, OSM_EINVAL, "experts: null argument");
  if ((flags & OSM_ADD_RESIDUAL) && !residual) return fail(ctx, OSM_EINVAL, "experts: residual missing");
  return experts_impl(L, x, T, ids, w, out, sgate, residual, flags);
}

int osm_moe_forward_cached(osm_layer* L, osm_cache* cache, uint32_t layer_id, const float* x,
                           uint32_t T, float* out, uint32_t* ids, float* w, float* sgate,
                           const float* residual, uint32_t flags) {
  int rc = layer_ready(L, T, true);
  if (rc) return rc;
  osm_context* ctx = L->ctx;
  if (!cache || !x || !out) return fail(ctx, OSM_EINVAL, "cached forward: null argument");
  if (int e = router_x_ok(L, x)) return e;
  if ((flags & OSM_ADD_RESIDUAL) && !residual)
    return fail(ctx, OSM_EINVAL, "cached forward: residual missing");
  if (flags & OSM_INPUT_F16) return fail(ctx, OSM_EINVAL, "cached forward: fp32 rows only");
  if (cache->slab != L->slab) return fail(ctx, OSM_EINVAL, "cached forward: the layer is not on the cache's slab");
  auto lit = cache->layers.find(layer_id);
  if (lit == cache->layers.end() || lit->second != L)
    return fail(ctx, OSM_EINVAL, "cached forward: layer_id is not bound to this layer");
  DeviceGuard dg(ctx->device);
  Scratch& s = ctx->sc;
  const size_t nk = (size_t)T * L->g.k;
  if (ctx->picks_cap < nk) {
    if (ctx->picks_host) cudaFreeHost(ctx->picks_host);
    ctx->picks_host = nullptr;
    ctx->picks_dev = nullptr;
    ctx->picks_cap = 0;
    OSM_CUDA(ctx, cudaHostAlloc(&ctx->picks_host, nk * 4, cudaHostAllocMapped));
    OSM_CUDA(ctx, cudaHostGetDevicePointer(reinterpret_cast<void**>(&ctx->picks_dev), ctx->picks_host, 0));
    ctx->picks_cap = nk;
  }
  if (!ctx->picks_ev) OSM_CUDA(ctx, cudaEventCreateWithFlags(&ctx->picks_ev, cudaEventDisableTiming));
  const bool prefill = (flags & OSM_PREFILL_BF16) != 0;
  osm::PfArgs pa;
  size_t psm = 0;
  osm::GemvArgs g;
  osm::GemvLaunch gl;
  osm::GrpArgs ga;
  size_t sgu = 0, sdn = 0;
  bool dec = false;
  osm::RouterArgs a = router_args(L, x, T);
  if (prefill) {
    if (!prefill_path(L, &pa, &psm)) return fail(ctx, OSM_EINVAL, "prefill: layer shapes not supported");
    a.xfrag = nullptr;
    a.xbf = s.xbf;
  } else {
    dec = gemv_path(L, T, &g, &gl);
    if (dec || grouped_path(L, &ga, &sgu, &sdn)) a.xfrag = nullptr;  // only the older kernels read it
  }
  a.chunk_pairs = chunk_pairs_for(L, T, prefill);
  // 1. route, with the shared gate and the activation operands; the picks go
  //    straight to mapped host memory
  a.force_exact = (flags & OSM_ROUTE_EXACT) ? 1 : 0;
  a.ids_out = ctx->picks_dev;
  a.weights_out = w;
  a.sgate_out = sgate;
  a.do_group = 0;
  a.pick_ptr = nullptr;
  ctx->cur_x = x;
  launch_router_pair(ctx, a);
  rc = check_launch(ctx, "router");
  if (rc) return rc;
  OSM_CUDA(ctx, cudaEventRecord(ctx->picks_ev, ctx->stream));
  if (ids) OSM_CUDA(ctx, cudaMemcpyAsync(ids, s.ids, nk * 4, cudaMemcpyDeviceToDevice, ctx->stream));
  const float* res = (flags & OSM_ADD_RESIDUAL) ? residual : nullptr;
  // 1b. early experts (one or two tokens): queued before the host has the
  //     picks, resolving them through the slot table as it stands, so the
  //     device runs them right behind the router while the host waits and
  //     acquires.  Their non-resident picks go to a side status word.
  const bool early = !prefill && dec && (flags & OSM_CACHED_EARLY);
  if (early) {
    OSM_CUDA(ctx, cudaMemsetAsync(s.early_status, 0, 4, ctx->stream));
    rc = run_experts(L, T, out, res, true, s.early_status);
    if (rc) return rc;
  }
  // 2. the host needs the picks to make them resident
  OSM_CUDA(ctx, cudaEventSynchronize(ctx->picks_ev));
  // 3. one acquire over the picks in token-major pick order (the order of
  //    the reference's expert_cache.get calls, routed_moe.cpp:319-327)
  const uint64_t misses0 = cache->misses;
  rc = osm_cache_acquire(cache, layer_id, ctx->picks_host, (uint32_t)nk);
  if (rc) return fail(ctx, rc, std::string("cached forward: ") + cache->err);
  // every pick was resident before the acquire: the early run used the
  // right slots and its output stands
  if (early && cache->misses == misses0) return OSM_OK;
  // 4. bind the picks to their slots and group them, then the experts; one
  //    token on the decode kernels needs neither (they read the slot table).
  //    After an early run with a miss this runs the experts again, behind
  //    the acquire's copies and slot-table writes.
  if (!prefill && dec) return run_experts(L, T, out, res, true);
  a.skip_route = 1;
  a.ids_out = nullptr;
  a.weights_out = nullptr;
  a.sgate_out = nullptr;
  a.pick_ptr = s.pick_ptr;
  a.do_group = 1;
  {
    Prof p(ctx, kKRouterSelect);
    osm::launch_group(a, ctx->stream, &ctx->launches);
  }
  rc = check_launch(ctx, "pick binding");
  if (rc) return rc;
  if (prefill) return run_prefill(L, T, out, res, pa, psm);
  return run_experts(L, T, out, res);
}

int osm_ep_create(osm_context* ctx, uint32_t world, uint32_t rank, uint32_t tokens_per_rank,
                  uint32_t k, uint32_t hidden, uint32_t experts_per_rank, int has_shared,
                  osm_ep** out) {
  if (!ctx || !out) return OSM_EINVAL;
  *out = nullptr;
  if (world == 0 || world > (uint32_t)osm::kEpMaxWorld || rank >= world)
    return fail(ctx, OSM_EINVAL, "expert parallel: 1 to 8 ranks, rank < world");
  if (tokens_per_rank == 0 || k == 0 || experts_per_rank == 0)
    return fail(ctx, OSM_EINVAL, "expert parallel: tokens, k and experts must be non-zero");
  if (hidden == 0 || hidden % 256 || hidden > 8192)
    return fail(ctx, OSM_EINVAL, "expert parallel: hidden must be a multiple of 256 up to 8192");
  if ((uint64_t)(world + 1) * tokens_per_rank * k > (1u << 24))
    return fail(ctx, OSM_EINVAL, "expert parallel: receive regions too large");
  DeviceGuard dg(ctx->device);
  auto* ep = new (std::nothrow) osm_ep();
  if (!ep) return OSM_ENOMEM;
  ep->ctx = ctx;
  ep->lay = osm::ep_layout((int)world, (int)rank, (int)tokens_per_rank, (int)k, (int)hidden,
                           (int)experts_per_rank, has_shared ? 1 : 0);
  if (cudaMalloc(&ep->own, ep->lay.total) != cudaSuccess ||
      cudaMalloc(&ep->sgate, (size_t)tokens_per_rank * 4) != cudaSuccess) {
    if (ep->own) cudaFree(ep->own);
    delete ep;
    return fail(ctx, OSM_ENOMEM, "expert parallel: device allocation failed");
  }
  // back rows, flags and counters zero; every receive slot empty
  cudaMemset(ep->own + ep->lay.o_back, 0, ep->lay.total - ep->lay.o_back);
  cudaMemset(ep->sgate, 0, (size_t)tokens_per_rank * 4);
  osm::launch_ep_clear_ids(ep->lay, ep->own, nullptr, nullptr);
  if (cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(ep->own);
    cudaFree(ep->sgate);
    delete ep;
    return fail(ctx, OSM_ECUDA, "expert parallel: block initialisation failed");
  }
  ep->peer[rank] = ep->own;
  *out = ep;
  return OSM_OK;
}

int osm_ep_ipc_handle(const osm_ep* ep, unsigned char* handle) {
  if (!ep || !handle) return OSM_EINVAL;
  DeviceGuard dg(ep->ctx->device);
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ep->own) != cudaSuccess)
    return fail(ep->ctx, OSM_ECUDA, "expert parallel: cudaIpcGetMemHandle failed");
  static_assert(sizeof(h) == OSM_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  return OSM_OK;
}

int osm_ep_open_peers(osm_ep* ep, const unsigned char* handles) {
  if (!ep || !handles) return OSM_EINVAL;
  if (ep->opened) return fail(ep->ctx, OSM_EINVAL, "expert parallel: peers already open");
  DeviceGuard dg(ep->ctx->device);
  for (int r = 0; r < ep->lay.world; ++r) {
    if (r == ep->lay.rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles + (size_t)r * OSM_IPC_HANDLE_BYTES, sizeof(h));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (q != ep->lay.rank && ep->peer[q]) {
          cudaIpcCloseMemHandle(ep->peer[q]);
          ep->peer[q] = nullptr;
        }
      return fail(ep->ctx, OSM_ECUDA, "expert parallel: cudaIpcOpenMemHandle failed");
    }
    ep->peer[r] = static_cast<unsigned char*>(p);
  }
  ep->opened = true;
  return OSM_OK;
}

int osm_ep_set_timeout(osm_ep* ep, uint32_t timeout_ms) {
  if (!ep || timeout_ms == 0) return OSM_EINVAL;
  ep->timeout_ns = (uint64_t)timeout_ms * 1000000ull;
  return OSM_OK;
}

int osm_ep_destroy(osm_ep* ep) {
  if (!ep) return OSM_EINVAL;
  DeviceGuard dg(ep->ctx->device);
  cudaStreamSynchronize(ep->ctx->stream);
  for (int r = 0; r < ep->lay.world; ++r)
    if (r != ep->lay.rank && ep->peer[r]) cudaIpcCloseMemHandle(ep->peer[r]);
  cudaFree(ep->own);
  cudaFree(ep->sgate);
  delete ep;
  return OSM_OK;
}

int osm_ep_forward(osm_ep* ep, osm_layer* router, osm_layer* experts, const float* x, uint32_t T,
                   float* out, uint32_t* ids_out, float* weights_out, uint32_t flags) {
  if (!ep || !router || !experts) return OSM_EINVAL;
  osm_context* ctx = ep->ctx;
  const osm::EpLayout& Ly = ep->lay;
  if (router->ctx != ctx || experts->ctx != ctx)
    return fail(ctx, OSM_EINVAL, "expert parallel: layers of another context");
  if (!ep->opened && Ly.world > 1) return fail(ctx, OSM_EINVAL, "expert parallel: peers not open");
  if (!x || !out || T == 0 || T > (uint32_t)Ly.T_r)
    return fail(ctx, OSM_EINVAL, "expert parallel: null input/output or tokens > tokens_per_rank");
  if (router->g.k != Ly.k || router->g.H != Ly.H || router->g.E != Ly.e_local * Ly.world)
    return fail(ctx, OSM_EINVAL, "expert parallel: router geometry differs from the block's");
  if (Ly.shared && !router->shared_slot)
    return fail(ctx, OSM_EINVAL, "expert parallel: the router layer needs the shared expert's gate");
  if (experts->g.k != 1 || experts->g.H != Ly.H || experts->g.E < Ly.e_local + Ly.shared ||
      experts->shared_slot)
    return fail(ctx, OSM_EINVAL, "expert parallel: experts layer must be k = 1 over the local experts");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(ctx, OSM_EINVAL, "expert parallel: x and out must be 16-byte aligned");
  const uint32_t R = (uint32_t)((Ly.world + 1) * Ly.cap);
  // scratch for both calls first, so that nothing moves within this one
  int rc = layer_ready(experts, R, true);
  if (!rc) rc = layer_ready(router, T, false);
  if (rc) return rc;
  DeviceGuard dg(ctx->device);
  Scratch& s = ctx->sc;
  // 1. route, with the shared gate
  osm::RouterArgs a = router_args(router, x, T);
  a.force_exact = (flags & OSM_ROUTE_EXACT) ? 1 : 0;
  a.ids_out = ids_out;
  a.weights_out = weights_out;
  a.do_group = 0;
  a.xfrag = nullptr;
  a.xbf = nullptr;
  a.pick_ptr = nullptr;
  a.sgate_w = Ly.shared ? router->sgate_w : nullptr;
  a.sgate_out = ep->sgate;
  launch_router_pair(ctx, a);
  rc = check_launch(ctx, "expert parallel router");
  if (rc) return rc;
  // 2. every pick's row into its owner's region, the shared rows locally
  osm::EpArgs e = ep_args(ep);
  e.x = x;
  e.ids = s.ids;
  e.w = s.weights;
  e.sgate = ep->sgate;
  e.T = (int)T;
  OSM_CUDA(ctx, cudaMemsetAsync(e.send_cnt, 0, (size_t)Ly.world * 4, ctx->stream));
  {
    Prof p(ctx, kKOther);
    osm::launch_ep_dispatch(e, ctx->num_sms, ctx->stream, &ctx->launches);
    osm::launch_ep_barrier(e, ++ep->epoch, ep->timeout_ns, ctx->stream, &ctx->launches);
  }
  rc = check_launch(ctx, "expert parallel dispatch");
  if (rc) return rc;
  // 3. this rank's experts over every region
  rc = ep_experts(ep, experts);
  if (rc) return rc;
  // 4. the weighted rows back to their sources, 5. the combine
  {
    Prof p(ctx, kKCombine);
    osm::launch_ep_return(e, reinterpret_cast<const uint16_t*>(s.partial), s.tp_pos, ctx->num_sms,
                          ctx->stream, &ctx->launches);
    osm::launch_ep_barrier(e, ++ep->epoch, ep->timeout_ns, ctx->stream, &ctx->launches);
    osm::launch_ep_combine(e, out, ctx->stream, &ctx->launches);
  }
  return check_launch(ctx, "expert parallel combine");
}

int osm_gather_sum_rows(osm_context* ctx, const void* rows_f16, const int64_t* pos, uint32_t tokens,
                        uint32_t k, uint32_t hidden, const void* extra_f16, float* out) {
  if (!ctx) return OSM_EINVAL;
  if (tokens == 0) return OSM_OK;
  if (!out || (k && (!rows_f16 || !pos))) return fail(ctx, OSM_EINVAL, "gather_sum_rows: null argument");
  if (hidden == 0 || hidden % 8) return fail(ctx, OSM_EINVAL, "gather_sum_rows: hidden must be a multiple of 8");
  if ((reinterpret_cast<uintptr_t>(rows_f16) | reinterpret_cast<uintptr_t>(extra_f16) |
       reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(ctx, OSM_EINVAL, "gather_sum_rows: rows, extra and out must be 16-byte aligned");
  DeviceGuard dg(ctx->device);
  osm::launch_gather_sum_rows(static_cast<const uint16_t*>(rows_f16), pos,
                              static_cast<const uint16_t*>(extra_f16), out, (int)tokens, (int)hidden,
                              (int)k, ctx->stream, &ctx->launches);
  return check_launch(ctx, "gather_sum_rows");
}

int osm_moe_sublayer_forward(osm_layer* L, const float* residual, uint32_t T, float* out,
                             float* normalized, uint32_t* ids, float* w, float* mass,
                             float* sgate, uint32_t flags) {
  int rc = layer_ready(L, T, true);
  if (rc) return rc;
  osm_context* ctx = L->ctx;
  if (!residual || !out) return fail(ctx, OSM_EINVAL, "sublayer: null input/output");
  DeviceGuard dg(ctx->device);
  float* nrm = normalized ? normalized : ctx->sc.normalized;
  {
    Prof p(ctx, kKRmsNorm);
    osm::launch_rmsnorm(residual, nrm, (int)T, L->g.H, L->norm_w, L->norm_eps,
                        (flags & OSM_RMSNORM_EXACT) != 0, ctx->stream, &ctx->launches);
  }
  rc = check_launch(ctx, "sublayer rmsnorm");
  if (rc) return rc;
  return osm_moe_forward(L, nrm, T, out, ids, w, mass, sgate, residual, flags | OSM_ADD_RESIDUAL);
}

}  // extern "C"

namespace {

// A plan's copy of x in and of out back: by the SMs (osm::launch_host_copy)
// when the host buffer is pinned memory mapped into the GPU (unified
// addressing), both sides are 16-byte aligned and the copy is at most 2 MiB;
// a copy-engine node otherwise.  Measured on a B200 (decode plans of 1-256
// tokens at hidden 2048, 8 KiB - 2 MiB each way): the SM copies take 12 us
// off a one-token call (48.6 -> 36.3 us) and 6 us off a 256-token call; a
// copy-engine node waits on its hand-off before and after the transfer.
// Larger copies keep the copy engine (not measured with SM copies).
constexpr size_t kPlanSmCopyInMax = (size_t)2 << 20;
constexpr size_t kPlanSmCopyOutMax = (size_t)2 << 20;

// The device address of a mapped pinned host buffer, or null.
void* mapped_host(const void* host) {
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, host) != cudaSuccess) {
    cudaGetLastError();  // not a CUDA pointer: a copy-engine node will report it
    return nullptr;
  }
  return at.type == cudaMemoryTypeHost ? at.devicePointer : nullptr;
}

bool sm_copy_ok(const void* dev, const void* host_dev, size_t bytes, size_t limit) {
  return host_dev != nullptr && bytes <= limit && bytes % 16 == 0 &&
         reinterpret_cast<uintptr_t>(dev) % 16 == 0 && reinterpret_cast<uintptr_t>(host_dev) % 16 == 0;
}

}  // namespace

extern "C" {

int osm_plan_create(osm_layer* L, uint32_t T, const float* x, float* out, uint32_t* ids,
                    float* w, const float* x_host, float* out_host, uint32_t flags,
                    osm_plan** res) {
  if (!res) return OSM_EINVAL;
  *res = nullptr;
  int rc = layer_ready(L, T, true);
  if (rc) return rc;
  osm_context* ctx = L->ctx;
  if (!x || !out) return fail(ctx, OSM_EINVAL, "plan: null input/output");
  if (ctx->stream == nullptr || ctx->stream == cudaStreamLegacy || ctx->stream == cudaStreamPerThread)
    return fail(ctx, OSM_EINVAL, "plan: capture needs a non-default stream");
  DeviceGuard dg(ctx->device);
  auto* plan = new (std::nothrow) osm_plan();
  if (!plan) return OSM_ENOMEM;
  plan->layer = L;
  const size_t bytes = (size_t)T * L->g.H * sizeof(float);
  // (pointer queries before the capture begins)
  void* const xh_dev = x_host ? mapped_host(x_host) : nullptr;
  void* const oh_dev = out_host ? mapped_host(out_host) : nullptr;
  const bool sm_in = x_host && sm_copy_ok(x, xh_dev, bytes, kPlanSmCopyInMax);
  const bool sm_out = out_host && sm_copy_ok(out, oh_dev, bytes, kPlanSmCopyOutMax);
  const bool prof = (flags & OSM_PLAN_PROFILE) != 0;
  const bool saved_prof = ctx->prof_on;
  std::vector<ProfRec> saved_recs;
  saved_recs.swap(ctx->recs);
  ctx->prof_on = prof;
  const uint64_t l0 = ctx->launches;
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) {
    ctx->prof_on = saved_prof;
    ctx->recs.swap(saved_recs);
    delete plan;
    return cuda_fail(ctx, e, "plan: begin capture");
  }
  cudaError_t ce = cudaSuccess;
  if (sm_in)
    ce = osm::launch_host_copy(const_cast<float*>(x), xh_dev, bytes, false, ctx->num_sms, ctx->stream,
                               &ctx->launches);
  else if (x_host)
    ce = cudaMemcpyAsync(const_cast<float*>(x), x_host, bytes, cudaMemcpyHostToDevice, ctx->stream);
  const uint32_t fw = flags & (OSM_ROUTE_EXACT | OSM_RMSNORM_EXACT);
  if (ce != cudaSuccess)
    rc = cuda_fail(ctx, ce, "plan: input copy");
  else if (flags & OSM_PLAN_SUBLAYER)
    rc = osm_moe_sublayer_forward(L, x, T, out, nullptr, ids, w, nullptr, nullptr, fw);
  else
    rc = osm_moe_forward(L, x, T, out, ids, w, nullptr, nullptr, nullptr, fw);
  if (rc == OSM_OK) {
    if (sm_out)
      ce = osm::launch_host_copy(oh_dev, out, bytes, true, ctx->num_sms, ctx->stream, &ctx->launches);
    else if (out_host)
      ce = cudaMemcpyAsync(out_host, out, bytes, cudaMemcpyDeviceToHost, ctx->stream);
    if (ce != cudaSuccess) rc = cuda_fail(ctx, ce, "plan: output copy");
  }
  e = cudaStreamEndCapture(ctx->stream, &graph);
  plan->kernels = (uint32_t)(ctx->launches - l0);
  ctx->launches = l0;
  plan->recs.swap(ctx->recs);
  ctx->recs.swap(saved_recs);
  ctx->prof_on = saved_prof;
  if (rc == OSM_OK && e != cudaSuccess) rc = cuda_fail(ctx, e, "plan: end capture");
  if (rc == OSM_OK) {
    e = cudaGraphInstantiate(&plan->exec, graph, 0);
    if (e != cudaSuccess) rc = cuda_fail(ctx, e, "plan: instantiate");
  }
  if (rc == OSM_OK) ++ctx->plans_alive;
  if (graph) cudaGraphDestroy(graph);
  if (rc != OSM_OK) {
    osm_plan_destroy(plan);
    return rc;
  }
  *res = plan;
  return OSM_OK;
}

int osm_plan_launch(osm_plan* plan) {
  if (!plan || !plan->exec) return OSM_EINVAL;
  osm_context* ctx = plan->layer->ctx;
  DeviceGuard dg(ctx->device);
  OSM_CUDA(ctx, cudaGraphLaunch(plan->exec, ctx->stream));
  ctx->launches += plan->kernels;
  return OSM_OK;
}

int osm_plan_destroy(osm_plan* plan) {
  if (!plan) return OSM_EINVAL;
  osm_context* ctx = plan->layer->ctx;
  DeviceGuard dg(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (plan->exec) {
    cudaGraphExecDestroy(plan->exec);
    --ctx->plans_alive;
  }
  for (const ProfRec& r : plan->recs) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  delete plan;
  return OSM_OK;
}

int osm_plan_profile_read(osm_plan* plan, double* ms, uint64_t* launches) {
  if (!plan) return OSM_EINVAL;
  osm_context* ctx = plan->layer->ctx;
  DeviceGuard dg(ctx->device);
  OSM_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  for (const ProfRec& r : plan->recs) {
    float t = 0.0f;
    if (cudaEventElapsedTime(&t, r.a, r.b) == cudaSuccess && r.kind >= 0 &&
        r.kind < OSM_KERNEL_KINDS) {
      if (ms) ms[r.kind] += t;
      if (launches) launches[r.kind] += 1;
    } else {
      cudaGetLastError();
    }
  }
  return OSM_OK;
}

uint32_t osm_plan_kernels(const osm_plan* plan) { return plan ? plan->kernels : 0; }

int osm_gen_normal(osm_context* ctx, uint64_t seed, uint64_t tensor, float sigma, float* out,
                   size_t n, size_t first) {
  if (!ctx || (n && !out)) return OSM_EINVAL;
  DeviceGuard dg(ctx->device);
  if (n == 0) return OSM_OK;
  osm::launch_gen_normal(seed, tensor, sigma, out, n, first, ctx->stream, &ctx->launches);
  return check_launch(ctx, "gen normal");
}

int osm_gen_expert_slots(osm_slab* s, uint64_t seed, uint64_t tensor_base, float sigma,
                         uint32_t first, uint32_t count) {
  if (!s) return OSM_EINVAL;
  osm_context* ctx = s->ctx;
  if ((uint64_t)first + count > s->slots) return fail(ctx, OSM_EINVAL, "gen: slot range");
  DeviceGuard dg(ctx->device);
  const osm_expert_layout& L = s->layout;
  for (uint32_t i = 0; i < count; ++i) {
    uint8_t* b = s->base + (size_t)(first + i) * L.stride;
    const uint64_t t = tensor_base + 3ull * i;
    osm::launch_gen_quant(seed, t + 0, sigma, (int)L.inter, (int)L.hidden,
                          reinterpret_cast<uint32_t*>(b + L.gate_w), reinterpret_cast<uint16_t*>(b + L.gate_s),
                          reinterpret_cast<uint16_t*>(b + L.gate_b), ctx->stream, &ctx->launches);
    osm::launch_gen_quant(seed, t + 1, sigma, (int)L.inter, (int)L.hidden,
                          reinterpret_cast<uint32_t*>(b + L.up_w), reinterpret_cast<uint16_t*>(b + L.up_s),
                          reinterpret_cast<uint16_t*>(b + L.up_b), ctx->stream, &ctx->launches);
    osm::launch_gen_quant(seed, t + 2, sigma, (int)L.hidden, (int)L.inter,
                          reinterpret_cast<uint32_t*>(b + L.down_w), reinterpret_cast<uint16_t*>(b + L.down_s),
                          reinterpret_cast<uint16_t*>(b + L.down_b), ctx->stream, &ctx->launches);
  }
  return check_launch(ctx, "gen expert slots");
}

}  // extern "C"


// ----------------------------------------------------------------------------
// HBM expert cache: the residency policy of VulkanResidentExpertCache
// (src/backend/vulkan_resident_expert_cache.cpp:40-200) over slab slots.
// ----------------------------------------------------------------------------

namespace {

uint64_t cache_key(uint32_t layer, uint32_t expert) { return ((uint64_t)layer << 32) | expert; }

int cache_fail(osm_cache* c, int code, const char* msg) {
  c->err = msg;
  return code;
}

osm_cache::Rank cache_rank(uint64_t key, const osm_cache::Node& n) {
  return {n.frequency, n.last_use, key};
}

// Records expert -> slot in the layer's host mirror now and queues the device
// table write for the end of the acquire.
void cache_bind_slot(osm_cache* c, osm_layer* L, uint32_t expert, int32_t slot) {
  L->slot_host[expert] = slot;
  // without a slab every entry of a bound layer stays -1 on the device
  if (c->slab) c->table_writes.emplace_back(L->slot_of + expert, slot);
}

// One get() of the reference: a hit refreshes frequency and recency; a miss
// asks the host source for the expert first (the reference fetches from its
// host cache and uploads before it evicts anything,
// vulkan_resident_expert_cache.cpp:101-140), so a failing source leaves the
// residency as it was (only the use count and the miss are recorded, as
// there); then it evicts the entry with the smallest (frequency, last use,
// key) until the newcomer fits and queues the expert's copy into a free slot.
// Entries touched in the current acquire (epoch) are not evicted.  The victim
// is the first unprotected entry of an ordered index, the same entry as the
// reference's linear scan (vulkan_resident_expert_cache.cpp:58-69) picks.
int cache_get(osm_cache* c, uint32_t layer, uint32_t expert, int32_t* slot_out) {
  ++c->tick;
  const uint64_t key = cache_key(layer, expert);
  const uint64_t freq = ++c->frequency_history[key];
  auto it = c->entries.find(key);
  if (it != c->entries.end()) {
    ++c->hits;
    c->order.erase(cache_rank(key, it->second));
    it->second.frequency = freq;
    it->second.last_use = c->tick;
    it->second.epoch = c->epoch;
    c->order.insert(cache_rank(key, it->second));
    if (slot_out) *slot_out = it->second.slot;
    return OSM_OK;
  }
  ++c->misses;
  const void* src = nullptr;
  if (c->slab || c->source) {
    if (!c->source || c->source(c->user, layer, expert, &src) != 0 || (c->slab && !src))
      return cache_fail(c, OSM_ERUNTIME, "cache: the host source could not provide the expert");
  }
  if (c->accounted > c->budget) return cache_fail(c, OSM_EINVAL, "cache: one expert exceeds the budget");
  while (!c->entries.empty() &&
         (c->resident_bytes + c->accounted > c->budget || (c->slab && c->free_slots.empty()))) {
    auto victim = c->entries.end();
    auto rank = c->order.begin();
    for (; rank != c->order.end(); ++rank) {
      auto e = c->entries.find(std::get<2>(*rank));
      if (e->second.epoch != c->epoch) {
        victim = e;
        break;
      }
    }
    if (victim == c->entries.end())
      return cache_fail(c, OSM_ENOMEM, "cache: the experts of one call do not fit in the budget");
    const uint32_t vl = (uint32_t)(victim->first >> 32), ve = (uint32_t)(victim->first & 0xFFFFFFFFu);
    auto lit = c->layers.find(vl);
    if (lit != c->layers.end()) cache_bind_slot(c, lit->second, ve, -1);
    if (victim->second.slot >= 0) c->free_slots.push_back(victim->second.slot);
    c->resident_bytes -= c->accounted;
    c->order.erase(rank);
    c->entries.erase(victim);
    ++c->evictions;
  }
  int32_t slot = -1;
  if (c->slab) {
    if (c->free_slots.empty()) return cache_fail(c, OSM_ENOMEM, "cache: no free slot");
    slot = c->free_slots.back();
    c->free_slots.pop_back();
    c->fills.emplace_back((uint32_t)slot, src);
    auto lit = c->layers.find(layer);
    if (lit != c->layers.end()) cache_bind_slot(c, lit->second, expert, slot);
  }
  osm_cache::Node n;
  n.slot = slot;
  n.frequency = freq;
  n.last_use = c->tick;
  n.epoch = c->epoch;
  c->entries.emplace(key, n);
  c->order.insert(cache_rank(key, n));
  c->resident_bytes += c->accounted;
  ++c->loads;
  if (slot_out) *slot_out = slot;
  return OSM_OK;
}

// Issues the acquire's queued copies and slot-table writes.  The copies run
// back to back on the slab's side stream after the work already queued on
// the compute stream (which may still read the slots being overwritten); the
// compute stream waits once for all of them, then the table writes follow in
// its order, ahead of the caller's next kernel.
int cache_flush(osm_cache* c) {
  int rc = OSM_OK;
  if (c->slab && !c->fills.empty()) {
    osm_slab* s = c->slab;
    osm_context* ctx = s->ctx;
    DeviceGuard dg(ctx->device);
    cudaError_t e = cudaSuccess;
    std::pair<cudaEvent_t, cudaEvent_t> tw{nullptr, nullptr};
    if (c->time_copies) {
      if (!c->spare_events.empty()) {
        tw = c->spare_events.back();
        c->spare_events.pop_back();
      } else {
        e = cudaEventCreate(&tw.first);
        if (e == cudaSuccess) e = cudaEventCreate(&tw.second);
      }
      if (e == cudaSuccess) e = cudaEventRecord(tw.first, ctx->stream);
    }
    if (e == cudaSuccess) e = cudaEventRecord(s->ev, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s->side, s->ev, 0);
    for (size_t i = 0; e == cudaSuccess && i < c->fills.size(); ++i) {
      e = cudaMemcpyAsync(s->base + (size_t)c->fills[i].first * s->layout.stride, c->fills[i].second,
                          s->layout.stride, cudaMemcpyHostToDevice, s->side);
      if (e == cudaSuccess) s->h2d_bytes += s->layout.stride;
    }
    if (e == cudaSuccess) e = cudaEventRecord(s->ev, s->side);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx->stream, s->ev, 0);
    if (e == cudaSuccess && tw.second) {
      e = cudaEventRecord(tw.second, ctx->stream);
      if (e == cudaSuccess) c->copy_waits.push_back(tw);
    }
    if (e != cudaSuccess) {
      if (tw.first) cudaEventDestroy(tw.first);
      if (tw.second) cudaEventDestroy(tw.second);
      rc = cache_fail(c, OSM_ECUDA, cudaGetErrorString(e));
    }
  }
  c->fills.clear();
  if (rc == OSM_OK && !c->table_writes.empty()) {
    osm_context* ctx = c->slab->ctx;
    DeviceGuard dg(ctx->device);
    osm::SlotUpdates u{};
    for (size_t i = 0; i < c->table_writes.size(); i += osm::SlotUpdates::kMax) {
      u.n = (int)std::min<size_t>(osm::SlotUpdates::kMax, c->table_writes.size() - i);
      for (int j = 0; j < u.n; ++j) {
        u.ptr[j] = c->table_writes[i + j].first;
        u.val[j] = c->table_writes[i + j].second;
      }
      osm::launch_slot_updates(u, ctx->stream, &ctx->launches);
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) rc = cache_fail(c, OSM_ECUDA, cudaGetErrorString(e));
  }
  c->table_writes.clear();
  return rc;
}

}  // namespace

extern "C" {

int osm_cache_create(osm_slab* slab, uint64_t budget_bytes, uint64_t accounted_bytes,
                     osm_cache_source_fn source, void* user, osm_cache** out) {
  if (!out) return OSM_EINVAL;
  *out = nullptr;
  if (budget_bytes == 0) return OSM_EINVAL;
  if (accounted_bytes == 0) {
    if (!slab) return OSM_EINVAL;
    accounted_bytes = slab->layout.stride;
  }
  if (slab && !source) return OSM_EINVAL;
  osm_cache* c = new (std::nothrow) osm_cache;
  if (!c) return OSM_ENOMEM;
  c->slab = slab;
  if (slab) c->device = slab->ctx->device;
  c->budget = budget_bytes;
  c->accounted = accounted_bytes;
  c->source = source;
  c->user = user;
  if (slab)
    for (uint32_t s = slab->slots; s > 0; --s) c->free_slots.push_back((int32_t)(s - 1));
  *out = c;
  return OSM_OK;
}

int osm_cache_destroy(osm_cache* c) {
  if (!c) return OSM_EINVAL;
  if (!c->copy_waits.empty() || !c->spare_events.empty()) {
    // events still pending are released by the driver once they complete
    DeviceGuard dg(c->device);
    for (auto& p : c->copy_waits) {
      cudaEventDestroy(p.first);
      cudaEventDestroy(p.second);
    }
    for (auto& p : c->spare_events) {
      cudaEventDestroy(p.first);
      cudaEventDestroy(p.second);
    }
  }
  delete c;
  return OSM_OK;
}

int osm_cache_time_copies(osm_cache* c, int enable) {
  if (!c) return OSM_EINVAL;
  if (enable && !c->slab) return cache_fail(c, OSM_EINVAL, "cache: copy timing needs a slab");
  c->time_copies = enable != 0;
  return OSM_OK;
}

int osm_cache_exposed_read(osm_cache* c, double* ms, uint64_t* waits) {
  if (!c || !ms) return OSM_EINVAL;
  double sum = 0.0;
  const uint64_t n = c->copy_waits.size();
  if (n) {
    DeviceGuard dg(c->slab->ctx->device);
    const cudaError_t e = cudaEventSynchronize(c->copy_waits.back().second);
    if (e != cudaSuccess) return cache_fail(c, OSM_ECUDA, cudaGetErrorString(e));
    for (auto& p : c->copy_waits) {
      float t = 0.f;
      if (cudaEventElapsedTime(&t, p.first, p.second) == cudaSuccess) sum += t;
      c->spare_events.push_back(p);
    }
    c->copy_waits.clear();
  }
  *ms = sum;
  if (waits) *waits = n;
  return OSM_OK;
}

const char* osm_cache_last_error(const osm_cache* c) { return c ? c->err.c_str() : "null cache"; }

int osm_cache_bind_layer(osm_cache* c, uint32_t layer_id, osm_layer* layer) {
  if (!c || !layer) return OSM_EINVAL;
  if (c->slab && layer->slab != c->slab)
    return cache_fail(c, OSM_EINVAL, "cache: the layer must be bound to the cache's slab");
  c->layers[layer_id] = layer;
  // experts of this layer already resident keep their slots; all others are
  // marked not resident
  for (uint32_t e = 0; e < (uint32_t)layer->g.E; ++e) {
    auto it = c->entries.find(cache_key(layer_id, e));
    layer->slot_host[e] = it != c->entries.end() ? it->second.slot : -1;
  }
  osm_context* ctx = layer->ctx;
  DeviceGuard dg(ctx->device);
  // pageable source: staged before the call returns
  const cudaError_t e = cudaMemcpyAsync(layer->slot_of, layer->slot_host.data(), layer->g.E * 4,
                                        cudaMemcpyHostToDevice, ctx->stream);
  if (e != cudaSuccess) return cache_fail(c, OSM_ECUDA, "cache: binding the layer failed");
  return OSM_OK;
}

int osm_cache_get(osm_cache* c, uint32_t layer_id, uint32_t expert, int32_t* slot_out) {
  if (!c) return OSM_EINVAL;
  ++c->epoch;
  const int rc = cache_get(c, layer_id, expert, slot_out);
  const int rc2 = cache_flush(c);
  return rc ? rc : rc2;
}

int osm_cache_acquire(osm_cache* c, uint32_t layer_id, const uint32_t* experts, uint32_t n) {
  if (!c || (n && !experts)) return OSM_EINVAL;
  // a call whose distinct experts cannot all be resident at once is refused
  // before anything changes (ExpertCache::fetch, src/cache/expert_cache.cpp:
  // 108-111, rejects an oversized request the same way)
  {
    std::vector<uint32_t> distinct(experts, experts + n);
    std::sort(distinct.begin(), distinct.end());
    const uint64_t d = (uint64_t)(std::unique(distinct.begin(), distinct.end()) - distinct.begin());
    if (d * c->accounted > c->budget || (c->slab && d > c->slab->slots))
      return cache_fail(c, OSM_ENOMEM, "cache: the experts of one call do not fit in the budget");
  }
  ++c->epoch;
  int rc = OSM_OK;
  for (uint32_t i = 0; i < n && rc == OSM_OK; ++i) rc = cache_get(c, layer_id, experts[i], nullptr);
  // what this call already changed is issued even when a later pick failed
  const int rc2 = cache_flush(c);
  return rc ? rc : rc2;
}

int osm_cache_contains(const osm_cache* c, uint32_t layer_id, uint32_t expert) {
  if (!c) return 0;
  return c->entries.count(cache_key(layer_id, expert)) ? 1 : 0;
}

int osm_cache_stats(const osm_cache* c, osm_cache_counts* out) {
  if (!c || !out) return OSM_EINVAL;
  out->hits = c->hits;
  out->misses = c->misses;
  out->loads = c->loads;
  out->evictions = c->evictions;
  out->resident_entries = c->entries.size();
  out->resident_bytes = c->resident_bytes;
  out->budget_bytes = c->budget;
  return OSM_OK;
}

}  // extern "C"

// ----------------------------------------------------------------------------
// Allocation-free single-expert forward.
//
// Some hosts cannot call cudaMalloc on the path that runs an expert: an
// inference server whose memory is owned by a pool allocator that forbids
// driver allocations after warm-up, a process that only borrows a device
// context it did not create, or code that runs where an allocation would
// synchronise the device.  osm_expert_forward_noalloc serves them: it takes
// no context and keeps its intermediates (activation and SwiGLU fragments,
// the one-expert work list) in a file-scope device array of fixed size that
// every GPU loading this library holds until the process exits.
// ----------------------------------------------------------------------------
namespace {

constexpr uint32_t kNaMaxTokens = 16;
constexpr uint32_t kNaMaxHidden = 2048;
constexpr uint32_t kNaMaxInter = 768;
constexpr size_t na_up(size_t v) { return (v + 255) / 256 * 256; }
// pairs of the one-expert work list: one per token (two per token reserved,
// as the context scratch sizes it)
constexpr size_t kNaPairs = 2 * kNaMaxTokens;
constexpr size_t kNaMaxTg = kNaPairs / osm::kTokGroup + 3;
constexpr size_t kNaXfrag = 0;
constexpr size_t kNaXsum = kNaXfrag + na_up(kNaMaxTokens * (kNaMaxHidden / 8) * 32);
constexpr size_t kNaNact = kNaXsum + na_up(kNaMaxTokens * (kNaMaxHidden / 8) * 4);
constexpr size_t kNaAct = kNaNact + na_up(4);
constexpr size_t kNaNtg = kNaAct + na_up(2 * sizeof(osm::ActEntry));
constexpr size_t kNaTge = kNaNtg + na_up(4);
constexpr size_t kNaTgb = kNaTge + na_up(kNaMaxTg * 4);
constexpr size_t kNaPtok = kNaTgb + na_up(kNaMaxTg * 4);
constexpr size_t kNaPpick = kNaPtok + na_up(kNaPairs * 4);
constexpr size_t kNaOrow = kNaPpick + na_up(kNaPairs * 4);
constexpr size_t kNaHfrag = kNaOrow + na_up(kNaPairs * 4);
constexpr size_t kNaHsum = kNaHfrag + na_up(kNaPairs * (kNaMaxInter / 8) * 32);
constexpr size_t kNaBytes = kNaHsum + na_up(kNaPairs * (kNaMaxInter / 8) * 4);

// The scratch of every call on this GPU.  Host code must not pass this name
// to a kernel: on the host it is a stand-in, not the device address.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNaBytes];

struct NaDevice {
  bool ready = false;
  uint8_t* base = nullptr;  // device address of g_noalloc_scratch
  int grid_cap = 0;
};
constexpr int kNaMaxDevices = 64;
std::mutex g_na_mu;
NaDevice g_na[kNaMaxDevices];

// Set-up of the current device, once: the scratch's device address and the
// kernel attributes the context creation would otherwise set.
int na_device(int dev, NaDevice** out) {
  if (dev < 0 || dev >= kNaMaxDevices) return OSM_EINVAL;
  std::lock_guard<std::mutex> lock(g_na_mu);
  NaDevice& d = g_na[dev];
  if (!d.ready) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
      return OSM_ECUDA;
    int sms = 0, optin = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
      return OSM_ECUDA;
    // the result of each call is checked directly: an error the caller left
    // pending is neither taken for this call's nor cleared
    if (osm::init_expert_attributes(optin > 64 * 1024 ? optin - 16 * 1024 : 48 * 1024) !=
        cudaSuccess)
      return OSM_ECUDA;
    d.base = static_cast<uint8_t*>(p);
    d.grid_cap = (sms > 0 ? sms : 148) * 4;
    d.ready = true;
  }
  *out = &d;
  return OSM_OK;
}

}  // namespace

extern "C" int osm_expert_forward_noalloc(const void* slot_dev, const osm_expert_layout* layout,
                                          const float* x_dev, uint32_t tokens, float* out_dev,
                                          void* cuda_stream) {
  if (!slot_dev || !x_dev || !out_dev || !layout_ok(layout)) return OSM_EINVAL;
  if (tokens == 0 || tokens > kNaMaxTokens || layout->hidden > kNaMaxHidden ||
      layout->inter > kNaMaxInter)
    return OSM_EINVAL;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return OSM_ECUDA;
  NaDevice* d = nullptr;
  int rc = na_device(dev, &d);
  if (rc) return rc;
  const cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
  const osm_expert_layout& L = *layout;
  uint8_t* b = d->base;
  auto at = [&](size_t off) { return b + off; };
  // every intermediate of the call starts cleared: the previous call's
  // contents stay in the array
  if (cudaMemsetAsync(b, 0, kNaBytes, st) != cudaSuccess) return OSM_ECUDA;
  uint4* xfrag = reinterpret_cast<uint4*>(at(kNaXfrag));
  float* xfsum = reinterpret_cast<float*>(at(kNaXsum));
  int* n_active = reinterpret_cast<int*>(at(kNaNact));
  osm::ActEntry* act = reinterpret_cast<osm::ActEntry*>(at(kNaAct));
  int* n_tg = reinterpret_cast<int*>(at(kNaNtg));
  int* tg_expert = reinterpret_cast<int*>(at(kNaTge));
  int* tg_begin = reinterpret_cast<int*>(at(kNaTgb));
  int* pair_tok = reinterpret_cast<int*>(at(kNaPtok));
  int* pair_pick = reinterpret_cast<int*>(at(kNaPpick));
  int* out_row = reinterpret_cast<int*>(at(kNaOrow));
  uint4* hfrag = reinterpret_cast<uint4*>(at(kNaHfrag));
  float* hfsum = reinterpret_cast<float*>(at(kNaHsum));
  if (osm::launch_frag_prep(x_dev, (int)tokens, (int)L.hidden, xfrag, xfsum, st, nullptr) !=
          cudaSuccess ||
      osm::launch_setup_single((int)tokens, static_cast<const uint8_t*>(slot_dev), n_active, act,
                               n_tg, tg_expert, tg_begin, pair_tok, pair_pick, out_row, st,
                               nullptr) != cudaSuccess)
    return OSM_ECUDA;
  osm::ProjArgs gu{};
  fill_sections(gu.sec, L, L, true);
  gu.n_tg = n_tg;
  gu.act = act;
  gu.tg_expert = tg_expert;
  gu.tg_begin = tg_begin;
  gu.pair_tok = pair_tok;
  gu.frag_stride = (int)L.hidden / 8;
  gu.frag = xfrag;
  gu.fsum8 = xfsum;
  gu.hfrag = hfrag;
  gu.hfsum8 = hfsum;
  gu.hK = (int)L.inter;
  const int ntg = (int)((tokens + osm::kTokGroup - 1) / osm::kTokGroup);
  const int tch = (int)std::min<uint32_t>(tokens, 8);
  if (osm::launch_proj(gu, osm::ProjKind::kGateUp, (int)L.inter, ntg, d->grid_cap, tch, st,
                       nullptr) != cudaSuccess)
    return OSM_ECUDA;
  osm::ProjArgs dn = gu;
  fill_sections(dn.sec, L, L, false);
  dn.frag_by_pair = 1;
  dn.frag_stride = (int)L.inter / 8;
  dn.frag = hfrag;
  dn.fsum8 = hfsum;
  dn.out = out_dev;
  dn.out_row = out_row;
  dn.pair_pick = pair_pick;
  dn.kp1 = 1;
  dn.ostride = (int)L.hidden;
  if (osm::launch_proj(dn, L.inter <= 512 ? osm::ProjKind::kDown : osm::ProjKind::kDown12,
                       (int)L.hidden, ntg, d->grid_cap, tch, st, nullptr) != cudaSuccess)
    return OSM_ECUDA;
  return OSM_OK;
}
