// osm_kernels.cuh -- launch interfaces of the sm_100a kernels (osm_kernels.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace osm {

// Router weight layout in HBM.  Row e is padded to Hp = roundup(H, 256) and
// split into 32 contiguous lane chunks of c = Hp/32 elements; lane l's chunk
// is stored as nvec = c/8 vectors of 8 bf16, vector m of every lane adjacent:
//   element (e, h), l = h / c, o = h % c  ->  ((e*nvec + o/8)*32 + l)*8 + o%8
// so the 32 lanes of a warp read 512 contiguous bytes per step while each lane
// walks its own contiguous chunk (needed by the error bound of the router).
// One active expert of a call (written by the grouping step): 32 bytes.
struct ActEntry {
  const uint8_t* ptr;  // slot base (null: not resident)
  int off;             // first pair position of its tokens
  int cnt;             // tokens routed to it
  int kind;            // 0 routed layout, 1 shared layout
  int tg0;             // first token group (groups of kTokGroup tokens)
  int pad0, pad1;
};
constexpr int kTokGroup = 32;  // tokens per projection work item

struct RouterGeom {
  int H, Hp, c, nvec, E, k;
  int f32w;                 // router stored as fp32 (else bf16)
  int q8;                   // router stored as MLX-affine 8-bit (one byte per weight; scale and
                            // bias per 64-group in RouterArgs::qmeta); the weight is
                            // fl(fl(scale * q) + bias), as cpu::dequantize_affine_rows
};

struct RouterArgs {
  RouterGeom g;
  const uint4* wp;          // permuted router rows (bf16 or fp32)
  const void* wx;           // router in 16 KB tiles (router_tile_kernel)
  const uint32_t* qmeta;    // q8: [E][H / 64] bf16 scale | bf16 bias << 16
  const float* bias;        // [E] or null
  const float* x;           // [B][H]
  int B;
  int norm;                 // norm_topk_prob
  int force_exact;
  int skip_route;           // routing given (osm_moe_experts): gate, fragments, grouping only
  float* logits;            // scratch [B][E]
  float* bounds;            // scratch [B][E]
  uint32_t* ids;            // scratch [B][k]
  float* weights;           // scratch [B][k]
  float* mass;              // scratch [B]
  uint32_t* ids_out;        // optional user copies
  float* weights_out;
  float* mass_out;
  float* logits_out;        // optional [B][E]: the full exact path's logits (W x + bias)
  // shared expert scalar gate
  const float* sgate_w;     // [H] or null
  float* sgate;             // scratch [B]
  float* sgate_out;         // optional
  // fragments of x for the expert kernels
  uint4* xfrag;             // [B][H/8][2]
  uint16_t* xbf;            // optional [B][H] fp16 copy of x (prefill)
  int chunk_pairs;          // pairs per chunk of the chunk list (8, or 128 for prefill)
  float* xfsum8;            // [B][H/8]
  // grouping (done by the last block)
  int do_group;
  const int* slot_of;       // [E]
  const uint8_t* slab;
  uint64_t slab_stride;
  const uint8_t* shared_slot;  // null without shared expert
  unsigned int* ticket;
  int* counts;              // [E+1] first pair position of each expert (deferred scatter)
  int* n_active;
  ActEntry* act;            // [E+1]
  int* n_tg;                // token groups of the call
  int* tg_expert;           // token group -> active entry
  int* tg_begin;            // token group -> first token within the entry
  int* pair_tok;            // [B*(k+1)]
  int* pair_pick;
  int* tp_pos;              // (token, pick) -> pair position
  int* n_ch;                // 8-token chunks of the call (null: not built)
  int2* chunks;             // chunk -> {active entry, first token within it}
  int* cursor;              // [E+1] pairs placed so far per expert (deferred scatter)
  int defer_scatter;        // pairs placed by scatter_pairs_kernel, not the last select block
  uint32_t* status;
  unsigned long long* exact_count;
  // slot base of each pick (null: bad id or not resident), written for the
  // one-token expert kernels; null pointer: not wanted
  const uint8_t** pick_ptr;  // [B][k]
};

// Allow up to max_smem bytes of dynamic shared memory for every kernel that
// uses it (once per device, before any launch or capture).
void init_router_attributes(int max_smem);
cudaError_t init_expert_attributes(int max_smem);

void launch_router_logits(const RouterArgs& a, cudaStream_t s, uint64_t* launches);
void launch_router_select(const RouterArgs& a, cudaStream_t s, uint64_t* launches);

// Grouping alone (expert list from a routing already in scratch).
void launch_group(const RouterArgs& a, cudaStream_t s, uint64_t* launches);

// Fragments of activations for the projection kernel: per 8-element chunk
// c of row r, two uint4 (hi, lo) holding bf16x2 pairs (x0,x4) (x1,x5)
// (x2,x6) (x3,x7), and the fp32 sequential sum of the 8 values.
cudaError_t launch_frag_prep(const float* x, int rows, int K, uint4* frag, float* fsum8,
                      cudaStream_t s, uint64_t* launches);

// Section offsets of one projection (weight, scales, biases) for the two
// slot layouts (0 routed, 1 shared); for a raw projection, base pointers are
// null and offsets carry the addresses.
struct ProjSections {
  uint64_t w[2], s[2], b[2];     // first (gate / single) projection
  uint64_t w2[2], s2[2], b2[2];  // paired projection (up)
  int rows[2];                   // output rows per layout
  int K[2];                      // input dim per layout
};

struct ProjArgs {
  ProjSections sec;
  int shared_first;              // active entry 0 is the shared expert (layout 1)
  const uint8_t* shared_ptr;     // its slot, readable before the routing exists
  const int* n_tg;
  const ActEntry* act;
  const int* tg_expert;
  const int* tg_begin;
  const int* pair_tok;           // pair -> input fragment row (for paired)
  int frag_by_pair;              // 1: input row = pair position
  int raw;                       // 1: sections are absolute addresses
  int frag_stride;               // chunks (of 8) per fragment row
  const uint4* frag;             // [row][frag_stride][2]
  const float* fsum8;            // [row][frag_stride]
  // paired outputs
  uint4* hfrag;                  // [pair][Kd/8][2]
  float* hfsum8;                 // [pair][Kd/8]
  int hK;                        // row length of hfrag (intermediate, max)
  // single outputs
  float* out;                    // [out_row][ostride]
  const int* out_row;            // pair -> output row, or null (row = pair_tok)
  const int* pair_pick;          // pair -> pick (used with kp1)
  int kp1;                       // k+1 (out row = tok*kp1 + pick) when out_row null
  int ostride;
};

enum class ProjKind { kGateUp, kDown, kDown12, kSingle };
// grid_cap: resident CTAs the device holds (SMs x CTAs per SM); the grid is
// persistent and strides over (active expert, tile) items.
// max_tg: upper bound of the call's token groups (grid sizing only).
cudaError_t launch_proj(const ProjArgs& a, ProjKind kind, int max_rows, int max_tg, int grid_cap,
                 int max_tokens_chunk, cudaStream_t s, uint64_t* launches);

// The 1-2 token path (osm_gemv.cu).
struct GemvArgs {
  ProjSections gu, dn;           // gate/up and down sections, both layouts
  const float* x;                // [B][H]
  int B, H, Imax, k, has_shared;
  const int* n_active;
  const ActEntry* act;
  const int* pair_tok;
  const int* tp_pos;
  // direct mode (one token, no grouping step): entry p < k is pick p of the
  // routing, entry k the shared expert
  int direct;
  const uint32_t* ids;           // [k]
  // [k] slot base of each pick (router-written); null: resolved here from
  // ids through slot_of (a token whose mass the router set to 0 has none)
  const uint8_t* const* pick_ptr;
  const float* mass;             // [1] with pick_ptr null
  int E;                         // experts (ids >= E are rejected)
  const int* slot_of;            // [E]
  const uint8_t* slab;
  uint64_t slab_stride;
  const uint8_t* shared_ptr;
  uint32_t* status;
  float* h;                      // [pairs][Imax] SwiGLU output
  const float* weights;          // [B][k]
  const float* sgate;            // [B]
  const float* residual;         // [B][H] or null
  float* out;                    // [B][H]
  // set by gemv_configure
  int total_max;                 // (gate, up) row pairs of all possible entries
  int per_cta;                   // pairs per gate/up CTA
  int nbuf;                      // 16-row tiles per gate/up CTA
  int cs_gu, cs_dn;              // scale-row copy granules (bytes)
  int rpc;                       // output rows per down CTA
  int max_entries;               // active entries the down CTA has room for
};
struct GemvLaunch {
  int grid_gu, grid_dn;
  size_t smem_gu, smem_dn;
};
constexpr int kChunkPad = 36;    // floats per staged 32-value chunk (bank spread)
constexpr int kDecWarps = 16;    // warps per CTA of the decode kernels
void init_gemv_attributes(int max_smem);
// false: the shapes or alignment do not suit the decode kernels (the caller
// uses the tensor-core path instead)
bool gemv_configure(GemvArgs& a, int max_active, int num_sms, int max_smem, GemvLaunch* out);
void launch_gemv_gateup(const GemvArgs& a, const GemvLaunch& l, cudaStream_t s,
                        uint64_t* launches);
void launch_gemv_down(const GemvArgs& a, const GemvLaunch& l, cudaStream_t s, uint64_t* launches);

// Three or more tokens (osm_gemv.cu): grouped projections over 8-token
// chunks of each active expert; down writes partial [token][k+1][H] rows for
// the combine kernel.
struct GrpArgs {
  ProjSections gu, dn;
  const float* x;                // [T][H]
  int H, Imax, kp1, has_shared;
  uint64_t slab_stride;
  const int* n_ch;               // chunks of up to 8 pairs of one active entry
  const int2* chunks;            // {active entry, first pair within it}
  const ActEntry* act;
  const int* pair_tok;
  const int* pair_pick;
  float* h;                      // [pairs][Imax] SwiGLU output
  float* partial;                // [T][kp1][H]
  uint32_t* status;
  // set by grouped_configure
  int rb_gu, ob_dn, st_gu, st_dn;  // row blocks; ring stages
};
void init_grouped_attributes(int max_smem);
bool grouped_configure(GrpArgs& a, int max_smem, size_t* smem_gu, size_t* smem_dn);
void launch_grouped_gateup(const GrpArgs& a, int grid, size_t smem, cudaStream_t s,
                           uint64_t* launches);
void launch_grouped_down(const GrpArgs& a, int grid, size_t smem, cudaStream_t s,
                         uint64_t* launches);

struct CombineArgs {
  const float* partial;          // [B][k+1][H]
  const float* weights;          // [B][k]
  const float* sgate;            // [B] or null (no shared expert)
  const float* residual;         // [B][H] or null
  float* out;                    // [B][H]
  int B, H, k;
};
void launch_combine(const CombineArgs& a, cudaStream_t s, uint64_t* launches);

// ---- prefill: 16-bit tensor-core (tcgen05, fp16 operands) grouped GEMM over 128-pair chunks ----
struct PfArgs {
  ProjSections gu, dn;
  const uint16_t* xb;            // [T][H] fp16 activations (gate/up B operand)
  uint16_t* hb;                  // [pairs][Imax] fp16 SwiGLU output (down B operand)
  uint16_t* pb;                  // [pairs][H] fp16 expert outputs
  const int* n_ch;               // chunks of up to 128 pairs of one active entry
  const int2* chunks;
  const ActEntry* act;
  const int* pair_tok;
  int H, Imax, nmt_gu, nmt_dn;   // M tiles (128 rows) per chunk
  uint32_t* status;
};
bool prefill_configure(const PfArgs& a, int has_shared, int max_smem, size_t* smem);
void init_prefill_attributes(int max_smem);
void launch_prefill_gateup(const PfArgs& a, int grid, size_t smem, cudaStream_t s, uint64_t* launches);
void launch_prefill_down(const PfArgs& a, int grid, size_t smem, cudaStream_t s, uint64_t* launches);
// out[t] = sum over p < k in order of rows[pos[t k + p]] (fp16 rows, fp32 sums),
// then + extra[t] (fp16, may be null); H % 8 == 0, all pointers 16-byte aligned
void launch_gather_sum_rows(const uint16_t* rows, const int64_t* pos, const uint16_t* extra,
                            float* out, int T, int H, int k, cudaStream_t s, uint64_t* launches);
// out[b] = sum over picks of w * pb[tp_pos[b][j]] in pick order, then sgate * the
// shared row, then the residual; H % 8 == 0, out and residual 16-byte aligned;
// f16_out: out holds fp16 rows
void launch_combine_bf16(const uint16_t* pb, const int* tp_pos, const float* weights,
                         const float* sgate, const float* residual, void* out, bool f16_out,
                         unsigned int* status, int B, int H, int k, cudaStream_t s,
                         uint64_t* launches);

// ---- tensor-core grouped experts with warp specialisation (osm_tc.cu) ----
// Items are (chunk of pairs sharing an expert, 128 weight rows).  PRECISE:
// bf16 operand planes (A = s q as hi + lo, exact; B = activations as hi +
// mid), three passes plus a bias step, outputs within 1e-4 of the fp32 path;
// chunks of kTcChunkPrecise pairs.  FAST: fp16 operands (A = fp16(s q + b)),
// one pass, outputs within 2e-3; chunks of kTcChunkFast pairs.
constexpr int kTcChunkPrecise = 32;
constexpr int kTcChunkFast = 96;
// TMA tensor maps (CUtensorMap, 128 bytes each) over the Q4 weight sections:
// [kind: 0 routed experts in the slab, 1 the shared expert][0 gate, 1 up,
// 2 down]; each map is words x rows x slots with an 8-word x 128-row box.
struct alignas(64) TcMaps {
  unsigned char m[2][3][128];
};
struct TcArgs {
  ProjSections gu, dn;
  const float* x;                // PRECISE gate/up: [T][H] fp32 rows
  const uint16_t* xb;            // FAST gate/up: [T][H] fp16 rows
  float* h;                      // PRECISE: [pairs][Imax] SwiGLU output
  uint16_t* hb;                  // FAST: [pairs][Imax] fp16 SwiGLU output
  float* partial;                // PRECISE down: [T][kp1][H] expert rows
  uint16_t* pb;                  // FAST down: [pairs][H] fp16 expert rows
  const int* n_ch;
  const int2* chunks;            // {active entry, first pair within it}
  const ActEntry* act;
  const int* pair_tok;
  const int* pair_pick;
  const uint8_t* slab;           // routed slots: slot = (ptr - slab) / slab_stride
  uint64_t slab_stride;
  int H, Imax, kp1, nmt_gu, nmt_dn;
  uint32_t* status;
};
// Encodes the three maps of one expert source: sections at base + off[s] with
// rows[s] rows of words[s] u32 words, `slots` slots slot_stride bytes apart.
bool tc_encode_maps(unsigned char (*dst)[128], const uint8_t* base, const uint64_t off[3],
                    const int rows[3], const int words[3], int slots, uint64_t slot_stride);
void init_tc_attributes(int max_smem);
bool tc_configure(TcArgs& a, int has_shared, int max_smem);
cudaError_t launch_tc_gateup(const TcArgs& a, const TcMaps& maps, bool precise, int grid,
                             cudaStream_t s, uint64_t* launches);
cudaError_t launch_tc_down(const TcArgs& a, const TcMaps& maps, bool precise, int grid,
                           cudaStream_t s, uint64_t* launches);

// 2-D tensor map over `rows` rows of row_bytes bytes (uint8, 128-byte
// swizzle, box 128 bytes x box_rows rows): the digit planes of osm_tcd.cu.
bool tc_encode_u8_rows(unsigned char* dst, const uint8_t* base, uint64_t rows, uint64_t row_bytes,
                       int box_rows);

// ---- tensor-core grouped experts on int8 digit planes (osm_tcd.cu) ----
// fp32 calls of 3+ tokens: Q4 nibbles (exact int8) against block-floating-
// point activations split into three int8 digit planes, tcgen05.mma
// kind::i8 with one s32 accumulator per 64-wide K group, the group scales
// applied in fp32 by the epilogue; outputs within 1e-4 of the fp32 path.
// Items are (chunk of <= kDgChunk pairs of one active entry, 128 rows).
constexpr int kDgChunk = 16;
struct DgArgs {
  TcArgs t;                      // sections, grouping, h / partial outputs, status
  const float2* xq;              // [pairs][H/64] {s 2^-14, group sum} of each pair's x row
  const float2* hq;              // [pairs][Imax/64] the same for h
};
// Tensor maps: the Q4 sections (TcMaps) and the digit planes of x per pair
// ([pairs * 3][H] bytes) and of h ([pairs * 3][Imax]), box 128 bytes x
// 16 (i + 1) rows for map i (an item of n pairs reads 16 ceil(3 n / 16) rows).
struct alignas(64) DgMaps {
  TcMaps q;
  unsigned char xd[3][128];
  unsigned char hd[3][128];
};
// Digit planes of `rows` fp32 rows of K inputs (K a multiple of 64): row r
// reads src row rowmap[r] (clamped to [0, nsrc)) or r, row stride ld floats;
// dst[r][d][K] int8, per 8 inputs the digits of the even positions then the
// odd ones (the A operand's nibble order); q[r][K/64] = {s 2^-14, sum of the
// group's inputs}.
void launch_digits(const float* src, const int* rowmap, int nsrc, int rows, int K, int ld,
                   uint8_t* dst, float2* q, cudaStream_t s, uint64_t* launches);
void init_dg_attributes(int max_smem);
bool dg_fits(int max_smem);
cudaError_t launch_dg_gateup(const DgArgs& a, const DgMaps& maps, int grid, cudaStream_t s,
                             uint64_t* launches);
cudaError_t launch_dg_down(const DgArgs& a, const DgMaps& maps, int grid, cudaStream_t s,
                           uint64_t* launches);

// ---- expert parallelism over peer memory (osm_ep.cu) ----
constexpr uint32_t kEpEmpty = 0xFFFFFFFFu;  // id of an empty receive slot
constexpr int kEpMaxWorld = 8;

// One rank's EP block; the same layout on every rank.  Offsets in bytes.
struct EpLayout {
  int world, rank, T_r, k, H, e_local, shared, cap;
  size_t o_rows, o_ids, o_wts, o_src, o_back, o_flags, o_cnt, total;
};
struct EpArgs {
  EpLayout lay;
  unsigned char* peer[kEpMaxWorld];  // every rank's block as this GPU addresses it
  const float* x;                    // [T][H] this rank's tokens
  const uint32_t* ids;               // [T][k] global expert ids
  const float* w;                    // [T][k] routing weights
  const float* sgate;                // [T] shared-expert gate (when lay.shared)
  int* send_cnt;                     // [world] slots claimed in each owner's region
  uint32_t* status;
  int T;
};
EpLayout ep_layout(int world, int rank, int T_r, int k, int H, int e_local, int shared);
void launch_ep_clear_ids(const EpLayout& L, unsigned char* own, cudaStream_t s, uint64_t* launches);
void launch_ep_dispatch(const EpArgs& a, int num_sms, cudaStream_t s, uint64_t* launches);
void launch_ep_barrier(const EpArgs& a, uint32_t epoch, uint64_t timeout_ns, cudaStream_t s,
                       uint64_t* launches);
void launch_ep_return(const EpArgs& a, const uint16_t* pb, const int* tp_pos, int num_sms,
                      cudaStream_t s, uint64_t* launches);
void launch_ep_combine(const EpArgs& a, float* out, cudaStream_t s, uint64_t* launches);

// Test hook: polls of the first bounded copy wait in each kernel file.
cudaError_t set_first_wait_polls_gemv(uint32_t polls);
cudaError_t set_first_wait_polls_prefill(uint32_t polls);
cudaError_t set_first_wait_polls_router(uint32_t polls);

void launch_rmsnorm(const float* in, float* out, int rows, int dim, const float* w,
                    float eps, bool exact, cudaStream_t s, uint64_t* launches);
// sc/bi: bf16 bits, or fp32 when f32_meta
void launch_dequant(const uint32_t* packed, const void* sc, const void* bi, bool f32_meta,
                    int rows, int K, int group, float* out, cudaStream_t s, uint64_t* launches);
void launch_gemv_any(const uint32_t* packed, const void* sc, const void* bi, bool f32_meta,
                     int rows, int K, int group, const float* x, int tokens, float* y,
                     cudaStream_t s, uint64_t* launches);
void launch_swiglu(const float* g, const float* u, float* out, size_t n, cudaStream_t s,
                   uint64_t* launches);
void launch_waccum(const float* src, float w, float* acc, size_t n, cudaStream_t s,
                   uint64_t* launches);
void launch_gen_normal(uint64_t seed, uint64_t tensor, float sigma, float* out, size_t n,
                       size_t first, cudaStream_t s, uint64_t* launches);
// Quantise `rows` x `cols` N(0, sigma) values of (seed, tensor) with the
// reference quantiser into packed/scales/biases (bf16) destinations.
void launch_gen_quant(uint64_t seed, uint64_t tensor, float sigma, int rows, int cols,
                      uint32_t* packed, uint16_t* sc, uint16_t* bi, cudaStream_t s,
                      uint64_t* launches);
// Permute fp32 [E][H] router rows (bf16-representable) into the router layout.
// Router tiles: 128 experts x 128 bytes of one row each (64 bf16 or 32 fp32
// weights), tiles of one 128-expert block consecutive along h; in each
// 128-byte row the 16-byte chunk c sits at c ^ (row & 7).
size_t router_tile_bytes(const RouterGeom& g);
// q8 router: layouts of the byte matrix q [E][H] (the packed words of an
// 8-bit MLX-affine module are its bytes in element order)
void launch_router_pack_q8(const uint8_t* q, const RouterGeom& g, void* wp, cudaStream_t s,
                           uint64_t* launches);
void launch_router_tile_q8(const uint8_t* q, const RouterGeom& g, void* wx, cudaStream_t s,
                           uint64_t* launches);
void launch_router_tile(const float* w, const RouterGeom& g, void* wx, cudaStream_t s,
                        uint64_t* launches);
void launch_router_pack(const float* w, const RouterGeom& g, void* wp, cudaStream_t s,
                        uint64_t* launches);
// Slot-table writes (expert -> slab slot) passed by value, so that the host
// batches a cache acquire's table changes into one launch without a staging
// buffer that a later acquire could overwrite before the copy ran.
struct SlotUpdates {
  static constexpr int kMax = 48;
  int n;
  int32_t val[kMax];
  int32_t* ptr[kMax];
};
void launch_slot_updates(const SlotUpdates& u, cudaStream_t s, uint64_t* launches);
// bytes (a multiple of 16, both pointers 16-byte aligned) between device
// memory and mapped pinned host memory, copied by the SMs.
cudaError_t launch_host_copy(void* dst, const void* src, size_t bytes, bool after_pdl, int num_sms,
                             cudaStream_t s, uint64_t* launches);
cudaError_t launch_setup_single(int T, const uint8_t* ptr, int* n_active, ActEntry* act, int* n_tg,
                         int* tg_expert, int* tg_begin, int* pair_tok, int* pair_pick,
                         int* out_row, cudaStream_t s, uint64_t* launches);

}  // namespace osm
