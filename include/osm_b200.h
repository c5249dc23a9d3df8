/*
 * osm_b200.h -- C ABI of the B200 (sm_100a) routed-MoE sublayer.
 *
 * Plain pointers, sizes and int status codes; no C++ or torch types.  Every
 * entry point names the interface of the reference (ingeniusvictor/
 * orbi-streammoe, paths inside that project) that it replaces.
 *
 * Conventions
 *  - Return 0 on success, a negative OSM_E* code on failure; the text of the
 *    last failure of a context is osm_last_error(ctx).  No C++ exception
 *    crosses this boundary (the reference's entry points are noexcept and
 *    report `executed=false` + `diagnostic`, e.g. src/model/routed_moe.cpp).
 *  - Pointers named *_dev are device pointers; *_host are host pointers.
 *  - Work is enqueued on the context's stream.  Functions documented as
 *    "synchronous" wait for the stream before returning, like the reference's
 *    fence waits (src/backend/vulkan_q4_gemv.cpp:1645-1657).
 *  - Geometry: Q4 = MLX affine 4-bit, eight nibbles per uint32 LSB first,
 *    group 64 along the input dimension, BF16 scale and bias
 *    (src/cpu/reference_ops.cpp:11-67, shaders/q4_gemv.comp:32-63).
 *  - The reference's C++ classes (VulkanComputeContext, VulkanFloatBuffer,
 *    VulkanResidentExpertCache, ... under include/orbi/streammoe/backend/)
 *    are implemented over this ABI by the C++ drop-in layer in
 *    orbi-streammoe_b200/host (headers with the reference's exact public
 *    declarations, sources replacing the .cpp files of src/backend).
 */
#ifndef OSM_B200_H
#define OSM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OSM_OK 0
#define OSM_EINVAL (-1)   /* invalid argument (reference: std::invalid_argument) */
#define OSM_ERUNTIME (-2) /* runtime failure (reference: std::runtime_error) */
#define OSM_ECUDA (-3)    /* a CUDA call failed */
#define OSM_ENOMEM (-4)   /* device or pinned allocation failed */
#define OSM_ENOTRES (-5)  /* a routed expert is not resident in the slab */
#define OSM_ETIMEOUT (-6) /* a bounded wait gave up */

/* Flags for osm_moe_forward / osm_moe_route / osm_rms_norm. */
#define OSM_ROUTE_EXACT 0x1u      /* route every token on the exact path */
#define OSM_RMSNORM_EXACT 0x2u    /* sequential RMSNorm sum (bit-exact)   */
#define OSM_ADD_RESIDUAL 0x4u     /* out = residual + MoE(...)            */
#define OSM_PREFILL_BF16 0x8u     /* experts as a 16-bit tensor-core grouped GEMM (tcgen05, fp16
                                     operands, fp32 accumulation) for prefill-sized batches; outputs
                                     within 2e-3 of the fp32 path; |x|, h < 65504 (status bit 5) */
#define OSM_INPUT_F16 0x10u       /* osm_moe_experts with OSM_PREFILL_BF16: x_dev holds fp16 rows
                                     [tokens][hidden] (layers without a shared expert) */
#define OSM_OUTPUT_F16 0x20u      /* osm_moe_experts with OSM_PREFILL_BF16: out_dev receives fp16
                                     rows [tokens][hidden] (each fp32 sum rounded once) */
#define OSM_PREFILL_NO_CHECK 0x40u /* osm_moe_forward with OSM_PREFILL_BF16: skip the range check.
                                     By default (and never inside stream capture) the call ends
                                     with a stream synchronisation that reads its status; when a
                                     value left the fp16 range it runs again on the fp32 path
                                     (status bit 6 then reports it) */
#define OSM_CACHED_EARLY 0x80u    /* osm_moe_forward_cached, one or two tokens: queue the expert
                                     kernels right behind the router, before the host has the
                                     picks; when the acquire finds every pick resident their
                                     output stands, otherwise they run again behind the copies */

typedef struct osm_context osm_context;
typedef struct osm_layer osm_layer;
typedef struct osm_slab osm_slab;
typedef struct osm_ep osm_ep;

#define OSM_IPC_HANDLE_BYTES 64

/* Byte offsets of the nine qpack sections inside one expert slot
 * (gate_proj/up_proj/down_proj . weight/scales/biases; the section table of
 * the reference's layout.json, src/container/qpack.cpp:67-97). */
typedef struct {
  uint32_t hidden;       /* H: input of gate/up, output of down        */
  uint32_t inter;        /* I: moe_intermediate_size                   */
  uint32_t group;        /* quantisation group (64)                    */
  uint32_t reserved;
  uint64_t gate_w, gate_s, gate_b;
  uint64_t up_w, up_s, up_b;
  uint64_t down_w, down_s, down_b;
  uint64_t stride;       /* bytes per slot                              */
} osm_expert_layout;

/* Fill `out` with the packed back-to-back layout (U32 weights, BF16
 * metadata) used by the reference's fixtures and the synthetic configs. */
int osm_expert_layout_packed(uint32_t hidden, uint32_t inter, uint32_t group,
                             osm_expert_layout* out);

/* ---- context: replaces VulkanComputeContext
 *      (include/orbi/streammoe/backend/vulkan_compute_context.hpp:19-49) ---- */
int osm_context_create(int device, uint32_t max_tokens, osm_context** out);
/* The device's name and SM count, for VulkanComputeContext::info()
 * (include/orbi/streammoe/backend/vulkan_compute_context.hpp:33). */
int osm_device_info(int device, char* name, size_t name_bytes, uint32_t* sms,
                    uint32_t* runtime_version);
int osm_context_destroy(osm_context* ctx);
const char* osm_last_error(const osm_context* ctx);
int osm_context_device(const osm_context* ctx);
void* osm_context_stream(const osm_context* ctx); /* cudaStream_t */
/* Enqueue all later work on `cuda_stream` (caller-owned; NULL is the CUDA
 * default stream).  osm_context_reset_stream returns to the context's own
 * non-blocking stream. */
int osm_context_set_stream(osm_context* ctx, void* cuda_stream);
int osm_context_reset_stream(osm_context* ctx);
int osm_context_synchronize(osm_context* ctx);
/* Device status word accumulated by kernels since the last call (bit 0
 * non-finite router input, bit 1 invalid softmax/mass, bit 2 non-resident
 * expert, bit 3 bad slot, bit 4 a bounded wait on an asynchronous weight
 * copy gave up, bit 5 an activation left the fp16 range on the
 * OSM_PREFILL_BF16 path, whose outputs are then invalid, bit 6 a checked
 * OSM_PREFILL_BF16 call found bit 5 and re-ran on the fp32 path, whose
 * outputs stand, bit 7 an expert-parallel barrier gave up waiting for a
 * rank, whose outputs are then invalid); the count of tokens
 * routed on the exact path. */
int osm_context_status(osm_context* ctx, uint32_t* status,
                       uint64_t* exact_tokens);

/* Test hook (no counterpart in the reference): the number of polls of the
 * first bounded wait a kernel makes on an asynchronous weight copy, on
 * `device`, for every later launch in this process.  When that wait gives up
 * the kernel sets status bit 4 and waits again with the full bound, so the
 * results stand; 0 makes every first wait give up at once, UINT32_MAX
 * restores the default. */
int osm_test_set_copy_wait_polls(int device, uint32_t polls);

/* ---- buffers: replaces VulkanFloatBuffer
 *      (include/orbi/streammoe/backend/vulkan_float_buffer.hpp:23-58) ---- */
int osm_device_alloc(osm_context* ctx, size_t bytes, void** dev);
int osm_device_free(osm_context* ctx, void* dev);
int osm_upload(osm_context* ctx, void* dev, const void* host, size_t bytes);
int osm_download(osm_context* ctx, void* host, const void* dev, size_t bytes);
int osm_host_alloc_pinned(size_t bytes, void** host);
int osm_host_free_pinned(void* host);

/* ---- element-wise ops (each replaces one Vulkan kernel) ---- */

/* run_vulkan_q4_dequant (src/backend/vulkan_q4_dequant.cpp:270,
 * shaders/q4_dequant.comp): out[r][c] = scale*q + bias, bit-exact with
 * cpu::dequantize_affine_rows (separate multiply and add, no FMA).  Any
 * group size that divides in_dim; in_dim a multiple of 8. */
int osm_q4_dequant(osm_context* ctx, const uint32_t* packed_dev,
                   const uint16_t* scales_bf16_dev,
                   const uint16_t* biases_bf16_dev, uint32_t rows,
                   uint32_t in_dim, uint32_t group, float* out_dev);

/* The same with fp32 scale and bias (the reference's device format,
 * src/backend/vulkan_q4_weights.cpp), for metadata bf16 cannot hold exactly;
 * any-geometry kernel. */
int osm_q4_dequant_f32(osm_context* ctx, const uint32_t* packed_dev,
                       const float* scales_dev, const float* biases_dev,
                       uint32_t rows, uint32_t in_dim, uint32_t group,
                       float* out_dev);

/* run_vulkan_q4_gemv_preloaded (include/orbi/streammoe/backend/
 * vulkan_q4_gemv.hpp:53-57): y[t][r] = sum_c w[r][c] * x[t][c] for `tokens`
 * input vectors (batched; the reference is tokens == 1).  Group 64, in_dim a
 * multiple of 64 up to 2048, out_dim a multiple of 16 and tokens up to the
 * context's max_tokens run on the row-tiled projection kernel; any other
 * geometry (group dividing in_dim, in_dim a multiple of 8) on a one-warp-per-
 * row kernel. */
int osm_q4_gemv(osm_context* ctx, const uint32_t* packed_dev,
                const uint16_t* scales_bf16_dev,
                const uint16_t* biases_bf16_dev, uint32_t out_dim,
                uint32_t in_dim, uint32_t group, const float* x_dev,
                uint32_t tokens, float* y_dev);
/* osm_q4_gemv with fp32 scale and bias (see osm_q4_dequant_f32). */
int osm_q4_gemv_f32(osm_context* ctx, const uint32_t* packed_dev,
                    const float* scales_dev, const float* biases_dev,
                    uint32_t out_dim, uint32_t in_dim, uint32_t group,
                    const float* x_dev, uint32_t tokens, float* y_dev);

/* run_vulkan_swiglu_buffers (include/orbi/streammoe/backend/
 * vulkan_swiglu.hpp:26-30): out = silu(gate) * up. */
int osm_swiglu(osm_context* ctx, const float* gate_dev, const float* up_dev,
               float* out_dev, size_t count);

/* run_vulkan_weighted_accumulate (include/orbi/streammoe/backend/
 * vulkan_weighted_accumulate.hpp:12-16): acc += weight * src. */
int osm_weighted_accumulate(osm_context* ctx, const float* src_dev,
                            float weight, float* acc_dev, size_t count);

/* run_vulkan_rms_norm (include/orbi/streammoe/backend/vulkan_rmsnorm.hpp:
 * 25-31): in place, rows x dim, weight_dev may be NULL (unit weight).
 * flags & OSM_RMSNORM_EXACT sums squares sequentially (bit-exact with
 * cpu::rms_norm_inplace); otherwise a block reduction (within 1e-6). */
int osm_rms_norm(osm_context* ctx, float* values_dev, uint32_t rows,
                 uint32_t dim, const float* weight_dev, float eps,
                 uint32_t flags);

/* VulkanResidentExpert::run_from_buffer (include/orbi/streammoe/backend/
 * vulkan_resident_expert.hpp:64-66): one expert's gate/up -> SwiGLU -> down
 * on `tokens` inputs; slot_dev points at one expert slot of `layout`. */
int osm_expert_forward(osm_context* ctx, const void* slot_dev,
                       const osm_expert_layout* layout, const float* x_dev,
                       uint32_t tokens, float* out_dev);

/* Allocation-free variant of osm_expert_forward.  It has no counterpart in
 * the reference: it is for hosts that cannot call cudaMalloc where experts
 * run (a server whose device memory belongs to a pool allocator that forbids
 * driver allocations after warm-up, or a plugin that only borrows a CUDA
 * context it did not create).  No context is needed and nothing is
 * allocated: the intermediates live in one fixed device array of this
 * library (254 KB, held on every GPU that loads it until the process
 * exits), on the device current at the call, launched on `cuda_stream`
 * (NULL: the legacy default stream).  Limits: tokens 1..16, hidden <= 2048,
 * inter <= 768; anything larger, or an unsupported layout, returns
 * OSM_EINVAL before any GPU work.  The first call on a device sets it up
 * (looks up the array's device address and sets kernel attributes); make
 * that first call before any stream capture.  Each call clears the array
 * before use.  All calls on a device share the one array: calls that can
 * overlap on the GPU (other streams, other host threads) race and must be
 * serialised by the caller.  Returns OSM_OK, OSM_EINVAL or OSM_ECUDA. */
int osm_expert_forward_noalloc(const void* slot_dev,
                               const osm_expert_layout* layout,
                               const float* x_dev, uint32_t tokens,
                               float* out_dev, void* cuda_stream);

/* ---- expert parallelism over NVLink peer memory (configs 2 and 3 across
 *      the GPUs of one box; no counterpart in the reference, whose sublayer
 *      runs on one device).  Rank r of W owns experts [r E/W, (r+1) E/W).
 *      Each rank allocates one EP block (receive regions, back rows,
 *      barrier flags), exports it with osm_ep_ipc_handle, and maps every
 *      other rank's block with osm_ep_open_peers (the handles gathered on the
 *      host, e.g. by torch.distributed.all_gather_object).  osm_ep_forward is
 *      then one call per step with no host synchronisation: route (ids exact
 *      as on one GPU), store each pick's fp16 row into its owner's block,
 *      barrier, run the owned experts (and this rank's shared-expert rows) on
 *      the tensor-core prefill path, store each weighted fp16 result into the
 *      source's back rows, barrier, sum each token's rows in pick order and
 *      its shared row (fp32).  Every rank must call it the same number of
 *      times.  A barrier waits at most the block's timeout (default 2 s,
 *      osm_ep_set_timeout) and then sets status bit 7.  Destroy the blocks
 *      only after every rank has finished using them (a host barrier). ---- */
int osm_ep_create(osm_context* ctx, uint32_t world, uint32_t rank,
                  uint32_t tokens_per_rank, uint32_t k, uint32_t hidden,
                  uint32_t experts_per_rank, int has_shared, osm_ep** out);
int osm_ep_ipc_handle(const osm_ep* ep, unsigned char* handle /* OSM_IPC_HANDLE_BYTES */);
/* handles: world x OSM_IPC_HANDLE_BYTES, rank order (this rank's is ignored) */
int osm_ep_open_peers(osm_ep* ep, const unsigned char* handles);
int osm_ep_set_timeout(osm_ep* ep, uint32_t timeout_ms);
int osm_ep_destroy(osm_ep* ep);
/* router: the full router (E = experts_per_rank * world, top-k; with
 * has_shared it holds the shared expert, whose gate it computes).  experts:
 * k = 1 over this rank's experts in slots 0..experts_per_rank-1 and, with
 * has_shared, the shared expert as local id experts_per_rank.  x_dev/out_dev
 * [tokens][hidden] fp32 (tokens <= tokens_per_rank); ids/weights outputs may
 * be NULL.  Flags: OSM_ROUTE_EXACT. */
int osm_ep_forward(osm_ep* ep, osm_layer* router, osm_layer* experts,
                   const float* x_dev, uint32_t tokens, float* out_dev,
                   uint32_t* ids_dev, float* weights_dev, uint32_t flags);

/* ---- expert slab: the HBM side of VulkanResidentExpertCache
 *      (include/orbi/streammoe/backend/vulkan_resident_expert_cache.hpp:
 *      27-83); the policy lives in the host layer ---- */
int osm_slab_create(osm_context* ctx, const osm_expert_layout* layout,
                    uint32_t slots, osm_slab** out);
int osm_slab_destroy(osm_slab* slab);
uint32_t osm_slab_slots(const osm_slab* slab);
void* osm_slab_slot_ptr(const osm_slab* slab, uint32_t slot);
/* The expert layout the slab was created with. */
int osm_slab_layout(const osm_slab* slab, osm_expert_layout* out);
/* Copy one slot's bytes from (ideally pinned) host memory on the slab's side
 * stream; the copy is ordered before the next kernel on the context stream
 * that reads the slab (an event is recorded and waited on). */
int osm_slab_fill_async(osm_slab* slab, uint32_t slot, const void* host_src);
/* Block until every fill issued so far has landed, with a time limit. */
int osm_slab_fill_wait(osm_slab* slab, uint32_t timeout_ms);
/* Bytes copied host->device by fills since creation. */
uint64_t osm_slab_h2d_bytes(const osm_slab* slab);

/* ---- HBM expert cache: the residency policy of VulkanResidentExpertCache
 *      (include/orbi/streammoe/backend/vulkan_resident_expert_cache.hpp:
 *      27-83, src/backend/vulkan_resident_expert_cache.cpp:40-200) over slab
 *      slots.  Each get() counts a use of (layer, expert); a miss evicts the
 *      resident entry with the smallest (use count, last use, key) -- use
 *      counts survive evictions -- until the newcomer's accounted bytes fit
 *      the budget and a slot is free, then copies the expert from the host
 *      source into the freed slot and rebinds the layers registered with
 *      osm_cache_bind_layer.  slab NULL: the policy alone (no copies). ---- */
typedef struct osm_cache osm_cache;
typedef struct osm_cache_counts {
  uint64_t hits, misses, loads, evictions;
  uint64_t resident_entries, resident_bytes, budget_bytes;
} osm_cache_counts;
/* Host level of the cache (ExpertCache::fetch, src/cache/expert_cache.cpp):
 * sets *src to the expert's slot bytes in (ideally pinned) host memory, which
 * must stay valid until the copy has landed; returns 0 on success. */
typedef int (*osm_cache_source_fn)(void* user, uint32_t layer, uint32_t expert,
                                   const void** src);
/* accounted_bytes 0: the slab's slot stride. */
int osm_cache_create(osm_slab* slab, uint64_t budget_bytes,
                     uint64_t accounted_bytes, osm_cache_source_fn source,
                     void* user, osm_cache** out);
int osm_cache_destroy(osm_cache* cache);
const char* osm_cache_last_error(const osm_cache* cache);
int osm_cache_bind_layer(osm_cache* cache, uint32_t layer_id, osm_layer* layer);
/* VulkanResidentExpertCache::get for one expert; *slot_out may be NULL. */
int osm_cache_get(osm_cache* cache, uint32_t layer_id, uint32_t expert,
                  int32_t* slot_out);
/* get() for each of n experts in order (the picks of a call); entries used by
 * this acquire are not evicted by it (OSM_ENOMEM when they cannot all fit). */
int osm_cache_acquire(osm_cache* cache, uint32_t layer_id,
                      const uint32_t* experts, uint32_t n);
int osm_cache_contains(const osm_cache* cache, uint32_t layer_id,
                       uint32_t expert);
int osm_cache_stats(const osm_cache* cache, osm_cache_counts* out);
/* Exposed-copy timing (the reference's config-4 "exposed H2D time"): with
 * enable set, every acquire that copies brackets its copies with a pair of
 * events on the compute stream, from their issue to the compute stream's
 * wait for them ending.  osm_cache_exposed_read waits for the recorded pairs
 * and returns their summed time in ms and their count, then starts over. */
int osm_cache_time_copies(osm_cache* cache, int enable);
int osm_cache_exposed_read(osm_cache* cache, double* ms, uint64_t* waits);

/* ---- one MoE layer: the dense state QwenCheckpointSparseMoeLayer keeps
 *      (src/model/checkpoint_sparse_moe.cpp:112-220): router, shared expert
 *      and its scalar gate, plus the table expert -> slab slot ---- */
typedef struct {
  uint32_t hidden;          /* H                                         */
  uint32_t experts;         /* E (<= 1024)                               */
  uint32_t top_k;           /* k (<= 32)                                 */
  uint32_t norm_topk_prob;  /* renormalise the selected weights          */
  const float* router_weight_host;   /* [E][H] fp32, row-major; kept as
                                        bf16 on the device when every
                                        value is bf16-representable, else
                                        as fp32 (a dequantised Q8 router) */
  const float* logit_bias_host;      /* [E] or NULL                      */
  const void* shared_slot_host;      /* one slot of shared_layout or NULL */
  osm_expert_layout shared_layout;   /* ignored without a shared expert  */
  const float* shared_gate_host;     /* [H] scalar gate (fp32)           */
  const float* norm_weight_host;     /* [H] post-attention norm or NULL  */
  float norm_eps;
} osm_layer_desc;

int osm_layer_create(osm_context* ctx, const osm_layer_desc* desc,
                     osm_layer** out);
int osm_layer_destroy(osm_layer* layer);
/* Bind routed experts to slab slots: slot_of_expert[e] = slot, or -1 when
 * expert e is not resident (routing to it then fails with OSM_ENOTRES). */
int osm_layer_bind_slab(osm_layer* layer, osm_slab* slab,
                        const int32_t* slot_of_expert_host);
/* The router as the checkpoint stores it: MLX-affine 8-bit, group 64
 * (packed_host: [experts][hidden / 4] u32, four values per word LSB first;
 * scales/biases: [experts][hidden / 64] bf16), kept 8-bit on the device
 * (hidden + 4 * hidden / 64 bytes per expert instead of 2 or 4 * hidden) and
 * dequantised as the kernels read it, in the operation order of
 * cpu::dequantize_affine_rows (src/cpu/reference_ops.cpp:11-67): the logits
 * and ids are those of the reference's fp32 router
 * (src/model/checkpoint_sparse_moe.cpp:159-162 dequantises the same module to
 * fp32 on the host).  Replaces the router given at creation.  Needs hidden a
 * multiple of 256, experts a multiple of 32, 16-byte aligned x in later
 * calls, and no plan of the context alive. */
int osm_layer_set_router_q8(osm_layer* layer, const uint32_t* packed_host,
                            const uint16_t* scales_bf16_host,
                            const uint16_t* biases_bf16_host, uint32_t group);
/* Rebind a single expert (cache fill / eviction). */
int osm_layer_set_slot(osm_layer* layer, uint32_t expert, int32_t slot);

/* route_qwen_top_k_cpu (include/orbi/streammoe/model/qwen_router.hpp:42-45):
 * logits = W x (+ bias), softmax, top-k, renormalise, for `tokens` rows of
 * x_dev.  ids_dev [tokens][k] u32, weights_dev [tokens][k], mass_dev
 * [tokens] (selected probability mass); any output may be NULL. */
int osm_moe_route(osm_layer* layer, const float* x_dev, uint32_t tokens,
                  uint32_t* ids_dev, float* weights_dev, float* mass_dev,
                  uint32_t flags);

/* route_qwen_top_k_cpu with its QwenRouterResult::logits: as osm_moe_route
 * with every token on the reference's own arithmetic (OSM_ROUTE_EXACT), and
 * the fp32 logits the softmax sees (W x, plus the layer's logit bias when it
 * has one) written to logits_dev [tokens][experts].  Inputs with a
 * non-finite value leave logits_dev unwritten and route to expert 0 with
 * weight 0, as osm_moe_route does. */
int osm_moe_route_logits(osm_layer* layer, const float* x_dev, uint32_t tokens,
                         float* logits_dev, uint32_t* ids_dev, float* weights_dev,
                         float* mass_dev);

/* run_qwen_sparse_moe_vulkan_accum (include/orbi/streammoe/model/
 * routed_moe.hpp:58-65), batched: route, run the picked experts and the
 * shared expert, combine in pick order.  Every picked expert must be bound
 * to a slab slot.  shared_gate_dev [tokens] receives sigmoid(g . x) (or 0
 * without a shared expert).  With OSM_ADD_RESIDUAL, residual_dev is added. */
int osm_moe_forward(osm_layer* layer, const float* x_dev, uint32_t tokens,
                    float* out_dev, uint32_t* ids_dev, float* weights_dev,
                    float* mass_dev, float* shared_gate_dev,
                    const float* residual_dev, uint32_t flags);

/* Expert half of osm_moe_forward for a routing already in device memory
 * (after osm_moe_route and host-side cache fills).  OSM_PREFILL_BF16 selects
 * the tensor-core prefill path as for osm_moe_forward; with OSM_INPUT_F16 the
 * rows are already fp16 (as an expert-parallel exchange delivers them), with
 * OSM_OUTPUT_F16 the output rows are fp16 (as the exchange returns them).  On
 * the prefill path out_dev and residual_dev are 16-byte aligned. */
int osm_moe_experts(osm_layer* layer, const float* x_dev, uint32_t tokens,
                    const uint32_t* ids_dev, const float* weights_dev,
                    float* out_dev, float* shared_gate_dev,
                    const float* residual_dev, uint32_t flags);

/* run_qwen_sparse_moe_vulkan_accum with its VulkanResidentExpertCache and
 * layer index (include/orbi/streammoe/model/routed_moe.hpp:58-65): route,
 * read the picks back to the host, make them resident through `cache` (one
 * osm_cache_acquire in token-major pick order; misses are copied from the
 * cache's host source on the slab's side stream), then run the experts and
 * the shared expert.  `layer` must be bound to `cache` as `layer_id`.  The
 * call returns once the picks are known and the copies and kernels are
 * queued; outputs as for osm_moe_forward (ids_dev, weights_dev,
 * shared_gate_dev may be NULL).  Flags: OSM_ROUTE_EXACT, OSM_PREFILL_BF16,
 * OSM_ADD_RESIDUAL, OSM_CACHED_EARLY (the result is the same; the early
 * run's non-resident picks do not reach osm_context_status). */
int osm_moe_forward_cached(osm_layer* layer, osm_cache* cache, uint32_t layer_id,
                           const float* x_dev, uint32_t tokens, float* out_dev,
                           uint32_t* ids_dev, float* weights_dev,
                           float* shared_gate_dev, const float* residual_dev,
                           uint32_t flags);

/* No counterpart in the reference (its MoE runs on one device): the return
 * step of an expert-parallel exchange.  out[t] (fp32, [tokens][hidden]) =
 * the sum, in order p = 0..k-1, of the fp16 rows rows_f16[pos[t k + p]]
 * (already weighted by their owners), then + extra_f16[t] when given (the
 * token's own shared-expert row); fp32 adds, one rounding each.  hidden % 8
 * == 0; rows, extra and out 16-byte aligned. */
int osm_gather_sum_rows(osm_context* ctx, const void* rows_f16, const int64_t* pos,
                        uint32_t tokens, uint32_t k, uint32_t hidden,
                        const void* extra_f16, float* out);

/* QwenCheckpointMoeSublayer::run (include/orbi/streammoe/model/
 * checkpoint_moe_sublayer.hpp:55-58): normalized = RMSNorm(residual),
 * out = residual + MoE(normalized).  normalized_dev may be NULL. */
int osm_moe_sublayer_forward(osm_layer* layer, const float* residual_dev,
                             uint32_t tokens, float* out_dev,
                             float* normalized_dev, uint32_t* ids_dev,
                             float* weights_dev, float* mass_dev,
                             float* shared_gate_dev, uint32_t flags);

/* ---- execution plans: one call captured as a CUDA graph (no counterpart in
 *      the reference, whose every GPU op is a synchronous submit + fence,
 *      src/backend/vulkan_q4_gemv.cpp:1645-1657).  A plan replays
 *      osm_moe_forward (or, with OSM_PLAN_SUBLAYER, osm_moe_sublayer_forward)
 *      on fixed device buffers with one graph launch.  When x_host / out_host
 *      (pinned) are given, the H2D copy of x and the D2H copy of out are part
 *      of the plan: copied by the SMs through the GPU's mapping of the pinned
 *      buffer when it is mapped, 16-byte aligned and at most 2 MiB, by
 *      copy-engine nodes otherwise.  With OSM_PLAN_PROFILE each kernel is
 *      bracketed by event nodes, read by osm_plan_profile_read. ---- */
#define OSM_PLAN_SUBLAYER 0x100u
#define OSM_PLAN_PROFILE 0x200u
typedef struct osm_plan osm_plan;
int osm_plan_create(osm_layer* layer, uint32_t tokens, const float* x_dev, float* out_dev,
                    uint32_t* ids_dev, float* weights_dev, const float* x_host,
                    float* out_host, uint32_t flags, osm_plan** out);
int osm_plan_launch(osm_plan* plan);
int osm_plan_destroy(osm_plan* plan);
/* Adds the last replay's per-kernel times (OSM_PLAN_PROFILE plans). */
int osm_plan_profile_read(osm_plan* plan, double* ms, uint64_t* launches);
/* Kernels one replay launches. */
uint32_t osm_plan_kernels(const osm_plan* plan);

/* Number of kernels this library launched on `ctx` since creation. */
uint64_t osm_context_launches(const osm_context* ctx);

/* Per-kernel timing (no counterpart in the reference, which has no GPU
 * timers): while enabled, every launch is bracketed by CUDA events on the
 * context stream.  _read synchronises, adds each kind's elapsed milliseconds
 * and launch count into ms[OSM_KERNEL_KINDS] / launches[OSM_KERNEL_KINDS]
 * (either may be NULL) and clears the records. */
#define OSM_KERNEL_KINDS 8
int osm_context_profile(osm_context* ctx, int enable);
int osm_context_profile_read(osm_context* ctx, double* ms, uint64_t* launches);
const char* osm_kernel_kind_name(int kind);

/* ---- synthetic data (seeded; identical stream on host and device) ---- */
/* N(0, sigma) fp32 values of stream (seed, tensor), elements
 * [first, first + n), into device memory. */
int osm_gen_normal(osm_context* ctx, uint64_t seed, uint64_t tensor,
                   float sigma, float* out_dev, size_t n, size_t first);
/* Generate `count` expert slots of `layout` into consecutive slab slots
 * starting at first_slot: gate/up/down ~ N(0, sigma) from tensors
 * tensor_base + 3*i + {0,1,2}, quantised with the reference quantiser
 * (src/conversion/single_expert_pilot.cpp:276-346), bf16 (RNE) metadata. */
int osm_gen_expert_slots(osm_slab* slab, uint64_t seed, uint64_t tensor_base,
                         float sigma, uint32_t first_slot, uint32_t count);

#ifdef __cplusplus
}
#endif
#endif
