/*
 * osm_oracle.h -- CPU restatement of the ORBI StreamMoE routed-MoE sublayer.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * path: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
 * may load it.  The product (orbi-streammoe_b200/) never links or calls it.
 *
 * Every function restates one function of the reference's CPU path
 * (src/cpu/reference_ops.cpp, src/model/qwen_router.cpp,
 * src/model/shared_expert.cpp, src/model/routed_moe.cpp,
 * src/model/checkpoint_moe_sublayer.cpp,
 * src/conversion/single_expert_pilot.cpp) with the same operation order, so
 * that on x86-64 (no FMA contraction: built with -ffp-contract=off) the
 * results are bit-identical to the reference compiled in place.  The
 * restatement is pinned against (a) the known-answer tests of the reference's
 * own test files (tests/golden/reference_kats.json) and (b) the reference
 * compiled from its sources (oracle/_ref/libosm_ref.so) on seeded inputs.
 *
 * Return codes: 0 ok, -1 invalid argument (reference: std::invalid_argument),
 * -2 runtime error (reference: std::runtime_error).
 */
#ifndef OSM_ORACLE_H
#define OSM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* reference_ops.cpp:11-67 */
int osm_oracle_dequantize_affine_rows(const uint32_t* packed, size_t rows,
                                      size_t packed_cols, const float* scales,
                                      const float* biases, uint32_t bits,
                                      uint32_t group_size, float* out);
/* reference_ops.cpp:69-94 */
int osm_oracle_matvec_row_major(const float* weight, size_t out_dim,
                                size_t in_dim, const float* x, float* out);
/* reference_ops.cpp:96-128; weight may be NULL (unit weight) */
int osm_oracle_rms_norm_inplace(float* values, size_t rows, size_t dim,
                                const float* weight, float eps);
/* reference_ops.cpp:130-151 */
int osm_oracle_softmax_inplace(float* values, size_t n);
/* reference_ops.cpp:153-212 */
int osm_oracle_route_top_k(const float* logits, size_t n, size_t k,
                           int normalize_selected, uint32_t* experts,
                           float* probabilities);
/* reference_ops.cpp:214-232 */
float osm_oracle_sigmoid(float v);
float osm_oracle_silu(float v);
int osm_oracle_swiglu_inplace(float* gate, const float* up, size_t n);

/* qwen_router.cpp:11-94.  logit_bias (nullable, [E]) is added to the logits
 * before top-k: the biased-router harness of the batch-decode config, which
 * calls matvec_row_major, adds the bias, then route_top_k and the renorm steps
 * of qwen_router.cpp:68-91.  logits_out receives the (biased) logits. */
int osm_oracle_route_qwen_top_k(const float* hidden, const float* router_weight,
                                const float* logit_bias, size_t hidden_size,
                                size_t expert_count, size_t top_k,
                                int norm_topk_prob, float* logits_out,
                                uint32_t* experts, float* weights,
                                float* selected_mass);

/* single_expert_pilot.cpp:276-346 (packed must be zeroed by the callee). */
int osm_oracle_quantize_affine_q4_rows(const float* values, size_t rows,
                                       size_t cols, size_t group_size,
                                       uint32_t* packed, float* scales,
                                       float* biases);

/* bf16 helpers.  Widening is vulkan_qpack_expert.cpp:54-56 (bits << 16);
 * narrowing is round-to-nearest-even (the harness choice for generated
 * scale/bias; NaN is kept quiet). */
float osm_oracle_bf16_to_f32(uint16_t bits);
uint16_t osm_oracle_f32_to_bf16_rne(float v);
void osm_oracle_bf16_widen(const uint16_t* in, float* out, size_t n);
void osm_oracle_bf16_narrow(const float* in, uint16_t* out, size_t n);

/* The expert slot layout used everywhere in this project: the qpack sections
 * gate_proj.{weight,scales,biases}, up_proj.{...}, down_proj.{...} packed
 * back to back (U32 words, BF16 metadata), as in the reference fixtures
 * (tests/weighted_routed_moe_test.cpp:139-163).  Offsets in bytes. */
typedef struct {
  size_t hidden, inter, group;
  size_t gate_w, gate_s, gate_b, up_w, up_s, up_b, down_w, down_s, down_b;
  size_t stride;
} osm_oracle_slot_layout;
void osm_oracle_slot_layout_make(size_t hidden, size_t inter, size_t group,
                                 osm_oracle_slot_layout* out);

/* Dequantise one expert slot to fp32 row-major gate [I,H], up [I,H],
 * down [H,I] (bind_qpack_q4_projection + dequantize_affine_rows, as the
 * reference test oracle does, tests/weighted_routed_moe_test.cpp:217-244). */
int osm_oracle_dequant_slot(const uint8_t* slot, size_t hidden, size_t inter,
                            size_t group, float* gate, float* up, float* down);

/* One expert MLP on fp32 weights: matvec(gate), matvec(up), swiglu, matvec
 * (down) (tests/weighted_routed_moe_test.cpp:246-252). */
int osm_oracle_expert_mlp(const float* gate, const float* up, const float* down,
                          size_t hidden, size_t inter, const float* x,
                          float* out);

/* shared_expert.cpp:11-87: out = sigmoid(scalar_gate . x) * down(...). */
int osm_oracle_shared_expert(const float* gate, const float* up,
                             const float* down, const float* scalar_gate,
                             size_t hidden, size_t inter, const float* x,
                             float* out, float* scale_out);

/* One token of the sparse MoE (routed_moe.cpp:254-430 semantics with the
 * host accumulation order of routed_moe.cpp:13-92): routed experts in pick
 * order, acc[i] += w*out[i], then the shared expert acc[i] += s*out[i].
 * expert_w[e] points at 3 fp32 matrices of expert e (gate, up, down, each
 * contiguous; NULL for experts that are not picked).  shared_* may be NULL
 * (no shared expert).  Writes the routing as osm_oracle_route_qwen_top_k. */
int osm_oracle_moe_token(const float* hidden, const float* router_weight,
                         const float* logit_bias, size_t hidden_size,
                         size_t expert_count, size_t top_k, int norm_topk_prob,
                         size_t inter, const float* const* expert_gate,
                         const float* const* expert_up,
                         const float* const* expert_down,
                         const float* shared_gate, const float* shared_up,
                         const float* shared_down, const float* scalar_gate,
                         size_t shared_inter, float* out, uint32_t* experts,
                         float* weights, float* selected_mass,
                         float* shared_scale);

/* osm_oracle_moe_token over Q4 expert slots (expert e at slots + e *
 * slot_stride; shared_slot may be NULL): dequantises only the picked experts
 * with osm_oracle_dequant_slot, then runs osm_oracle_moe_token -- the same
 * arithmetic without every expert in fp32.  The shared expert has the routed
 * experts' intermediate size. */
int osm_oracle_moe_token_slots(const float* hidden, const float* router_weight,
                               const float* logit_bias, size_t hidden_size,
                               size_t expert_count, size_t top_k,
                               int norm_topk_prob, size_t inter,
                               const uint8_t* slots, size_t slot_stride,
                               const uint8_t* shared_slot,
                               const float* scalar_gate, float* out,
                               uint32_t* experts, float* weights,
                               float* selected_mass, float* shared_scale);

/* checkpoint_moe_sublayer.cpp:21-33 */
int osm_oracle_add_residual(const float* residual, const float* branch,
                            float* out, size_t n);

/* Seeded synthetic data: splitmix64 counter hash -> two uniforms -> Box-Muller
 * evaluated in double, rounded to float, times sigma.  element i of stream
 * (seed, tensor) is independent of every other element. */
uint64_t osm_oracle_hash(uint64_t seed, uint64_t tensor, uint64_t index);
void osm_oracle_gen_normal(uint64_t seed, uint64_t tensor, float sigma,
                           float* out, size_t n, size_t first_index);

/* Generate one expert slot: gate/up [I,H], down [H,I] ~ N(0, sigma) from
 * (seed, tensor_base + {0,1,2}), quantised with the reference quantiser and
 * bf16-rounded (RNE) scale/bias.  slot must hold layout.stride bytes. */
int osm_oracle_gen_expert_slot(uint64_t seed, uint64_t tensor_base, float sigma,
                               size_t hidden, size_t inter, size_t group,
                               uint8_t* slot);

#ifdef __cplusplus
}
#endif
#endif
