/*
 * osm_oracle.c -- CPU restatement of the reference's routed-MoE CPU path.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker; see osm_oracle.h).  Built
 * with -O2 -ffp-contract=off so that every multiply and add rounds on its
 * own, as the reference's x86-64 build does.  Each function names the
 * reference lines it restates; operation order is kept so results are
 * bit-identical to the reference compiled in place (oracle/_ref).
 */
#include "osm_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define OK 0
#define EINVAL_ARG (-1)
#define ERUNTIME (-2)

/* reference_ops.cpp:11-67 -- out = scale * q + bias, q read LSB-first. */
int osm_oracle_dequantize_affine_rows(const uint32_t* packed, size_t rows,
                                      size_t packed_cols, const float* scales,
                                      const float* biases, uint32_t bits,
                                      uint32_t group_size, float* out) {
  if (bits != 4 && bits != 8) return EINVAL_ARG;
  if (group_size == 0) return EINVAL_ARG;
  if (rows == 0 || packed_cols == 0) return EINVAL_ARG;
  const size_t per_word = 32u / bits;
  const size_t logical_cols = packed_cols * per_word;
  if (logical_cols % group_size != 0) return EINVAL_ARG;
  const size_t groups_per_row = logical_cols / group_size;
  const uint32_t mask = (1u << bits) - 1u;
  for (size_t row = 0; row < rows; ++row) {
    for (size_t w = 0; w < packed_cols; ++w) {
      uint32_t word = packed[row * packed_cols + w];
      const size_t col_base = w * per_word;
      for (size_t lane = 0; lane < per_word; ++lane) {
        const size_t col = col_base + lane;
        const size_t group = col / group_size;
        const float q = (float)(word & mask);
        const float s = scales[row * groups_per_row + group];
        const float b = biases[row * groups_per_row + group];
        out[row * logical_cols + col] = s * q + b;
        word >>= bits;
      }
    }
  }
  return OK;
}

/* reference_ops.cpp:69-94 -- sequential fp32 sum, one rounding per op. */
int osm_oracle_matvec_row_major(const float* weight, size_t out_dim,
                                size_t in_dim, const float* x, float* out) {
  if (out_dim == 0 || in_dim == 0) return EINVAL_ARG;
  for (size_t row = 0; row < out_dim; ++row) {
    float acc = 0.0f;
    const float* w = weight + row * in_dim;
    for (size_t col = 0; col < in_dim; ++col) acc += w[col] * x[col];
    out[row] = acc;
  }
  return OK;
}

/* reference_ops.cpp:96-128 */
int osm_oracle_rms_norm_inplace(float* values, size_t rows, size_t dim,
                                const float* weight, float eps) {
  if (rows == 0 || dim == 0) return EINVAL_ARG;
  if (eps < 0.0f) return EINVAL_ARG;
  for (size_t row = 0; row < rows; ++row) {
    float* v = values + row * dim;
    float sum_sq = 0.0f;
    for (size_t i = 0; i < dim; ++i) sum_sq += v[i] * v[i];
    const float scale = 1.0f / sqrtf(sum_sq / (float)dim + eps);
    for (size_t i = 0; i < dim; ++i) {
      const float w = weight == NULL ? 1.0f : weight[i];
      v[i] *= scale * w;
    }
  }
  return OK;
}

/* reference_ops.cpp:130-151 */
int osm_oracle_softmax_inplace(float* values, size_t n) {
  if (n == 0) return EINVAL_ARG;
  float max_value = values[0];
  for (size_t i = 1; i < n; ++i)
    if (max_value < values[i]) max_value = values[i];
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    values[i] = expf(values[i] - max_value);
    sum += values[i];
  }
  if (!(sum > 0.0f) || !isfinite(sum)) return ERUNTIME;
  for (size_t i = 0; i < n; ++i) values[i] /= sum;
  return OK;
}

/* reference_ops.cpp:153-212.  Candidates are visited in id order; a
 * candidate enters a full list only if strictly greater than the last pick,
 * and the list is kept stably sorted by descending probability, so equal
 * probabilities keep the lower expert id first. */
int osm_oracle_route_top_k(const float* logits, size_t n, size_t k,
                           int normalize_selected, uint32_t* experts,
                           float* probabilities) {
  if (n == 0) return EINVAL_ARG;
  if (k == 0 || k > n) return EINVAL_ARG;
  float* p = (float*)malloc(n * sizeof(float));
  if (p == NULL) return ERUNTIME;
  memcpy(p, logits, n * sizeof(float));
  int rc = osm_oracle_softmax_inplace(p, n);
  if (rc != OK) {
    free(p);
    return rc;
  }
  size_t count = 0;
  for (size_t e = 0; e < n; ++e) {
    const float cand = p[e];
    if (count == k) {
      if (!(cand > probabilities[k - 1])) continue;
      --count; /* drop the back, then re-insert stably */
    }
    size_t pos = count;
    /* stable insertion: after every pick whose probability is >= cand */
    while (pos > 0 && probabilities[pos - 1] < cand) {
      probabilities[pos] = probabilities[pos - 1];
      experts[pos] = experts[pos - 1];
      --pos;
    }
    probabilities[pos] = cand;
    experts[pos] = (uint32_t)e;
    ++count;
  }
  free(p);
  if (normalize_selected) {
    float sum = 0.0f;
    for (size_t i = 0; i < k; ++i) sum += probabilities[i];
    if (!(sum > 0.0f) || !isfinite(sum)) return ERUNTIME;
    for (size_t i = 0; i < k; ++i) probabilities[i] /= sum;
  }
  return OK;
}

/* reference_ops.cpp:214-220 */
float osm_oracle_sigmoid(float v) { return 1.0f / (1.0f + expf(-v)); }
float osm_oracle_silu(float v) { return v * osm_oracle_sigmoid(v); }

/* reference_ops.cpp:222-232 */
int osm_oracle_swiglu_inplace(float* gate, const float* up, size_t n) {
  for (size_t i = 0; i < n; ++i) gate[i] = osm_oracle_silu(gate[i]) * up[i];
  return OK;
}

/* qwen_router.cpp:11-94 (validation order kept; bias: see header). */
int osm_oracle_route_qwen_top_k(const float* hidden, const float* router_weight,
                                const float* logit_bias, size_t hidden_size,
                                size_t expert_count, size_t top_k,
                                int norm_topk_prob, float* logits_out,
                                uint32_t* experts, float* weights,
                                float* selected_mass) {
  if (hidden_size == 0 || expert_count == 0 || top_k == 0) return EINVAL_ARG;
  if (top_k > expert_count) return EINVAL_ARG;
  if (expert_count > 0xFFFFFFFFull) return EINVAL_ARG;
  for (size_t i = 0; i < hidden_size; ++i)
    if (!isfinite(hidden[i])) return EINVAL_ARG;
  for (size_t i = 0; i < expert_count * hidden_size; ++i)
    if (!isfinite(router_weight[i])) return EINVAL_ARG;
  int rc = osm_oracle_matvec_row_major(router_weight, expert_count, hidden_size,
                                       hidden, logits_out);
  if (rc != OK) return rc;
  if (logit_bias != NULL)
    for (size_t e = 0; e < expert_count; ++e) logits_out[e] += logit_bias[e];
  rc = osm_oracle_route_top_k(logits_out, expert_count, top_k, 0, experts,
                              weights);
  if (rc != OK) return rc;
  float mass = 0.0f;
  for (size_t i = 0; i < top_k; ++i) mass += weights[i];
  if (!(mass > 0.0f) || !isfinite(mass)) return ERUNTIME;
  *selected_mass = mass;
  if (norm_topk_prob)
    for (size_t i = 0; i < top_k; ++i) weights[i] /= mass;
  return OK;
}

/* single_expert_pilot.cpp:276-346 -- per group min/max affine, scale =
 * range/15 (1 if range is 0), bias = min, q = clamp(lround((v-bias)/scale)). */
int osm_oracle_quantize_affine_q4_rows(const float* values, size_t rows,
                                       size_t cols, size_t group_size,
                                       uint32_t* packed, float* scales,
                                       float* biases) {
  if (rows == 0 || cols == 0 || group_size == 0 || cols % 8 != 0 ||
      cols % group_size != 0)
    return EINVAL_ARG;
  const size_t packed_cols = cols / 8;
  const size_t groups_per_row = cols / group_size;
  memset(packed, 0, rows * packed_cols * sizeof(uint32_t));
  for (size_t row = 0; row < rows; ++row) {
    for (size_t g = 0; g < groups_per_row; ++g) {
      const size_t begin = row * cols + g * group_size;
      const size_t end = begin + group_size;
      float minimum = INFINITY, maximum = -INFINITY;
      for (size_t i = begin; i < end; ++i) {
        const float v = values[i];
        if (!isfinite(v)) return ERUNTIME;
        /* std::min(a, b) returns a unless b < a; std::max(a, b) returns a
         * unless a < b. */
        if (v < minimum) minimum = v;
        if (maximum < v) maximum = v;
      }
      const float range = maximum - minimum;
      const float scale = range > 0.0f ? range / 15.0f : 1.0f;
      const float bias = minimum;
      const size_t gi = row * groups_per_row + g;
      scales[gi] = scale;
      biases[gi] = bias;
      for (size_t i = begin; i < end; ++i) {
        const size_t col = i - row * cols;
        const float normalized = (values[i] - bias) / scale;
        long rounded = lroundf(normalized);
        if (rounded < 0) rounded = 0;
        if (rounded > 15) rounded = 15;
        const uint32_t q = (uint32_t)rounded;
        packed[row * packed_cols + col / 8] |= q << ((col % 8) * 4u);
        const float reconstructed = scale * (float)q + bias;
        const float error = fabsf(reconstructed - values[i]);
        const float allowed =
            range > 0.0f ? scale * 0.5001f + 1e-6f : 1e-6f;
        if (error > allowed) return ERUNTIME;
      }
    }
  }
  return OK;
}

float osm_oracle_bf16_to_f32(uint16_t bits) {
  uint32_t u = (uint32_t)bits << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

uint16_t osm_oracle_f32_to_bf16_rne(float v) {
  uint32_t u;
  memcpy(&u, &v, sizeof u);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu) != 0)
    return (uint16_t)((u >> 16) | 0x0040u);
  const uint32_t lsb = (u >> 16) & 1u;
  return (uint16_t)((u + 0x7FFFu + lsb) >> 16);
}

void osm_oracle_bf16_widen(const uint16_t* in, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = osm_oracle_bf16_to_f32(in[i]);
}

void osm_oracle_bf16_narrow(const float* in, uint16_t* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = osm_oracle_f32_to_bf16_rne(in[i]);
}

void osm_oracle_slot_layout_make(size_t hidden, size_t inter, size_t group,
                                 osm_oracle_slot_layout* L) {
  const size_t gu_w = inter * hidden / 2; /* U32 words, 8 nibbles each */
  const size_t gu_m = inter * (hidden / group) * 2;
  const size_t dn_w = hidden * inter / 2;
  const size_t dn_m = hidden * (inter / group) * 2;
  L->hidden = hidden;
  L->inter = inter;
  L->group = group;
  L->gate_w = 0;
  L->gate_s = L->gate_w + gu_w;
  L->gate_b = L->gate_s + gu_m;
  L->up_w = L->gate_b + gu_m;
  L->up_s = L->up_w + gu_w;
  L->up_b = L->up_s + gu_m;
  L->down_w = L->up_b + gu_m;
  L->down_s = L->down_w + dn_w;
  L->down_b = L->down_s + dn_m;
  L->stride = L->down_b + dn_m;
}

static int dequant_proj(const uint8_t* slot, size_t w_off, size_t s_off,
                        size_t b_off, size_t rows, size_t cols, size_t group,
                        float* out) {
  const size_t groups = rows * (cols / group);
  float* s = (float*)malloc(groups * sizeof(float));
  float* b = (float*)malloc(groups * sizeof(float));
  if (s == NULL || b == NULL) {
    free(s);
    free(b);
    return ERUNTIME;
  }
  uint16_t* tmp = (uint16_t*)malloc(groups * sizeof(uint16_t));
  if (tmp == NULL) {
    free(s);
    free(b);
    return ERUNTIME;
  }
  memcpy(tmp, slot + s_off, groups * 2);
  osm_oracle_bf16_widen(tmp, s, groups);
  memcpy(tmp, slot + b_off, groups * 2);
  osm_oracle_bf16_widen(tmp, b, groups);
  free(tmp);
  uint32_t* packed = (uint32_t*)malloc(rows * cols / 2);
  if (packed == NULL) {
    free(s);
    free(b);
    return ERUNTIME;
  }
  memcpy(packed, slot + w_off, rows * cols / 2);
  const int rc = osm_oracle_dequantize_affine_rows(packed, rows, cols / 8, s, b,
                                                   4, (uint32_t)group, out);
  free(packed);
  free(s);
  free(b);
  return rc;
}

int osm_oracle_dequant_slot(const uint8_t* slot, size_t hidden, size_t inter,
                            size_t group, float* gate, float* up, float* down) {
  osm_oracle_slot_layout L;
  osm_oracle_slot_layout_make(hidden, inter, group, &L);
  int rc = dequant_proj(slot, L.gate_w, L.gate_s, L.gate_b, inter, hidden,
                        group, gate);
  if (rc == OK)
    rc = dequant_proj(slot, L.up_w, L.up_s, L.up_b, inter, hidden, group, up);
  if (rc == OK)
    rc = dequant_proj(slot, L.down_w, L.down_s, L.down_b, hidden, inter, group,
                      down);
  return rc;
}

int osm_oracle_expert_mlp(const float* gate, const float* up, const float* down,
                          size_t hidden, size_t inter, const float* x,
                          float* out) {
  float* g = (float*)malloc(inter * sizeof(float));
  float* u = (float*)malloc(inter * sizeof(float));
  if (g == NULL || u == NULL) {
    free(g);
    free(u);
    return ERUNTIME;
  }
  int rc = osm_oracle_matvec_row_major(gate, inter, hidden, x, g);
  if (rc == OK) rc = osm_oracle_matvec_row_major(up, inter, hidden, x, u);
  if (rc == OK) rc = osm_oracle_swiglu_inplace(g, u, inter);
  if (rc == OK) rc = osm_oracle_matvec_row_major(down, hidden, inter, g, out);
  free(g);
  free(u);
  return rc;
}

/* shared_expert.cpp:11-87 */
int osm_oracle_shared_expert(const float* gate, const float* up,
                             const float* down, const float* scalar_gate,
                             size_t hidden, size_t inter, const float* x,
                             float* out, float* scale_out) {
  if (hidden == 0 || inter == 0) return EINVAL_ARG;
  int rc = osm_oracle_expert_mlp(gate, up, down, hidden, inter, x, out);
  if (rc != OK) return rc;
  float gate_logit = 0.0f;
  for (size_t i = 0; i < hidden; ++i) gate_logit += scalar_gate[i] * x[i];
  const float scale = osm_oracle_sigmoid(gate_logit);
  if (!isfinite(scale)) return ERUNTIME;
  for (size_t i = 0; i < hidden; ++i) out[i] *= scale;
  *scale_out = scale;
  return OK;
}

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
                         float* shared_scale) {
  float* logits = (float*)malloc(expert_count * sizeof(float));
  float* tmp = (float*)malloc(hidden_size * sizeof(float));
  if (logits == NULL || tmp == NULL) {
    free(logits);
    free(tmp);
    return ERUNTIME;
  }
  int rc = osm_oracle_route_qwen_top_k(hidden, router_weight, logit_bias,
                                       hidden_size, expert_count, top_k,
                                       norm_topk_prob, logits, experts, weights,
                                       selected_mass);
  for (size_t i = 0; rc == OK && i < hidden_size; ++i) out[i] = 0.0f;
  for (size_t k = 0; rc == OK && k < top_k; ++k) {
    const uint32_t e = experts[k];
    if (expert_gate[e] == NULL) {
      rc = ERUNTIME;
      break;
    }
    if (!isfinite(weights[k])) {
      rc = ERUNTIME;
      break;
    }
    rc = osm_oracle_expert_mlp(expert_gate[e], expert_up[e], expert_down[e],
                               hidden_size, inter, hidden, tmp);
    for (size_t i = 0; rc == OK && i < hidden_size; ++i)
      out[i] += weights[k] * tmp[i];
  }
  *shared_scale = 0.0f;
  if (rc == OK && shared_gate != NULL) {
    float s = 0.0f;
    rc = osm_oracle_expert_mlp(shared_gate, shared_up, shared_down,
                               hidden_size, shared_inter, hidden, tmp);
    if (rc == OK) {
      float gate_logit = 0.0f;
      for (size_t i = 0; i < hidden_size; ++i)
        gate_logit += scalar_gate[i] * hidden[i];
      s = osm_oracle_sigmoid(gate_logit);
      if (!isfinite(s)) rc = ERUNTIME;
    }
    for (size_t i = 0; rc == OK && i < hidden_size; ++i) out[i] += s * tmp[i];
    *shared_scale = s;
  }
  free(logits);
  free(tmp);
  return rc;
}

/* osm_oracle_moe_token over Q4 expert slots: routes, dequantises only the
 * picked experts (and the shared expert) with osm_oracle_dequant_slot, then
 * runs osm_oracle_moe_token on them -- the same arithmetic without holding
 * every expert in fp32.  slots: expert e at slots + e * slot_stride. */
int osm_oracle_moe_token_slots(const float* hidden, const float* router_weight,
                               const float* logit_bias, size_t hidden_size,
                               size_t expert_count, size_t top_k,
                               int norm_topk_prob, size_t inter,
                               const uint8_t* slots, size_t slot_stride,
                               const uint8_t* shared_slot,
                               const float* scalar_gate, float* out,
                               uint32_t* experts, float* weights,
                               float* selected_mass, float* shared_scale) {
  const size_t H = hidden_size, I = inter, per = 2 * I * H + H * I;
  float* logits = (float*)malloc(expert_count * sizeof(float));
  const float** g = (const float**)calloc(expert_count, sizeof(float*));
  const float** u = (const float**)calloc(expert_count, sizeof(float*));
  const float** d = (const float**)calloc(expert_count, sizeof(float*));
  float* deq = (float*)malloc((top_k + 1) * per * sizeof(float));
  int rc = (logits && g && u && d && deq) ? OK : ERUNTIME;
  if (rc == OK)
    rc = osm_oracle_route_qwen_top_k(hidden, router_weight, logit_bias, H,
                                     expert_count, top_k, norm_topk_prob,
                                     logits, experts, weights, selected_mass);
  for (size_t k = 0; rc == OK && k < top_k; ++k) {
    const uint32_t e = experts[k];
    if (g[e] != NULL) continue;
    float* base = deq + k * per;
    rc = osm_oracle_dequant_slot(slots + (size_t)e * slot_stride, H, I, 64,
                                 base, base + I * H, base + 2 * I * H);
    g[e] = base;
    u[e] = base + I * H;
    d[e] = base + 2 * I * H;
  }
  float* sh = deq + top_k * per;
  if (rc == OK && shared_slot != NULL)
    rc = osm_oracle_dequant_slot(shared_slot, H, I, 64, sh, sh + I * H,
                                 sh + 2 * I * H);
  if (rc == OK)
    rc = osm_oracle_moe_token(hidden, router_weight, logit_bias, H,
                              expert_count, top_k, norm_topk_prob, I, g, u, d,
                              shared_slot ? sh : NULL,
                              shared_slot ? sh + I * H : NULL,
                              shared_slot ? sh + 2 * I * H : NULL, scalar_gate,
                              I, out, experts, weights, selected_mass,
                              shared_scale);
  free(logits);
  free(g);
  free(u);
  free(d);
  free(deq);
  return rc;
}

int osm_oracle_add_residual(const float* residual, const float* branch,
                            float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = residual[i] + branch[i];
  return OK;
}

static uint64_t splitmix64(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

uint64_t osm_oracle_hash(uint64_t seed, uint64_t tensor, uint64_t index) {
  return splitmix64(splitmix64(seed ^ splitmix64(tensor)) + index);
}

void osm_oracle_gen_normal(uint64_t seed, uint64_t tensor, float sigma,
                           float* out, size_t n, size_t first_index) {
  const uint64_t base = splitmix64(seed ^ splitmix64(tensor));
  for (size_t i = 0; i < n; ++i) {
    const uint64_t h1 = splitmix64(base + (uint64_t)(first_index + i));
    const uint64_t h2 = splitmix64(h1);
    const double u1 = (double)((h1 >> 11) + 1) * 0x1.0p-53; /* (0, 1] */
    const double u2 = (double)(h2 >> 11) * 0x1.0p-53;       /* [0, 1) */
    const double r = sqrt(-2.0 * log(u1));
    const double v = r * cos(6.283185307179586 * u2);
    out[i] = (float)v * sigma;
  }
}

int osm_oracle_gen_expert_slot(uint64_t seed, uint64_t tensor_base, float sigma,
                               size_t hidden, size_t inter, size_t group,
                               uint8_t* slot) {
  osm_oracle_slot_layout L;
  osm_oracle_slot_layout_make(hidden, inter, group, &L);
  const size_t n = hidden * inter;
  float* v = (float*)malloc(n * sizeof(float));
  uint32_t* packed = (uint32_t*)malloc(n / 2);
  const size_t groups = n / group;
  float* s = (float*)malloc(groups * sizeof(float));
  float* b = (float*)malloc(groups * sizeof(float));
  uint16_t* h = (uint16_t*)malloc(groups * sizeof(uint16_t));
  int rc = (v && packed && s && b && h) ? OK : ERUNTIME;
  const size_t w_off[3] = {L.gate_w, L.up_w, L.down_w};
  const size_t s_off[3] = {L.gate_s, L.up_s, L.down_s};
  const size_t b_off[3] = {L.gate_b, L.up_b, L.down_b};
  for (int p = 0; p < 3 && rc == OK; ++p) {
    const size_t rows = p < 2 ? inter : hidden;
    const size_t cols = p < 2 ? hidden : inter;
    osm_oracle_gen_normal(seed, tensor_base + (uint64_t)p, sigma, v, n, 0);
    rc = osm_oracle_quantize_affine_q4_rows(v, rows, cols, group, packed, s, b);
    if (rc != OK) break;
    memcpy(slot + w_off[p], packed, n / 2);
    osm_oracle_bf16_narrow(s, h, groups);
    memcpy(slot + s_off[p], h, groups * 2);
    osm_oracle_bf16_narrow(b, h, groups);
    memcpy(slot + b_off[p], h, groups * 2);
  }
  free(v);
  free(packed);
  free(s);
  free(b);
  free(h);
  return rc;
}
