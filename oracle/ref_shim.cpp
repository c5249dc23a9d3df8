// ref_shim.cpp -- extern "C" access to the reference's own CPU path.
//
// TEST INFRASTRUCTURE ONLY.  Compiled (by oracle/Makefile) together with the
// reference's sources where they lie (src/cpu/reference_ops.cpp,
// src/model/qwen_router.cpp, src/model/shared_expert.cpp,
// src/cache/expert_cache.cpp, src/conversion/single_expert_pilot.cpp, ...)
// into oracle/_ref/libosm_ref.so.  It pins the C restatement
// (osm_oracle.c) bit-for-bit and is the CPU baseline timed by bench.py
// ("cpu_baseline.kind": "reference").  Nothing here is shipped.
#include <chrono>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <optional>
#include <span>
#include <stdexcept>
#include <thread>
#include <vector>

#include "orbi/streammoe/cache/expert_cache.hpp"
#include "orbi/streammoe/conversion/single_expert_pilot.hpp"
#include "orbi/streammoe/cpu/reference_ops.hpp"
#include "orbi/streammoe/model/qwen_router.hpp"
#include "orbi/streammoe/model/shared_expert.hpp"

namespace osm = orbi::streammoe;

namespace {

template <typename F>
int guarded(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::invalid_argument&) {
    return -1;
  } catch (const std::exception&) {
    return -2;
  } catch (...) {
    return -2;
  }
}

// Biased-router harness: matvec_row_major, add the bias, route_top_k with
// normalize=false, then the renorm steps of qwen_router.cpp:68-91.  With a
// null bias it is route_qwen_top_k_cpu itself.
void route(const float* hidden, const float* router_weight,
           const float* logit_bias, std::size_t H, std::size_t E,
           std::size_t k, bool norm, float* logits_out, std::uint32_t* ids,
           float* weights, float* mass_out) {
  const osm::QwenRouterConfig cfg{
      .hidden_size = H, .expert_count = E, .top_k = k, .norm_topk_prob = norm};
  if (logit_bias == nullptr) {
    const auto r = osm::route_qwen_top_k_cpu(
        std::span<const float>(hidden, H),
        std::span<const float>(router_weight, E * H), cfg);
    for (std::size_t e = 0; e < E; ++e) logits_out[e] = r.logits[e];
    for (std::size_t i = 0; i < k; ++i) {
      ids[i] = r.picks[i].expert;
      weights[i] = r.picks[i].weight;
    }
    *mass_out = r.selected_probability_mass;
    return;
  }
  auto logits = osm::cpu::matvec_row_major(
      std::span<const float>(router_weight, E * H), E, H,
      std::span<const float>(hidden, H));
  for (std::size_t e = 0; e < E; ++e) logits[e] += logit_bias[e];
  const auto raw = osm::cpu::route_top_k(logits, k, false);
  float mass = 0.0F;
  for (const auto& p : raw) mass += p.probability;
  if (!(mass > 0.0F) || !std::isfinite(mass))
    throw std::runtime_error("router mass");
  for (std::size_t e = 0; e < E; ++e) logits_out[e] = logits[e];
  for (std::size_t i = 0; i < k; ++i) {
    ids[i] = raw[i].expert;
    weights[i] = norm ? raw[i].probability / mass : raw[i].probability;
  }
  *mass_out = mass;
}

class ShimStorage final : public osm::ExpertStorage {
 public:
  explicit ShimStorage(std::size_t stride) : stride_(stride) {}
  std::size_t expert_stride_bytes() const noexcept override { return stride_; }
  void read_experts(std::span<osm::ExpertReadRequest> requests) override {
    ++batch_calls;
    if (fail_next) {
      fail_next = false;
      throw std::runtime_error("synthetic read failure");
    }
    for (auto& r : requests)
      for (std::size_t i = 0; i < stride_; ++i)
        r.destination[i] = static_cast<std::byte>(
            (r.id.layer * 37U + r.id.expert * 11U + i) & 0xFFU);
  }
  bool fail_next{};
  std::size_t batch_calls{};

 private:
  std::size_t stride_;
};

struct ShimCache {
  ShimStorage storage;
  osm::ExpertCache cache;
  ShimCache(std::size_t stride, std::size_t budget, std::size_t min_slots)
      : storage(stride), cache(storage, budget, min_slots) {}
};

}  // namespace

extern "C" {

int osm_ref_dequantize_affine_rows(const std::uint32_t* packed, std::size_t rows,
                                   std::size_t packed_cols, const float* scales,
                                   const float* biases, std::uint32_t bits,
                                   std::uint32_t group, float* out) {
  return guarded([&] {
    const std::size_t per_word = bits == 0 ? 1 : 32U / bits;
    const std::size_t groups =
        group == 0 ? 0 : rows * (packed_cols * per_word) / group;
    const auto v = osm::cpu::dequantize_affine_rows(
        std::span<const std::uint32_t>(packed, rows * packed_cols), rows,
        packed_cols, std::span<const float>(scales, groups),
        std::span<const float>(biases, groups),
        osm::cpu::AffineQuantSpec{.bits = bits, .group_size = group});
    std::memcpy(out, v.data(), v.size() * sizeof(float));
  });
}

int osm_ref_matvec_row_major(const float* w, std::size_t out_dim,
                             std::size_t in_dim, const float* x, float* out) {
  return guarded([&] {
    const auto v = osm::cpu::matvec_row_major(
        std::span<const float>(w, out_dim * in_dim), out_dim, in_dim,
        std::span<const float>(x, in_dim));
    std::memcpy(out, v.data(), v.size() * sizeof(float));
  });
}

int osm_ref_rms_norm_inplace(float* values, std::size_t rows, std::size_t dim,
                             const float* weight, float eps) {
  return guarded([&] {
    osm::cpu::rms_norm_inplace(
        std::span<float>(values, rows * dim), rows, dim,
        weight ? std::span<const float>(weight, dim) : std::span<const float>(),
        eps);
  });
}

int osm_ref_softmax_inplace(float* values, std::size_t n) {
  return guarded(
      [&] { osm::cpu::softmax_inplace(std::span<float>(values, n)); });
}

int osm_ref_route_top_k(const float* logits, std::size_t n, std::size_t k,
                        int normalize, std::uint32_t* ids, float* probs) {
  return guarded([&] {
    const auto picks = osm::cpu::route_top_k(std::span<const float>(logits, n),
                                             k, normalize != 0);
    for (std::size_t i = 0; i < picks.size(); ++i) {
      ids[i] = picks[i].expert;
      probs[i] = picks[i].probability;
    }
  });
}

float osm_ref_sigmoid(float v) { return osm::cpu::sigmoid(v); }
float osm_ref_silu(float v) { return osm::cpu::silu(v); }

int osm_ref_swiglu_inplace(float* gate, const float* up, std::size_t n) {
  return guarded([&] {
    osm::cpu::swiglu_inplace(std::span<float>(gate, n),
                             std::span<const float>(up, n));
  });
}

int osm_ref_route_qwen_top_k(const float* hidden, const float* router_weight,
                             const float* logit_bias, std::size_t H,
                             std::size_t E, std::size_t k, int norm,
                             float* logits_out, std::uint32_t* ids,
                             float* weights, float* mass) {
  return guarded([&] {
    route(hidden, router_weight, logit_bias, H, E, k, norm != 0, logits_out,
          ids, weights, mass);
  });
}

int osm_ref_quantize_affine_q4_rows(const float* values, std::size_t rows,
                                    std::size_t cols, std::size_t group,
                                    std::uint32_t* packed, float* scales,
                                    float* biases) {
  return guarded([&] {
    std::vector<float> v(values, values + rows * cols);
    const auto q = osm::quantize_affine_q4_rows(v, rows, cols, group);
    std::memcpy(packed, q.packed.data(), q.packed.size() * 4);
    std::memcpy(scales, q.scales.data(), q.scales.size() * 4);
    std::memcpy(biases, q.biases.data(), q.biases.size() * 4);
  });
}

int osm_ref_shared_expert(const float* gate, const float* up,
                          const float* down, const float* scalar_gate,
                          std::size_t H, std::size_t I, const float* x,
                          float* out, float* scale) {
  const auto r = osm::run_shared_expert_cpu(
      std::span<const float>(x, H),
      osm::SharedExpertWeights{
          .gate_proj = std::span<const float>(gate, I * H),
          .up_proj = std::span<const float>(up, I * H),
          .down_proj = std::span<const float>(down, H * I),
          .scalar_gate = std::span<const float>(scalar_gate, H)},
      osm::SharedExpertConfig{.hidden_size = H, .intermediate_size = I});
  if (!r.executed) return -2;
  std::memcpy(out, r.values.data(), H * sizeof(float));
  *scale = r.scalar_gate;
  return 0;
}

// One token of the sparse MoE on the reference's CPU primitives, in the
// accumulation order of routed_moe.cpp:13-92 (pick order) followed by the
// shared expert (routed_moe.cpp:381-404 adds s*out last).
static int moe_token(const float* x, const float* router_weight,
                     const float* bias, std::size_t H, std::size_t E,
                     std::size_t k, int norm, std::size_t I,
                     const float* const* eg, const float* const* eu,
                     const float* const* ed, const float* sg, const float* su,
                     const float* sd, const float* scalar_gate, std::size_t SI,
                     float* out, std::uint32_t* ids, float* weights,
                     float* mass, float* shared_scale) {
  return guarded([&] {
    std::vector<float> logits(E);
    route(x, router_weight, bias, H, E, k, norm != 0, logits.data(), ids,
          weights, mass);
    const std::span<const float> xs(x, H);
    std::vector<float> acc(H, 0.0F);
    for (std::size_t p = 0; p < k; ++p) {
      const auto e = ids[p];
      if (eg[e] == nullptr) throw std::runtime_error("expert not provided");
      auto g = osm::cpu::matvec_row_major(std::span<const float>(eg[e], I * H),
                                          I, H, xs);
      const auto u = osm::cpu::matvec_row_major(
          std::span<const float>(eu[e], I * H), I, H, xs);
      osm::cpu::swiglu_inplace(g, u);
      const auto y = osm::cpu::matvec_row_major(
          std::span<const float>(ed[e], H * I), H, I, g);
      for (std::size_t i = 0; i < H; ++i) acc[i] += weights[p] * y[i];
    }
    *shared_scale = 0.0F;
    if (sg != nullptr) {
      const auto r = osm::run_shared_expert_cpu(
          xs,
          osm::SharedExpertWeights{
              .gate_proj = std::span<const float>(sg, SI * H),
              .up_proj = std::span<const float>(su, SI * H),
              .down_proj = std::span<const float>(sd, H * SI),
              .scalar_gate = std::span<const float>(scalar_gate, H)},
          osm::SharedExpertConfig{.hidden_size = H, .intermediate_size = SI});
      if (!r.executed) throw std::runtime_error(r.diagnostic);
      for (std::size_t i = 0; i < H; ++i) acc[i] += r.values[i];
      *shared_scale = r.scalar_gate;
    }
    std::memcpy(out, acc.data(), H * sizeof(float));
  });
}

int osm_ref_moe_token(const float* x, const float* router_weight,
                      const float* bias, std::size_t H, std::size_t E,
                      std::size_t k, int norm, std::size_t I,
                      const float* const* eg, const float* const* eu,
                      const float* const* ed, const float* sg, const float* su,
                      const float* sd, const float* scalar_gate, std::size_t SI,
                      float* out, std::uint32_t* ids, float* weights,
                      float* mass, float* shared_scale) {
  return moe_token(x, router_weight, bias, H, E, k, norm, I, eg, eu, ed, sg,
                   su, sd, scalar_gate, SI, out, ids, weights, mass,
                   shared_scale);
}

// Token-parallel CPU baseline: B tokens split in contiguous slices over
// `threads` std::threads (tokens are independent).  Returns the wall time of
// the whole batch in seconds through *seconds; 0 on success.
int osm_ref_moe_batch(const float* x, std::size_t B, const float* router_weight,
                      const float* bias, std::size_t H, std::size_t E,
                      std::size_t k, int norm, std::size_t I,
                      const float* const* eg, const float* const* eu,
                      const float* const* ed, const float* sg, const float* su,
                      const float* sd, const float* scalar_gate, std::size_t SI,
                      float* out, std::uint32_t* ids, float* weights,
                      int threads, double* seconds) {
  if (threads < 1) threads = 1;
  std::vector<int> rc(static_cast<std::size_t>(threads), 0);
  const auto t0 = std::chrono::steady_clock::now();
  auto work = [&](int t) {
    const std::size_t lo = B * static_cast<std::size_t>(t) / threads;
    const std::size_t hi = B * static_cast<std::size_t>(t + 1) / threads;
    for (std::size_t b = lo; b < hi && rc[t] == 0; ++b) {
      float mass = 0.0F, ss = 0.0F;
      rc[t] = moe_token(x + b * H, router_weight, bias, H, E, k, norm, I, eg,
                        eu, ed, sg, su, sd, scalar_gate, SI, out + b * H,
                        ids + b * k, weights + b * k, &mass, &ss);
    }
  };
  if (threads == 1) {
    work(0);
  } else {
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t) pool.emplace_back(work, t);
    for (auto& th : pool) th.join();
  }
  *seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0)
                 .count();
  for (int v : rc)
    if (v != 0) return v;
  return 0;
}

// The reference's host expert cache (src/cache/expert_cache.cpp) behind a
// synthetic storage, so the drop-in cache's slot policy can be compared with
// it fetch by fetch.
void* osm_ref_cache_create(std::size_t stride, std::size_t budget,
                           std::size_t min_slots) {
  try {
    return new ShimCache(stride, budget, min_slots);
  } catch (...) {
    return nullptr;
  }
}

void osm_ref_cache_destroy(void* c) { delete static_cast<ShimCache*>(c); }

void osm_ref_cache_fail_next(void* c) {
  static_cast<ShimCache*>(c)->storage.fail_next = true;
}

// Fetch `n` experts of `layer`; slots_out[i] = slot of experts[i].  Returns
// 0, or -2 when the reference throws (storage failure, oversized batch).
int osm_ref_cache_fetch(void* c, std::uint32_t layer,
                        const std::uint32_t* experts, std::size_t n,
                        std::size_t* slots_out) {
  auto* sc = static_cast<ShimCache*>(c);
  return guarded([&] {
    const auto entries =
        sc->cache.fetch(layer, std::span<const std::uint32_t>(experts, n));
    for (std::size_t i = 0; i < entries.size(); ++i)
      slots_out[i] = entries[i].slot;
  });
}

// Resident slot of (layer, expert) or -1.
long long osm_ref_cache_resident_slot(void* c, std::uint32_t layer,
                                      std::uint32_t expert) {
  const auto s =
      static_cast<ShimCache*>(c)->cache.resident_slot(layer, expert);
  return s.has_value() ? static_cast<long long>(*s) : -1;
}

// stats: hits, misses, allocated_slots, capacity_slots, logical_bytes,
// budget_bytes, storage batch calls.
void osm_ref_cache_stats(void* c, std::size_t* out7) {
  auto* sc = static_cast<ShimCache*>(c);
  const auto s = sc->cache.stats();
  out7[0] = s.hits;
  out7[1] = s.misses;
  out7[2] = s.allocated_slots;
  out7[3] = s.capacity_slots;
  out7[4] = s.logical_bytes;
  out7[5] = s.budget_bytes;
  out7[6] = sc->storage.batch_calls;
}

}  // extern "C"
