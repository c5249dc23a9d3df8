// The reference's routed-MoE entry points (include/orbi/streammoe/model/
// routed_moe.hpp of ingeniusvictor/orbi-streammoe) with their signatures,
// argument checks and diagnostics, built for the B200 in place of the
// reference's src/model/routed_moe.cpp:
//
//   * routing runs on the device: osm_moe_route_logits over a router layer
//     the compute context keeps per router weight, on the reference's own
//     arithmetic (sequential fp32 logits, softmax with a sequential sum,
//     stable top-k, lower id first on ties), so logits, picks, weights and
//     the selected mass are those of route_qwen_top_k_cpu
//     (src/model/qwen_router.cpp:11-94); only the k picks and the E logits
//     come back to the host;
//   * the routed experts are made resident through VulkanResidentExpertCache
//     in pick order, one get() per pick as the reference does, and when all
//     of them sit in the cache's slab they run as one osm_moe_experts call
//     (the decode kernels: gate/up + SwiGLU + down for every pick, with the
//     weighted combine in pick order, one fp32 multiply and one add per pick,
//     from zero);
//   * an expert outside the slab (another geometry), or a pick a later
//     pick's load evicted, runs on its own and is added by
//     osm_weighted_accumulate, which is the reference's order too.
//
// The shared expert (run_qwen_sparse_moe_vulkan_accum) is added last with
// its scalar gate, as in the reference (src/model/routed_moe.cpp:374-405).
#include "orbi/streammoe/model/routed_moe.hpp"

#include <bit>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <exception>
#include <limits>
#include <optional>
#include <stdexcept>
#include <string>
#include <vector>

#include "orbi/streammoe/backend/vulkan_float_buffer.hpp"
#include "orbi/streammoe/backend/vulkan_weighted_accumulate.hpp"
#include "osm_b200.h"
#include "osm_host_util.hpp"

namespace orbi::streammoe {
namespace {

// The argument contract of route_qwen_top_k_cpu (src/model/qwen_router.cpp:
// 15-58), thrown as it throws.  The router weight's values are checked when
// its device layer is made (osm_layer_create rejects a non-finite value with
// the same message) and compared with that checked copy at every later use.
void check_route_args(std::span<const float> hidden, std::span<const float> router_weight,
                      const QwenRouterConfig& c) {
  if (c.hidden_size == 0U || c.expert_count == 0U || c.top_k == 0U)
    throw std::invalid_argument("qwen router: dimensions and top_k must be non-zero");
  if (c.top_k > c.expert_count)
    throw std::invalid_argument("qwen router: top_k cannot exceed expert_count");
  if (c.expert_count > static_cast<std::size_t>(std::numeric_limits<std::uint32_t>::max()))
    throw std::invalid_argument("qwen router: expert_count exceeds routed-expert id range");
  if (hidden.size() != c.hidden_size)
    throw std::invalid_argument("qwen router: hidden vector size mismatch");
  if (c.expert_count > std::numeric_limits<std::size_t>::max() / c.hidden_size)
    throw std::invalid_argument("qwen router: weight shape overflows size_t");
  if (router_weight.size() != c.expert_count * c.hidden_size)
    throw std::invalid_argument("qwen router: router weight size mismatch");
  for (const float v : hidden)
    if (!std::isfinite(v))
      throw std::invalid_argument("qwen router: hidden vector contains non-finite value");
  if (c.hidden_size > std::numeric_limits<std::uint32_t>::max())
    throw std::invalid_argument("qwen router: hidden size exceeds the device router");
}

// One routing on the device.  `route` keeps the picks on the device for the
// expert call: ids [k] (u32) then weights [k], then the mass.
struct DeviceRoute {
  osm_layer* router = nullptr;
  std::optional<VulkanFloatBuffer> route;
  QwenRouterResult result;

  const std::uint32_t* ids_dev() const {
    return reinterpret_cast<const std::uint32_t*>(route->device_data());
  }
  const float* weights_dev() const { return route->device_data() + result.picks.size(); }
};

// Routes the hidden vector already uploaded to `x`; throws on failure, as
// route_qwen_top_k_cpu does.
DeviceRoute route_on_device(VulkanComputeContext& context, const VulkanFloatBuffer& x,
                            std::span<const float> hidden, std::span<const float> router_weight,
                            const QwenRouterConfig& c) {
  check_route_args(hidden, router_weight, c);
  DeviceRoute r;
  std::string d;
  r.router = context.router_layer(router_weight, static_cast<std::uint32_t>(c.hidden_size),
                                  static_cast<std::uint32_t>(c.expert_count),
                                  static_cast<std::uint32_t>(c.top_k), c.norm_topk_prob, &d);
  if (!r.router) throw std::invalid_argument(d);
  const std::size_t E = c.expert_count, k = c.top_k;
  auto logits = VulkanFloatBuffer::create(context, E, &d);
  if (!logits) throw std::runtime_error("device router: logits buffer: " + d);
  r.route = VulkanFloatBuffer::create(context, 2 * k + 1, &d);
  if (!r.route) throw std::runtime_error("device router: route buffer: " + d);
  osm_context* ctx = context.osm();
  std::uint32_t status = 0;
  osm_context_status(ctx, &status, nullptr);  // start this call's status word from zero
  float* rd = r.route->device_data();
  int rc = osm_moe_route_logits(r.router, x.device_data(), 1, logits->device_data(),
                                reinterpret_cast<std::uint32_t*>(rd), rd + k, rd + 2 * k);
  if (rc != OSM_OK) throw std::runtime_error(osmh::err(ctx, rc, "device router launch failed"));
  auto lv = logits->download(&d);  // synchronises the stream
  auto rv = r.route->download(&d);
  if (!lv || !rv) throw std::runtime_error("device router: download failed: " + d);
  osm_context_status(ctx, &status, nullptr);
  if (status & 0x3u)
    throw std::runtime_error("device router: non-finite logits or softmax mass (status " +
                             std::to_string(status) + ")");
  r.result.logits = std::move(*lv);
  r.result.picks.resize(k);
  for (std::size_t j = 0; j < k; ++j) {
    r.result.picks[j].expert = std::bit_cast<std::uint32_t>((*rv)[j]);
    r.result.picks[j].weight = (*rv)[k + j];
  }
  r.result.selected_probability_mass = (*rv)[2 * k];
  return r;
}

// Uploads `hidden` into a new device buffer; nullopt with a diagnostic.
std::optional<VulkanFloatBuffer> upload(VulkanComputeContext& context, std::span<const float> v,
                                        std::string* d) {
  auto b = VulkanFloatBuffer::create(context, v.size(), d);
  if (b && !b->upload(v, d)) return std::nullopt;
  return b;
}

// A pick held in the cache's slab, waiting for the one expert call.
struct SlabPick {
  std::uint32_t expert;
  std::uint32_t slot;
  float weight;
};

// Makes every pick resident through `cache` (one get() per pick, in pick
// order) and adds weight x expert(x) of each to `acc`, in pick order.  `acc`
// is made (zeroed, the first expert's output size) when the caller has not
// made it.  False with *diag set, worded with `who`, on the first failure.
bool run_routed(VulkanComputeContext& context, VulkanResidentExpertCache& cache,
                std::uint32_t layer, const DeviceRoute& route, const VulkanFloatBuffer& x,
                std::optional<VulkanFloatBuffer>& acc, const std::string& who,
                std::string* diag) {
  osm_context* ctx = context.osm();
  const auto& picks = route.result.picks;
  std::vector<SlabPick> pending;
  bool fused = true;  // every pick so far waits in the slab
  std::optional<VulkanFloatBuffer> tmp;
  std::string d;

  // Runs the waiting picks one by one from their slots.
  auto flush = [&]() -> bool {
    if (pending.empty()) return true;
    osm_slab* slab = cache.slab();
    osm_expert_layout L{};
    if (osm_slab_layout(slab, &L) != OSM_OK) {
      *diag = who + " routed expert slab is missing";
      return false;
    }
    if (!tmp) tmp = VulkanFloatBuffer::create(context, acc->size(), &d);
    if (!tmp) {
      *diag = who + " expert output allocation failed: " + d;
      return false;
    }
    for (const auto& p : pending) {
      int rc = osm_expert_forward(ctx, osm_slab_slot_ptr(slab, p.slot), &L, x.device_data(), 1,
                                  tmp->device_data());
      if (rc == OSM_OK)
        rc = osm_weighted_accumulate(ctx, tmp->device_data(), p.weight, acc->device_data(),
                                     acc->size());
      if (rc != OSM_OK) {
        *diag = who + " routed expert " + std::to_string(p.expert) +
                " execution failed: " + osmh::err(ctx, rc, "expert kernels");
        return false;
      }
    }
    pending.clear();
    return true;
  };

  for (const auto& pick : picks) {
    if (!std::isfinite(pick.weight)) {
      *diag = who + " encountered non-finite routing weight";
      return false;
    }
    auto* resident = cache.get(layer, pick.expert, &d);
    if (resident == nullptr) {
      *diag = who + " routed expert " + std::to_string(pick.expert) + " load failed: " + d;
      return false;
    }
    if (!acc) {
      acc = VulkanFloatBuffer::create(context, resident->output_dim(), &d);
      if (!acc || !acc->upload(std::vector<float>(resident->output_dim(), 0.0F), &d)) {
        *diag = who + " accumulator allocation failed: " + d;
        return false;
      }
    }
    if (resident->input_dim() != x.size() || resident->output_dim() != acc->size()) {
      *diag = who + " routed expert geometry mismatch";
      return false;
    }
    // A load may have evicted a waiting pick of this call.  Its slot keeps
    // its bytes until the next load (a newcomer is uploaded into a slot that
    // was free before the evictions), so the waiting picks run now.
    for (const auto& p : pending)
      if (!cache.contains(layer, p.expert)) fused = false;
    if (!fused && !flush()) return false;
    osm_slab* slab = cache.slab();
    if (slab != nullptr && resident->slab() == slab && resident->slab_slot() >= 0) {
      pending.push_back({pick.expert, static_cast<std::uint32_t>(resident->slab_slot()),
                         pick.weight});
      if (!fused && !flush()) return false;
      continue;
    }
    // an expert in a slab of its own (another geometry): run it here
    fused = false;
    if (!flush()) return false;
    const auto dispatch = resident->run_from_buffer(context, x);
    const auto* out = resident->output_buffer();
    if (!dispatch.executed || out == nullptr) {
      *diag = who + " routed expert " + std::to_string(pick.expert) +
              " execution failed: " + dispatch.diagnostic;
      return false;
    }
    const auto a = run_vulkan_weighted_accumulate(context, *out, pick.weight, *acc);
    if (!a.executed) {
      *diag = who + " routed accumulation failed: " + a.diagnostic;
      return false;
    }
  }
  if (fused && !pending.empty() && pending.size() == picks.size()) {
    // every pick in the slab: one expert call, combine in pick order from zero
    std::vector<std::int32_t> slot_of(route.result.logits.size(), -1);
    for (const auto& p : pending) slot_of[p.expert] = static_cast<std::int32_t>(p.slot);
    if (osm_layer_bind_slab(route.router, cache.slab(), slot_of.data()) == OSM_OK) {
      std::uint32_t status = 0;
      osm_context_status(ctx, &status, nullptr);
      int rc = osm_moe_experts(route.router, x.device_data(), 1, route.ids_dev(),
                               route.weights_dev(), acc->device_data(), nullptr, nullptr, 0);
      if (rc == OSM_OK) rc = osm_context_synchronize(ctx);
      if (rc == OSM_OK) rc = osm_context_status(ctx, &status, nullptr);
      if (rc != OSM_OK || (status & 0x1Cu)) {
        *diag = who + " routed experts failed: " +
                (rc != OSM_OK ? osmh::err(ctx, rc, "expert kernels")
                              : "device status " + std::to_string(status));
        return false;
      }
      pending.clear();
      return true;
    }
  }
  return flush();
}

// The final output: downloaded, non-empty and (when asked) finite.
bool finish(VulkanFloatBuffer& acc, std::vector<float>* values, bool check_finite,
            const std::string& who, std::string* diag) {
  std::string d;
  auto v = acc.download(&d);
  if (!v) {
    *diag = who + " final output download failed: " + d;
    return false;
  }
  if (v->empty()) {
    *diag = who + " produced no output";
    return false;
  }
  for (const float f : *v)
    if (check_finite && !std::isfinite(f)) {
      *diag = who + " produced non-finite output";
      return false;
    }
  *values = std::move(*v);
  return true;
}

// Shared body of the two routed-only entry points.
RoutedMoeResult routed_only(VulkanComputeContext& context, VulkanResidentExpertCache& cache,
                            std::uint32_t layer, std::span<const float> hidden,
                            std::span<const float> router_weight, QwenRouterConfig config,
                            const std::string& who, bool check_finite,
                            const char* done) noexcept {
  RoutedMoeResult result;
  if (!context.valid()) {
    result.diagnostic = who + " requires a valid compute context";
    return result;
  }
  if (cache.context().native_device() != context.native_device()) {
    result.diagnostic = who + " expert cache belongs to another device";
    return result;
  }
  try {
    std::string d;
    auto x = upload(context, hidden, &d);
    if (!x) {
      result.diagnostic = who + " hidden upload failed: " + d;
      return result;
    }
    auto route = route_on_device(context, *x, hidden, router_weight, config);
    result.routing = route.result;
    if (result.routing.picks.empty()) {
      result.diagnostic = who + " selected no experts";
      return result;
    }
    std::optional<VulkanFloatBuffer> acc;
    if (!run_routed(context, cache, layer, route, *x, acc, who, &result.diagnostic)) return result;
    if (!finish(*acc, &result.values, check_finite, who, &result.diagnostic)) return result;
    result.executed = true;
    result.diagnostic = done;
    return result;
  } catch (const std::exception& e) {
    result.diagnostic = who + " exception: " + e.what();
    result.values.clear();
    return result;
  } catch (...) {
    result.diagnostic = who + " encountered an unknown exception";
    result.values.clear();
    return result;
  }
}

}  // namespace

// src/model/routed_moe.cpp:13-93 of the reference: the same result, with the
// routing and the weighted sum on the device of the cache's context.
RoutedMoeResult run_weighted_routed_moe(VulkanResidentExpertCache& expert_cache,
                                        std::uint32_t layer, std::span<const float> hidden,
                                        std::span<const float> router_weight,
                                        QwenRouterConfig router_config) noexcept {
  return routed_only(expert_cache.context(), expert_cache, layer, hidden, router_weight,
                     router_config, "routed MoE", true,
                     "weighted routed MoE executed on the device router and resident expert cache");
}

// src/model/routed_moe.cpp:95-252 of the reference.
RoutedMoeResult run_weighted_routed_moe_vulkan_accum(VulkanComputeContext& context,
                                                     VulkanResidentExpertCache& expert_cache,
                                                     std::uint32_t layer,
                                                     std::span<const float> hidden,
                                                     std::span<const float> router_weight,
                                                     QwenRouterConfig router_config) noexcept {
  return routed_only(context, expert_cache, layer, hidden, router_weight, router_config,
                     "device-accumulated routed MoE", false,
                     "routed MoE accumulated on the device from one uploaded hidden vector");
}

// src/model/routed_moe.cpp:254-431 of the reference: routed Top-K weighted
// sum plus the sigmoid-gated shared expert in one device accumulator.
QwenSparseMoeResult run_qwen_sparse_moe_vulkan_accum(VulkanComputeContext& context,
                                                     VulkanResidentExpertCache& expert_cache,
                                                     VulkanResidentSharedExpert& shared_expert,
                                                     std::uint32_t layer,
                                                     std::span<const float> hidden,
                                                     std::span<const float> router_weight,
                                                     QwenRouterConfig router_config) noexcept {
  const std::string who = "Qwen sparse MoE";
  QwenSparseMoeResult result;
  if (!context.valid()) {
    result.diagnostic = who + " requires a valid compute context";
    return result;
  }
  if (!shared_expert.valid() || shared_expert.native_device() != context.native_device()) {
    result.diagnostic = who + " shared expert is invalid or belongs to another device";
    return result;
  }
  if (shared_expert.input_dim() != hidden.size() || shared_expert.output_dim() != hidden.size()) {
    result.diagnostic = who + " shared expert geometry does not match hidden size";
    return result;
  }
  if (expert_cache.context().native_device() != context.native_device()) {
    result.diagnostic = who + " expert cache belongs to another device";
    return result;
  }
  try {
    std::string d;
    auto x = upload(context, hidden, &d);
    if (!x) {
      result.diagnostic = who + " hidden upload failed: " + d;
      return result;
    }
    auto route = route_on_device(context, *x, hidden, router_weight, router_config);
    result.routing = route.result;
    if (result.routing.picks.empty()) {
      result.diagnostic = who + " selected no routed experts";
      return result;
    }
    std::optional<VulkanFloatBuffer> acc =
        upload(context, std::vector<float>(shared_expert.output_dim(), 0.0F), &d);
    if (!acc) {
      result.diagnostic = who + " accumulator allocation failed: " + d;
      return result;
    }
    if (!run_routed(context, expert_cache, layer, route, *x, acc, who, &result.diagnostic))
      return result;
    const auto shared = shared_expert.run_from_buffer(context, *x);
    if (!shared.executed) {
      result.diagnostic = who + " shared expert execution failed: " + shared.diagnostic;
      return result;
    }
    const auto scale = shared_expert.scalar_scale(hidden, &d);
    if (!scale) {
      result.diagnostic = who + " shared scalar gate failed: " + d;
      return result;
    }
    const auto* shared_out = shared_expert.output_buffer();
    if (shared_out == nullptr) {
      result.diagnostic = who + " shared expert exposed no output buffer";
      return result;
    }
    const auto a = run_vulkan_weighted_accumulate(context, *shared_out, *scale, *acc);
    if (!a.executed) {
      result.diagnostic = who + " shared accumulation failed: " + a.diagnostic;
      return result;
    }
    auto v = acc->download(&d);
    if (!v) {
      result.diagnostic = who + " final output download failed: " + d;
      return result;
    }
    result.executed = true;
    result.shared_gate = *scale;
    result.values = std::move(*v);
    result.diagnostic = who + " combined routed and shared experts in one device accumulator";
    return result;
  } catch (const std::exception& e) {
    result.diagnostic = who + " exception: " + e.what();
    result.values.clear();
    return result;
  } catch (...) {
    result.diagnostic = who + " encountered an unknown exception";
    result.values.clear();
    return result;
  }
}

}  // namespace orbi::streammoe
