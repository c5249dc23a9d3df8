// One MoE expert resident in HBM: its qpack slot bytes (gate/up/down Q4 rows,
// bf16 scale and bias) in a slot of an expert slab, run by libosm_b200's
// expert kernels.  As include/orbi/streammoe/backend/vulkan_resident_expert.hpp
// of the reference; accounted_bytes() keeps the reference's accounting
// (packed words + fp32 metadata + activation buffers,
// src/backend/vulkan_resident_expert.cpp:258-280) so cache budgets mean the
// same.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <optional>
#include <span>
#include <string>
#include <vector>

#include "orbi/streammoe/backend/vulkan_compute_context.hpp"
#include "orbi/streammoe/backend/vulkan_float_buffer.hpp"
#include "orbi/streammoe/cache/expert_cache.hpp"
#include "orbi/streammoe/container/qpack.hpp"

struct osm_slab;

namespace orbi::streammoe {

struct VulkanResidentExpertResult {
  bool executed{};
  std::vector<float> values;
  std::string diagnostic;
};

class VulkanResidentExpert {
 public:
  VulkanResidentExpert();
  ~VulkanResidentExpert();

  VulkanResidentExpert(const VulkanResidentExpert&) = delete;
  VulkanResidentExpert& operator=(const VulkanResidentExpert&) = delete;
  VulkanResidentExpert(VulkanResidentExpert&&) noexcept;
  VulkanResidentExpert& operator=(VulkanResidentExpert&&) noexcept;

  // Uploads the entry's slot into its own one-slot slab; the entry is only
  // read during the call.
  [[nodiscard]] static std::optional<VulkanResidentExpert> create(
      VulkanComputeContext& context,
      const QpackReader& reader,
      const ExpertCacheEntry& entry,
      std::string* diagnostic = nullptr) noexcept;

  // The same into slot `slot` of a caller-owned slab of the expert's layout
  // (the resident expert cache's slab); not in the reference.
  [[nodiscard]] static std::optional<VulkanResidentExpert> create_in_slab(
      VulkanComputeContext& context,
      const QpackReader& reader,
      const ExpertCacheEntry& entry,
      osm_slab* slab,
      std::uint32_t slot,
      std::string* diagnostic = nullptr) noexcept;

  [[nodiscard]] bool valid() const noexcept;
  [[nodiscard]] std::size_t input_dim() const noexcept;
  [[nodiscard]] std::size_t intermediate_dim() const noexcept;
  [[nodiscard]] std::size_t output_dim() const noexcept;
  [[nodiscard]] std::size_t packed_weight_bytes() const noexcept;
  [[nodiscard]] std::size_t accounted_bytes() const noexcept;
  [[nodiscard]] std::uintptr_t native_device() const noexcept;

  // gate/up -> SwiGLU -> down for one input vector (host in, host out).
  [[nodiscard]] VulkanResidentExpertResult run(
      VulkanComputeContext& context,
      std::span<const float> x) noexcept;

  // The same from a device buffer into this expert's reusable output buffer.
  [[nodiscard]] VulkanBufferDispatchResult run_from_buffer(
      VulkanComputeContext& context,
      const VulkanFloatBuffer& x) noexcept;

  // Valid until this expert is moved, destroyed or run again.
  [[nodiscard]] const VulkanFloatBuffer* output_buffer() const noexcept;

  // The slab slot holding this expert (not in the reference).
  [[nodiscard]] std::int32_t slab_slot() const noexcept;
  // The slab holding this expert: the cache's, or one of its own (not in
  // the reference).
  [[nodiscard]] osm_slab* slab() const noexcept;

 private:
  struct Impl;
  explicit VulkanResidentExpert(std::unique_ptr<Impl> impl) noexcept;
  std::unique_ptr<Impl> impl_;
};

}  // namespace orbi::streammoe
