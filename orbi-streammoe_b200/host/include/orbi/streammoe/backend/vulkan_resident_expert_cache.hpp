// HBM expert cache: resident experts keyed (layer, expert) in the slots of one
// expert slab, filled from the host ExpertCache, evicting the entry with the
// smallest (use count, last use, key) when the accounted bytes would exceed
// the budget; use counts survive evictions.  Semantics of the reference's
// src/backend/vulkan_resident_expert_cache.cpp (get() fetches and uploads
// before it evicts, so a failed fetch changes no residency); public interface
// as include/orbi/streammoe/backend/vulkan_resident_expert_cache.hpp.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <span>
#include <string>

#include "orbi/streammoe/backend/vulkan_compute_context.hpp"
#include "orbi/streammoe/backend/vulkan_resident_expert.hpp"
#include "orbi/streammoe/cache/expert_cache.hpp"
#include "orbi/streammoe/container/qpack.hpp"

namespace orbi::streammoe {

struct VulkanResidentExpertCacheStats {
  std::size_t hits{};
  std::size_t misses{};
  std::size_t loads{};
  std::size_t evictions{};
  std::size_t resident_entries{};
  std::size_t resident_bytes{};
  std::size_t budget_bytes{};
};

class VulkanResidentExpertCache {
 public:
  // Throws std::invalid_argument for an invalid context or a zero budget.
  VulkanResidentExpertCache(
      VulkanComputeContext& context,
      const QpackReader& reader,
      ExpertCache& host_cache,
      std::size_t budget_bytes);
  ~VulkanResidentExpertCache();

  VulkanResidentExpertCache(const VulkanResidentExpertCache&) = delete;
  VulkanResidentExpertCache& operator=(const VulkanResidentExpertCache&) = delete;

  // Non-owning; valid until the entry is evicted.  nullptr + diagnostic on
  // failure.
  [[nodiscard]] VulkanResidentExpert* get(
      std::uint32_t layer,
      std::uint32_t expert,
      std::string* diagnostic = nullptr) noexcept;

  [[nodiscard]] VulkanResidentExpertResult run(
      std::uint32_t layer,
      std::uint32_t expert,
      std::span<const float> x) noexcept;

  [[nodiscard]] bool contains(
      std::uint32_t layer,
      std::uint32_t expert) const noexcept;

  [[nodiscard]] VulkanResidentExpertCacheStats stats() const noexcept;
  [[nodiscard]] ExpertCacheStats host_stats() const noexcept;

  // The slab every resident expert lives in (not in the reference).
  [[nodiscard]] osm_slab* slab() const noexcept;
  // The compute context the cache uploads into (not in the reference).
  [[nodiscard]] VulkanComputeContext& context() const noexcept;

 private:
  struct Impl;
  std::unique_ptr<Impl> impl_;
};

}  // namespace orbi::streammoe
