// RMSNorm rows on the device with the reference's sequential sum, so the
// result is bit-identical to cpu::rms_norm_inplace (osm_rms_norm with
// OSM_RMSNORM_EXACT).  As include/orbi/streammoe/backend/vulkan_rmsnorm.hpp
// of the reference.
#pragma once

#include <cstddef>
#include <span>
#include <string>
#include <vector>

#include "orbi/streammoe/backend/vulkan_compute_context.hpp"

namespace orbi::streammoe {

struct VulkanRmsNormResult {
  bool executed{};
  std::vector<float> values;
  std::string diagnostic;
};

// input row-major [rows, dim]; weight [dim] or empty (unit weight).
[[nodiscard]] VulkanRmsNormResult run_vulkan_rms_norm(
    VulkanComputeContext& context,
    std::span<const float> input,
    std::size_t rows,
    std::size_t dim,
    std::span<const float> weight,
    float eps) noexcept;

}  // namespace orbi::streammoe
