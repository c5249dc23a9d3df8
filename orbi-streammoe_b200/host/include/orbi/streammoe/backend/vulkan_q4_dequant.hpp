// MLX affine Q4 rows dequantised on the device (osm_q4_dequant: s q + b with a
// separate multiply and add, bit-exact with cpu::dequantize_affine_rows).  As
// include/orbi/streammoe/backend/vulkan_q4_dequant.hpp of the reference.
// Scales and biases arrive widened to fp32; the device kernels store them as
// bf16, so values that are not bf16-representable are refused.
#pragma once

#include <cstddef>
#include <cstdint>
#include <span>
#include <string>
#include <vector>

#include "orbi/streammoe/backend/vulkan_compute_context.hpp"

namespace orbi::streammoe {

struct VulkanQ4DequantResult {
  bool executed{};
  std::vector<float> values;
  std::string diagnostic;
};

[[nodiscard]] VulkanQ4DequantResult run_vulkan_q4_dequant(
    VulkanComputeContext& context,
    std::span<const std::uint32_t> packed,
    std::size_t rows,
    std::size_t packed_cols,
    std::span<const float> scales,
    std::span<const float> biases,
    std::size_t group_size) noexcept;

}  // namespace orbi::streammoe
