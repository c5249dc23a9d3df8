// y = W x from MLX affine Q4 rows on the device (osm_q4_gemv).  As
// include/orbi/streammoe/backend/vulkan_q4_gemv.hpp of the reference.
// fp32 scales/biases must be bf16-representable (the device format).
#pragma once

#include <cstddef>
#include <cstdint>
#include <span>
#include <string>
#include <vector>

#include "orbi/streammoe/backend/vulkan_compute_context.hpp"
#include "orbi/streammoe/backend/vulkan_float_buffer.hpp"
#include "orbi/streammoe/backend/vulkan_q4_weights.hpp"

namespace orbi::streammoe {

struct VulkanQ4GemvResult {
  bool executed{};
  std::vector<float> values;
  std::string diagnostic;
};

[[nodiscard]] VulkanQ4GemvResult run_vulkan_q4_gemv(
    VulkanComputeContext& context,
    std::span<const std::uint32_t> packed,
    std::size_t out_dim,
    std::size_t packed_cols,
    std::span<const float> scales,
    std::span<const float> biases,
    std::size_t group_size,
    std::span<const float> x) noexcept;

[[nodiscard]] VulkanBufferDispatchResult run_vulkan_q4_gemv_buffers(
    VulkanComputeContext& context,
    std::span<const std::uint32_t> packed,
    std::size_t out_dim,
    std::size_t packed_cols,
    std::span<const float> scales,
    std::span<const float> biases,
    std::size_t group_size,
    const VulkanFloatBuffer& x,
    VulkanFloatBuffer& y) noexcept;

[[nodiscard]] VulkanBufferDispatchResult run_vulkan_q4_gemv_preloaded(
    VulkanComputeContext& context,
    const VulkanQ4ProjectionWeights& weights,
    const VulkanFloatBuffer& x,
    VulkanFloatBuffer& y) noexcept;

}  // namespace orbi::streammoe
