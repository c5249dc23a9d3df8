// accumulator[i] += weight * source[i] on the device (osm_weighted_accumulate).
// As include/orbi/streammoe/backend/vulkan_weighted_accumulate.hpp of the
// reference.
#pragma once

#include <string>

#include "orbi/streammoe/backend/vulkan_compute_context.hpp"
#include "orbi/streammoe/backend/vulkan_float_buffer.hpp"

namespace orbi::streammoe {

[[nodiscard]] VulkanBufferDispatchResult run_vulkan_weighted_accumulate(
    VulkanComputeContext& context,
    const VulkanFloatBuffer& source,
    float weight,
    VulkanFloatBuffer& accumulator) noexcept;

}  // namespace orbi::streammoe
