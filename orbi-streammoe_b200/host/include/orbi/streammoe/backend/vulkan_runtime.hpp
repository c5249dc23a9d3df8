// Compute-runtime probe: lists the CUDA devices this process can use, in the
// shape of the reference's include/orbi/streammoe/backend/vulkan_runtime.hpp
// (loader = the CUDA runtime, instance = at least one device, every device
// has compute queue family 0).
#pragma once

#include <cstdint>
#include <optional>
#include <string>
#include <vector>

namespace orbi::streammoe {

struct VulkanDeviceInfo {
  std::string name;
  std::uint32_t vendor_id{};                      // 0x10DE
  std::uint32_t device_id{};                      // CUDA ordinal
  std::uint32_t api_version{};                    // CUDA runtime version
  std::uint32_t device_type{};                    // 2: discrete GPU
  std::optional<std::uint32_t> compute_queue_family;
  std::uint32_t max_compute_workgroup_invocations{};
  std::uint32_t max_compute_shared_memory_size{};
  std::uint64_t max_storage_buffer_range{};
};

struct VulkanProbeResult {
  bool loader_available{};
  std::uint32_t loader_api_version{};
  bool instance_created{};
  std::vector<VulkanDeviceInfo> devices;
  std::string diagnostic;
};

[[nodiscard]] VulkanProbeResult probe_vulkan_runtime() noexcept;

}  // namespace orbi::streammoe
