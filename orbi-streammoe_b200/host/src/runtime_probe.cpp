// probe_vulkan_runtime over osm_device_info: one entry per CUDA device.
#include <exception>
#include <string>

#include "orbi/streammoe/backend/vulkan_runtime.hpp"
#include "osm_b200.h"

namespace orbi::streammoe {

VulkanProbeResult probe_vulkan_runtime() noexcept {
  VulkanProbeResult r;
  try {
    for (int d = 0; d < 64; ++d) {
      char name[256] = {0};
      std::uint32_t sms = 0, rt = 0;
      if (osm_device_info(d, name, sizeof(name), &sms, &rt) != OSM_OK) break;
      r.loader_available = true;
      r.loader_api_version = rt;
      VulkanDeviceInfo info;
      info.name = name;
      info.vendor_id = 0x10DEu;
      info.device_id = static_cast<std::uint32_t>(d);
      info.api_version = rt;
      info.device_type = 2;
      info.compute_queue_family = 0u;
      info.max_compute_workgroup_invocations = 1024;       // threads per block
      info.max_compute_shared_memory_size = 227u * 1024u;  // opt-in shared memory per block
      info.max_storage_buffer_range = ~0ull;
      r.devices.push_back(std::move(info));
    }
    r.instance_created = !r.devices.empty();
    r.diagnostic = r.devices.empty() ? "no CUDA device is available"
                                     : std::to_string(r.devices.size()) + " CUDA device(s)";
  } catch (const std::exception& e) {
    r.diagnostic = std::string("CUDA probe exception: ") + e.what();
  }
  return r;
}

}  // namespace orbi::streammoe
