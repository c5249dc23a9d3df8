// CUDA-backed VulkanComputeContext: the device context the model layer passes
// around keeps its reference name so src/model compiles unchanged; here it
// owns an osm_context (one B200, one stream) of libosm_b200.
//
// Public interface as include/orbi/streammoe/backend/vulkan_compute_context.hpp
// of the reference (ingeniusvictor/orbi-streammoe).
#pragma once

#include <cstdint>
#include <memory>
#include <optional>
#include <span>
#include <string>

struct osm_context;
struct osm_layer;

namespace orbi::streammoe {

struct VulkanComputeContextInfo {
  std::string device_name;
  std::uint32_t vendor_id{};           // 0x10DE
  std::uint32_t device_id{};           // CUDA device ordinal
  std::uint32_t api_version{};         // CUDA runtime version
  std::uint32_t queue_family_index{};  // always 0 (one stream)
};

class VulkanComputeContext {
 public:
  VulkanComputeContext();
  ~VulkanComputeContext();

  VulkanComputeContext(const VulkanComputeContext&) = delete;
  VulkanComputeContext& operator=(const VulkanComputeContext&) = delete;
  VulkanComputeContext(VulkanComputeContext&&) noexcept;
  VulkanComputeContext& operator=(VulkanComputeContext&&) noexcept;

  // The current CUDA device (or OSM_DEVICE); std::nullopt with a diagnostic
  // when no CUDA device or libosm_b200 context is available.
  [[nodiscard]] static std::optional<VulkanComputeContext> create(
      std::string* diagnostic = nullptr) noexcept;

  [[nodiscard]] bool valid() const noexcept;
  [[nodiscard]] const VulkanComputeContextInfo& info() const noexcept;

  // Opaque handles as integers.  native_device() is the osm_context pointer
  // (the identity the resident objects compare against); native_queue() the
  // CUDA stream; the others have no CUDA counterpart and are 0.
  [[nodiscard]] std::uintptr_t native_instance() const noexcept;
  [[nodiscard]] std::uintptr_t native_physical_device() const noexcept;
  [[nodiscard]] std::uintptr_t native_device() const noexcept;
  [[nodiscard]] std::uintptr_t native_queue() const noexcept;
  [[nodiscard]] std::uintptr_t native_command_pool() const noexcept;

  // CUDA-side handle for the other backend classes (not in the reference).
  [[nodiscard]] osm_context* osm() const noexcept;

  // The device router for a router weight (not in the reference): a
  // libosm_b200 layer holding `weight` ([experts][hidden], row-major), made
  // at the first call for that span and reused while the span's address,
  // size, geometry and contents stay the same (the contents are compared
  // with a host copy at every call, so a caller that rewrites its router in
  // place gets a new layer).  Owned by this context; nullptr with a
  // diagnostic when the library rejects the router.
  [[nodiscard]] osm_layer* router_layer(std::span<const float> weight,
                                        std::uint32_t hidden,
                                        std::uint32_t experts,
                                        std::uint32_t top_k,
                                        bool norm_topk_prob,
                                        std::string* diagnostic = nullptr) noexcept;

 private:
  struct Impl;
  explicit VulkanComputeContext(std::unique_ptr<Impl> impl) noexcept;
  std::unique_ptr<Impl> impl_;
};

}  // namespace orbi::streammoe
