// The reference's backend classes (VulkanComputeContext, VulkanFloatBuffer,
// VulkanQ4ProjectionWeights, the element-wise ops, the qpack projection
// binding) implemented over the C ABI of libosm_b200 (include/osm_b200.h),
// so that the model layer of ingeniusvictor/orbi-streammoe (src/model/*)
// compiles and runs unchanged on a B200.  Every GPU operation goes through
// an osm_* call; this file holds host code only.
#include <bit>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "orbi/streammoe/backend/vulkan_compute_context.hpp"
#include "orbi/streammoe/backend/vulkan_float_buffer.hpp"
#include "orbi/streammoe/backend/vulkan_q4_dequant.hpp"
#include "orbi/streammoe/backend/vulkan_q4_gemv.hpp"
#include "orbi/streammoe/backend/vulkan_q4_weights.hpp"
#include "orbi/streammoe/backend/vulkan_qpack_expert.hpp"
#include "orbi/streammoe/backend/vulkan_rmsnorm.hpp"
#include "orbi/streammoe/backend/vulkan_swiglu.hpp"
#include "orbi/streammoe/backend/vulkan_weighted_accumulate.hpp"
#include "osm_b200.h"
#include "osm_host_util.hpp"

namespace orbi::streammoe {

namespace osmh {

void set(std::string* d, std::string v) {
  if (d) *d = std::move(v);
}

std::string err(osm_context* ctx, int rc, const char* what) {
  std::string s = std::string(what) + " (osm status " + std::to_string(rc) + ")";
  if (ctx) s += ": " + std::string(osm_last_error(ctx));
  return s;
}

bool bf16_exact(float v, std::uint16_t* bits) {
  const auto u = std::bit_cast<std::uint32_t>(v);
  if (u & 0xFFFFu) return false;
  *bits = static_cast<std::uint16_t>(u >> 16);
  return true;
}

bool narrow_bf16(std::span<const float> in, std::vector<std::uint16_t>& out, std::string* d,
                 const char* label) {
  out.resize(in.size());
  for (std::size_t i = 0; i < in.size(); ++i) {
    if (!bf16_exact(in[i], &out[i])) {
      set(d, std::string(label) +
                 ": affine scale/bias values must be bf16-representable (the device format)");
      return false;
    }
  }
  return true;
}

}  // namespace osmh

// ---------------------------------------------------------------------------
// VulkanComputeContext
// ---------------------------------------------------------------------------
struct VulkanComputeContext::Impl {
  osm_context* ctx = nullptr;
  VulkanComputeContextInfo info;

  // Device routers of the router weights this context has routed with, the
  // least recently used dropped past kMaxRouters.
  struct Router {
    const float* data = nullptr;
    std::size_t size = 0;
    std::uint32_t hidden = 0, experts = 0, top_k = 0;
    bool norm = false;
    std::vector<float> copy;  // contents at upload, compared at every use
    osm_layer* layer = nullptr;
    std::uint64_t last_use = 0;
  };
  static constexpr std::size_t kMaxRouters = 256;
  std::vector<Router> routers;
  std::uint64_t tick = 0;

  ~Impl() {
    for (auto& r : routers) osm_layer_destroy(r.layer);
    if (ctx) osm_context_destroy(ctx);
  }
};

VulkanComputeContext::VulkanComputeContext() = default;
VulkanComputeContext::~VulkanComputeContext() = default;
VulkanComputeContext::VulkanComputeContext(VulkanComputeContext&&) noexcept = default;
VulkanComputeContext& VulkanComputeContext::operator=(VulkanComputeContext&&) noexcept = default;
VulkanComputeContext::VulkanComputeContext(std::unique_ptr<Impl> impl) noexcept
    : impl_(std::move(impl)) {}

std::optional<VulkanComputeContext> VulkanComputeContext::create(std::string* diagnostic) noexcept {
  try {
    int device = 0;
    if (const char* v = std::getenv("OSM_DEVICE")) device = std::atoi(v);
    char name[256] = {0};
    std::uint32_t sms = 0, rt = 0;
    if (osm_device_info(device, name, sizeof(name), &sms, &rt) != OSM_OK) {
      osmh::set(diagnostic, "no CUDA device " + std::to_string(device) + " is available");
      return std::nullopt;
    }
    auto impl = std::make_unique<Impl>();
    // one-token calls of the reference API; 64 rows leaves room for small batches
    const int rc = osm_context_create(device, 64, &impl->ctx);
    if (rc != OSM_OK || !impl->ctx) {
      osmh::set(diagnostic, osmh::err(nullptr, rc, "CUDA context creation failed"));
      return std::nullopt;
    }
    impl->info.device_name = name;
    impl->info.vendor_id = 0x10DEu;
    impl->info.device_id = static_cast<std::uint32_t>(device);
    impl->info.api_version = rt;
    impl->info.queue_family_index = 0;
    osmh::set(diagnostic, std::string("CUDA compute context on ") + name + " (" +
                              std::to_string(sms) + " SMs)");
    return VulkanComputeContext(std::move(impl));
  } catch (const std::exception& e) {
    osmh::set(diagnostic, std::string("CUDA context creation exception: ") + e.what());
    return std::nullopt;
  }
}

bool VulkanComputeContext::valid() const noexcept { return impl_ && impl_->ctx; }

const VulkanComputeContextInfo& VulkanComputeContext::info() const noexcept {
  static const VulkanComputeContextInfo empty{};
  return impl_ ? impl_->info : empty;
}

// Handles: instance and device are the osm_context (one per process and
// GPU here), the physical device is the CUDA ordinal + 1 (0 stays "none"),
// queue and command pool are the context's CUDA stream.
std::uintptr_t VulkanComputeContext::native_instance() const noexcept { return native_device(); }
std::uintptr_t VulkanComputeContext::native_physical_device() const noexcept {
  return impl_ && impl_->ctx ? static_cast<std::uintptr_t>(osm_context_device(impl_->ctx)) + 1 : 0;
}
std::uintptr_t VulkanComputeContext::native_device() const noexcept {
  return impl_ ? reinterpret_cast<std::uintptr_t>(impl_->ctx) : 0;
}
std::uintptr_t VulkanComputeContext::native_queue() const noexcept {
  return impl_ && impl_->ctx ? reinterpret_cast<std::uintptr_t>(osm_context_stream(impl_->ctx)) : 0;
}
std::uintptr_t VulkanComputeContext::native_command_pool() const noexcept { return native_queue(); }
osm_context* VulkanComputeContext::osm() const noexcept { return impl_ ? impl_->ctx : nullptr; }

osm_layer* VulkanComputeContext::router_layer(std::span<const float> weight, std::uint32_t hidden,
                                              std::uint32_t experts, std::uint32_t top_k,
                                              bool norm_topk_prob, std::string* diagnostic) noexcept {
  if (!valid()) {
    osmh::set(diagnostic, "device router requires a valid compute context");
    return nullptr;
  }
  auto& m = *impl_;
  try {
    ++m.tick;
    for (auto it = m.routers.begin(); it != m.routers.end(); ++it) {
      if (it->data != weight.data() || it->size != weight.size() || it->hidden != hidden ||
          it->experts != experts || it->top_k != top_k || it->norm != norm_topk_prob)
        continue;
      if (std::memcmp(it->copy.data(), weight.data(), weight.size_bytes()) == 0) {
        it->last_use = m.tick;
        return it->layer;
      }
      osm_layer_destroy(it->layer);  // rewritten in place: upload it again
      m.routers.erase(it);
      break;
    }
    if (m.routers.size() >= Impl::kMaxRouters) {
      auto lru = m.routers.begin();
      for (auto it = m.routers.begin(); it != m.routers.end(); ++it)
        if (it->last_use < lru->last_use) lru = it;
      osm_layer_destroy(lru->layer);
      m.routers.erase(lru);
    }
    if (weight.size() != static_cast<std::size_t>(hidden) * experts) {
      osmh::set(diagnostic, "device router: weight size does not match experts x hidden");
      return nullptr;
    }
    osm_layer_desc d{};
    d.hidden = hidden;
    d.experts = experts;
    d.top_k = top_k;
    d.norm_topk_prob = norm_topk_prob ? 1u : 0u;
    d.router_weight_host = weight.data();
    osm_layer* layer = nullptr;
    const int rc = osm_layer_create(m.ctx, &d, &layer);
    if (rc != OSM_OK || !layer) {
      osmh::set(diagnostic, osmh::err(m.ctx, rc, "device router upload failed"));
      return nullptr;
    }
    Impl::Router r;
    r.data = weight.data();
    r.size = weight.size();
    r.hidden = hidden;
    r.experts = experts;
    r.top_k = top_k;
    r.norm = norm_topk_prob;
    r.copy.assign(weight.begin(), weight.end());
    r.layer = layer;
    r.last_use = m.tick;
    m.routers.push_back(std::move(r));
    return layer;
  } catch (const std::exception& e) {
    osmh::set(diagnostic, std::string("device router exception: ") + e.what());
    return nullptr;
  }
}

// ---------------------------------------------------------------------------
// VulkanFloatBuffer
// ---------------------------------------------------------------------------
struct VulkanFloatBuffer::Impl {
  osm_context* ctx = nullptr;
  float* dev = nullptr;
  std::size_t n = 0;
  ~Impl() {
    if (ctx && dev) osm_device_free(ctx, dev);
  }
};

VulkanFloatBuffer::VulkanFloatBuffer() = default;
VulkanFloatBuffer::~VulkanFloatBuffer() = default;
VulkanFloatBuffer::VulkanFloatBuffer(VulkanFloatBuffer&&) noexcept = default;
VulkanFloatBuffer& VulkanFloatBuffer::operator=(VulkanFloatBuffer&&) noexcept = default;
VulkanFloatBuffer::VulkanFloatBuffer(std::unique_ptr<Impl> impl) noexcept : impl_(std::move(impl)) {}

std::optional<VulkanFloatBuffer> VulkanFloatBuffer::create(VulkanComputeContext& context,
                                                           std::size_t element_count,
                                                           std::string* diagnostic) noexcept {
  if (!context.valid()) {
    osmh::set(diagnostic, "float buffer requires a valid compute context");
    return std::nullopt;
  }
  if (element_count == 0) {
    osmh::set(diagnostic, "float buffer element count must be non-zero");
    return std::nullopt;
  }
  try {
    auto impl = std::make_unique<Impl>();
    impl->ctx = context.osm();
    void* p = nullptr;
    const int rc = osm_device_alloc(impl->ctx, element_count * sizeof(float), &p);
    if (rc != OSM_OK) {
      osmh::set(diagnostic, osmh::err(impl->ctx, rc, "float buffer allocation failed"));
      impl->ctx = nullptr;
      return std::nullopt;
    }
    impl->dev = static_cast<float*>(p);
    impl->n = element_count;
    return VulkanFloatBuffer(std::move(impl));
  } catch (const std::exception& e) {
    osmh::set(diagnostic, std::string("float buffer exception: ") + e.what());
    return std::nullopt;
  }
}

bool VulkanFloatBuffer::valid() const noexcept { return impl_ && impl_->dev; }
std::size_t VulkanFloatBuffer::size() const noexcept { return impl_ ? impl_->n : 0; }
std::size_t VulkanFloatBuffer::size_bytes() const noexcept { return size() * sizeof(float); }

bool VulkanFloatBuffer::upload(std::span<const float> values, std::string* diagnostic) noexcept {
  if (!valid()) {
    osmh::set(diagnostic, "float buffer is not valid");
    return false;
  }
  if (values.size() != impl_->n) {
    osmh::set(diagnostic, "float buffer upload size mismatch");
    return false;
  }
  const int rc = osm_upload(impl_->ctx, impl_->dev, values.data(), values.size_bytes());
  if (rc != OSM_OK) {
    osmh::set(diagnostic, osmh::err(impl_->ctx, rc, "float buffer upload failed"));
    return false;
  }
  return true;
}

std::optional<std::vector<float>> VulkanFloatBuffer::download(std::string* diagnostic) const noexcept {
  if (!valid()) {
    osmh::set(diagnostic, "float buffer is not valid");
    return std::nullopt;
  }
  try {
    std::vector<float> out(impl_->n);
    const int rc = osm_download(impl_->ctx, out.data(), impl_->dev, out.size() * sizeof(float));
    if (rc != OSM_OK) {
      osmh::set(diagnostic, osmh::err(impl_->ctx, rc, "float buffer download failed"));
      return std::nullopt;
    }
    return out;
  } catch (const std::exception& e) {
    osmh::set(diagnostic, std::string("float buffer download exception: ") + e.what());
    return std::nullopt;
  }
}

std::uintptr_t VulkanFloatBuffer::native_buffer() const noexcept {
  return impl_ ? reinterpret_cast<std::uintptr_t>(impl_->dev) : 0;
}
std::uintptr_t VulkanFloatBuffer::native_device() const noexcept {
  return impl_ ? reinterpret_cast<std::uintptr_t>(impl_->ctx) : 0;
}
float* VulkanFloatBuffer::device_data() const noexcept { return impl_ ? impl_->dev : nullptr; }

// ---------------------------------------------------------------------------
// element-wise ops
// ---------------------------------------------------------------------------
namespace {

bool same_device(const VulkanComputeContext& c, const VulkanFloatBuffer& b) {
  return b.valid() && b.native_device() == c.native_device();
}

// Host vectors <-> temporary device buffers for the span-based entry points.
struct DeviceVec {
  osm_context* ctx = nullptr;
  void* p = nullptr;
  ~DeviceVec() {
    if (ctx && p) osm_device_free(ctx, p);
  }
  int alloc(osm_context* c, std::size_t bytes) {
    ctx = c;
    return osm_device_alloc(c, bytes, &p);
  }
  int put(osm_context* c, const void* host, std::size_t bytes) {
    int rc = alloc(c, bytes);
    if (rc == OSM_OK && bytes) rc = osm_upload(c, p, host, bytes);
    return rc;
  }
};

}  // namespace

VulkanBufferDispatchResult run_vulkan_weighted_accumulate(VulkanComputeContext& context,
                                                          const VulkanFloatBuffer& source, float weight,
                                                          VulkanFloatBuffer& accumulator) noexcept {
  VulkanBufferDispatchResult r;
  if (!context.valid() || !same_device(context, source) || !same_device(context, accumulator)) {
    r.diagnostic = "weighted accumulate: invalid context or buffers";
    return r;
  }
  if (source.size() != accumulator.size()) {
    r.diagnostic = "weighted accumulate: buffer sizes differ";
    return r;
  }
  osm_context* ctx = context.osm();
  int rc = osm_weighted_accumulate(ctx, source.device_data(), weight, accumulator.device_data(),
                                   source.size());
  if (rc == OSM_OK) rc = osm_context_synchronize(ctx);
  if (rc != OSM_OK) {
    r.diagnostic = osmh::err(ctx, rc, "weighted accumulate failed");
    return r;
  }
  r.executed = true;
  r.diagnostic = "weighted accumulate executed on CUDA";
  return r;
}

VulkanRmsNormResult run_vulkan_rms_norm(VulkanComputeContext& context, std::span<const float> input,
                                        std::size_t rows, std::size_t dim, std::span<const float> weight,
                                        float eps) noexcept {
  VulkanRmsNormResult r;
  if (!context.valid()) {
    r.diagnostic = "RMSNorm requires a valid compute context";
    return r;
  }
  if (rows == 0 || dim == 0 || input.size() != rows * dim) {
    r.diagnostic = "RMSNorm input shape mismatch";
    return r;
  }
  if (!weight.empty() && weight.size() != dim) {
    r.diagnostic = "RMSNorm weight shape mismatch";
    return r;
  }
  if (!std::isfinite(eps) || eps < 0.0f) {
    r.diagnostic = "RMSNorm eps must be finite and non-negative";
    return r;
  }
  try {
    osm_context* ctx = context.osm();
    DeviceVec v, w;
    int rc = v.put(ctx, input.data(), input.size_bytes());
    if (rc == OSM_OK && !weight.empty()) rc = w.put(ctx, weight.data(), weight.size_bytes());
    if (rc == OSM_OK)
      rc = osm_rms_norm(ctx, static_cast<float*>(v.p), (uint32_t)rows, (uint32_t)dim,
                        static_cast<const float*>(w.p), eps, OSM_RMSNORM_EXACT);
    r.values.resize(input.size());
    if (rc == OSM_OK) rc = osm_download(ctx, r.values.data(), v.p, input.size_bytes());
    if (rc != OSM_OK) {
      r.values.clear();
      r.diagnostic = osmh::err(ctx, rc, "RMSNorm failed");
      return r;
    }
    r.executed = true;
    r.diagnostic = "RMSNorm executed on CUDA (sequential sum, bit-exact with the CPU reference)";
    return r;
  } catch (const std::exception& e) {
    r.values.clear();
    r.diagnostic = std::string("RMSNorm exception: ") + e.what();
    return r;
  }
}

VulkanSwiGluResult run_vulkan_swiglu(VulkanComputeContext& context, std::span<const float> gate,
                                     std::span<const float> up) noexcept {
  VulkanSwiGluResult r;
  if (!context.valid() || gate.empty() || gate.size() != up.size()) {
    r.diagnostic = "SwiGLU: invalid context or input sizes";
    return r;
  }
  try {
    osm_context* ctx = context.osm();
    DeviceVec g, u, o;
    int rc = g.put(ctx, gate.data(), gate.size_bytes());
    if (rc == OSM_OK) rc = u.put(ctx, up.data(), up.size_bytes());
    if (rc == OSM_OK) rc = o.alloc(ctx, gate.size_bytes());
    if (rc == OSM_OK)
      rc = osm_swiglu(ctx, static_cast<const float*>(g.p), static_cast<const float*>(u.p),
                      static_cast<float*>(o.p), gate.size());
    r.values.resize(gate.size());
    if (rc == OSM_OK) rc = osm_download(ctx, r.values.data(), o.p, gate.size_bytes());
    if (rc != OSM_OK) {
      r.values.clear();
      r.diagnostic = osmh::err(ctx, rc, "SwiGLU failed");
      return r;
    }
    r.executed = true;
    r.diagnostic = "SwiGLU executed on CUDA";
    return r;
  } catch (const std::exception& e) {
    r.values.clear();
    r.diagnostic = std::string("SwiGLU exception: ") + e.what();
    return r;
  }
}

VulkanBufferDispatchResult run_vulkan_swiglu_buffers(VulkanComputeContext& context,
                                                     const VulkanFloatBuffer& gate,
                                                     const VulkanFloatBuffer& up,
                                                     VulkanFloatBuffer& output) noexcept {
  VulkanBufferDispatchResult r;
  if (!context.valid() || !same_device(context, gate) || !same_device(context, up) ||
      !same_device(context, output) || gate.size() != up.size() || gate.size() != output.size()) {
    r.diagnostic = "SwiGLU: invalid context or buffers";
    return r;
  }
  osm_context* ctx = context.osm();
  int rc = osm_swiglu(ctx, gate.device_data(), up.device_data(), output.device_data(), gate.size());
  if (rc == OSM_OK) rc = osm_context_synchronize(ctx);
  if (rc != OSM_OK) {
    r.diagnostic = osmh::err(ctx, rc, "SwiGLU failed");
    return r;
  }
  r.executed = true;
  r.diagnostic = "SwiGLU executed on CUDA";
  return r;
}

namespace {

// Checks the affine Q4 geometry the reference's kernels accept.
bool q4_geometry(std::size_t rows, std::size_t packed_cols, std::size_t group, std::size_t packed,
                 std::size_t scales, std::size_t biases, std::string* d) {
  if (rows == 0 || packed_cols == 0 || group == 0) {
    osmh::set(d, "affine Q4: dimensions and group size must be non-zero");
    return false;
  }
  const std::size_t cols = packed_cols * 8;
  if (cols % group) {
    osmh::set(d, "affine Q4: logical columns must be divisible by the group size");
    return false;
  }
  const std::size_t groups = rows * (cols / group);
  if (packed != rows * packed_cols || scales != groups || biases != groups) {
    osmh::set(d, "affine Q4: packed/scale/bias sizes disagree with the geometry");
    return false;
  }
  return true;
}

}  // namespace

VulkanQ4DequantResult run_vulkan_q4_dequant(VulkanComputeContext& context,
                                            std::span<const std::uint32_t> packed, std::size_t rows,
                                            std::size_t packed_cols, std::span<const float> scales,
                                            std::span<const float> biases,
                                            std::size_t group_size) noexcept {
  VulkanQ4DequantResult r;
  if (!context.valid()) {
    r.diagnostic = "Q4 dequant requires a valid compute context";
    return r;
  }
  if (!q4_geometry(rows, packed_cols, group_size, packed.size(), scales.size(), biases.size(),
                   &r.diagnostic))
    return r;
  try {
    // bf16 metadata (the slot format) when it holds the values exactly, else fp32
    std::vector<std::uint16_t> sb, bb;
    const bool bf16 = osmh::narrow_bf16(scales, sb, nullptr, "") &&
                      osmh::narrow_bf16(biases, bb, nullptr, "");
    osm_context* ctx = context.osm();
    DeviceVec p, s, b, o;
    const std::size_t cols = packed_cols * 8;
    int rc = p.put(ctx, packed.data(), packed.size_bytes());
    if (rc == OSM_OK)
      rc = bf16 ? s.put(ctx, sb.data(), sb.size() * 2) : s.put(ctx, scales.data(), scales.size_bytes());
    if (rc == OSM_OK)
      rc = bf16 ? b.put(ctx, bb.data(), bb.size() * 2) : b.put(ctx, biases.data(), biases.size_bytes());
    if (rc == OSM_OK) rc = o.alloc(ctx, rows * cols * sizeof(float));
    if (rc == OSM_OK)
      rc = bf16 ? osm_q4_dequant(ctx, static_cast<const uint32_t*>(p.p),
                                 static_cast<const uint16_t*>(s.p), static_cast<const uint16_t*>(b.p),
                                 (uint32_t)rows, (uint32_t)cols, (uint32_t)group_size,
                                 static_cast<float*>(o.p))
                : osm_q4_dequant_f32(ctx, static_cast<const uint32_t*>(p.p),
                                     static_cast<const float*>(s.p), static_cast<const float*>(b.p),
                                     (uint32_t)rows, (uint32_t)cols, (uint32_t)group_size,
                                     static_cast<float*>(o.p));
    r.values.resize(rows * cols);
    if (rc == OSM_OK) rc = osm_download(ctx, r.values.data(), o.p, r.values.size() * sizeof(float));
    if (rc != OSM_OK) {
      r.values.clear();
      r.diagnostic = osmh::err(ctx, rc, "Q4 dequant failed");
      return r;
    }
    r.executed = true;
    r.diagnostic = "affine Q4 dequant executed on CUDA";
    return r;
  } catch (const std::exception& e) {
    r.values.clear();
    r.diagnostic = std::string("Q4 dequant exception: ") + e.what();
    return r;
  }
}

// ---------------------------------------------------------------------------
// VulkanQ4ProjectionWeights
// ---------------------------------------------------------------------------
struct VulkanQ4ProjectionWeights::Impl {
  osm_context* ctx = nullptr;
  void* packed = nullptr;
  void* s16 = nullptr;
  void* b16 = nullptr;
  std::size_t out_dim = 0, packed_cols = 0, group = 0;
  std::optional<VulkanFloatBuffer> scales, biases;  // fp32 copies (the reference's accounting)
  ~Impl() {
    if (ctx) {
      if (packed) osm_device_free(ctx, packed);
      if (s16) osm_device_free(ctx, s16);
      if (b16) osm_device_free(ctx, b16);
    }
  }
};

VulkanQ4ProjectionWeights::VulkanQ4ProjectionWeights() = default;
VulkanQ4ProjectionWeights::~VulkanQ4ProjectionWeights() = default;
VulkanQ4ProjectionWeights::VulkanQ4ProjectionWeights(VulkanQ4ProjectionWeights&&) noexcept = default;
VulkanQ4ProjectionWeights& VulkanQ4ProjectionWeights::operator=(VulkanQ4ProjectionWeights&&) noexcept =
    default;
VulkanQ4ProjectionWeights::VulkanQ4ProjectionWeights(std::unique_ptr<Impl> impl) noexcept
    : impl_(std::move(impl)) {}

std::optional<VulkanQ4ProjectionWeights> VulkanQ4ProjectionWeights::create(
    VulkanComputeContext& context, std::span<const std::uint32_t> packed, std::size_t out_dim,
    std::size_t packed_cols, std::span<const float> scales, std::span<const float> biases,
    std::size_t group_size, std::string* diagnostic) noexcept {
  std::string local;
  if (!context.valid()) {
    osmh::set(diagnostic, "Q4 weights require a valid compute context");
    return std::nullopt;
  }
  if (!q4_geometry(out_dim, packed_cols, group_size, packed.size(), scales.size(), biases.size(),
                   &local)) {
    osmh::set(diagnostic, local);
    return std::nullopt;
  }
  try {
    // bf16 copies of the metadata (read by the row-tiled kernel) when bf16
    // holds the values exactly; the fp32 buffers below serve the rest
    std::vector<std::uint16_t> sb, bb;
    const bool bf16 = osmh::narrow_bf16(scales, sb, nullptr, "") &&
                      osmh::narrow_bf16(biases, bb, nullptr, "");
    auto impl = std::make_unique<Impl>();
    osm_context* ctx = context.osm();
    impl->ctx = ctx;
    impl->out_dim = out_dim;
    impl->packed_cols = packed_cols;
    impl->group = group_size;
    int rc = osm_device_alloc(ctx, packed.size_bytes(), &impl->packed);
    if (rc == OSM_OK) rc = osm_upload(ctx, impl->packed, packed.data(), packed.size_bytes());
    if (bf16) {
      if (rc == OSM_OK) rc = osm_device_alloc(ctx, sb.size() * 2, &impl->s16);
      if (rc == OSM_OK) rc = osm_upload(ctx, impl->s16, sb.data(), sb.size() * 2);
      if (rc == OSM_OK) rc = osm_device_alloc(ctx, bb.size() * 2, &impl->b16);
      if (rc == OSM_OK) rc = osm_upload(ctx, impl->b16, bb.data(), bb.size() * 2);
    }
    if (rc != OSM_OK) {
      osmh::set(diagnostic, osmh::err(ctx, rc, "Q4 weights upload failed"));
      return std::nullopt;
    }
    impl->scales = VulkanFloatBuffer::create(context, scales.size(), &local);
    impl->biases = VulkanFloatBuffer::create(context, biases.size(), &local);
    if (!impl->scales || !impl->biases || !impl->scales->upload(scales, &local) ||
        !impl->biases->upload(biases, &local)) {
      osmh::set(diagnostic, "Q4 weights metadata upload failed: " + local);
      return std::nullopt;
    }
    osmh::set(diagnostic, "affine Q4 projection weights resident in HBM");
    return VulkanQ4ProjectionWeights(std::move(impl));
  } catch (const std::exception& e) {
    osmh::set(diagnostic, std::string("Q4 weights exception: ") + e.what());
    return std::nullopt;
  }
}

bool VulkanQ4ProjectionWeights::valid() const noexcept {
  return impl_ && impl_->packed && impl_->scales && impl_->biases;
}
std::size_t VulkanQ4ProjectionWeights::out_dim() const noexcept { return impl_ ? impl_->out_dim : 0; }
std::size_t VulkanQ4ProjectionWeights::packed_cols() const noexcept {
  return impl_ ? impl_->packed_cols : 0;
}
std::size_t VulkanQ4ProjectionWeights::in_dim() const noexcept { return packed_cols() * 8; }
std::size_t VulkanQ4ProjectionWeights::group_size() const noexcept { return impl_ ? impl_->group : 0; }
std::uintptr_t VulkanQ4ProjectionWeights::native_device() const noexcept {
  return impl_ ? reinterpret_cast<std::uintptr_t>(impl_->ctx) : 0;
}
std::uintptr_t VulkanQ4ProjectionWeights::native_packed_buffer() const noexcept {
  return impl_ ? reinterpret_cast<std::uintptr_t>(impl_->packed) : 0;
}
std::size_t VulkanQ4ProjectionWeights::packed_size_bytes() const noexcept {
  return impl_ ? impl_->out_dim * impl_->packed_cols * 4 : 0;
}
const VulkanFloatBuffer& VulkanQ4ProjectionWeights::scales_buffer() const noexcept {
  static const VulkanFloatBuffer empty;
  return impl_ && impl_->scales ? *impl_->scales : empty;
}
const VulkanFloatBuffer& VulkanQ4ProjectionWeights::biases_buffer() const noexcept {
  static const VulkanFloatBuffer empty;
  return impl_ && impl_->biases ? *impl_->biases : empty;
}
const std::uint32_t* VulkanQ4ProjectionWeights::device_packed() const noexcept {
  return impl_ ? static_cast<const std::uint32_t*>(impl_->packed) : nullptr;
}
const std::uint16_t* VulkanQ4ProjectionWeights::device_scales_bf16() const noexcept {
  return impl_ ? static_cast<const std::uint16_t*>(impl_->s16) : nullptr;
}
const std::uint16_t* VulkanQ4ProjectionWeights::device_biases_bf16() const noexcept {
  return impl_ ? static_cast<const std::uint16_t*>(impl_->b16) : nullptr;
}

// ---------------------------------------------------------------------------
// Q4 GEMV
// ---------------------------------------------------------------------------
VulkanBufferDispatchResult run_vulkan_q4_gemv_preloaded(VulkanComputeContext& context,
                                                        const VulkanQ4ProjectionWeights& weights,
                                                        const VulkanFloatBuffer& x,
                                                        VulkanFloatBuffer& y) noexcept {
  VulkanBufferDispatchResult r;
  if (!context.valid() || !weights.valid() || weights.native_device() != context.native_device() ||
      !same_device(context, x) || !same_device(context, y)) {
    r.diagnostic = "Q4 GEMV: invalid context, weights or buffers";
    return r;
  }
  if (x.size() != weights.in_dim() || y.size() != weights.out_dim()) {
    r.diagnostic = "Q4 GEMV: buffer shapes disagree with the weights";
    return r;
  }
  osm_context* ctx = context.osm();
  const auto od = (uint32_t)weights.out_dim(), id = (uint32_t)weights.in_dim(),
             gs = (uint32_t)weights.group_size();
  int rc = weights.device_scales_bf16()
               ? osm_q4_gemv(ctx, weights.device_packed(), weights.device_scales_bf16(),
                             weights.device_biases_bf16(), od, id, gs, x.device_data(), 1,
                             y.device_data())
               : osm_q4_gemv_f32(ctx, weights.device_packed(),
                                 weights.scales_buffer().device_data(),
                                 weights.biases_buffer().device_data(), od, id, gs,
                                 x.device_data(), 1, y.device_data());
  if (rc == OSM_OK) rc = osm_context_synchronize(ctx);
  if (rc != OSM_OK) {
    r.diagnostic = osmh::err(ctx, rc, "Q4 GEMV failed");
    return r;
  }
  r.executed = true;
  r.diagnostic = "affine Q4 GEMV executed on CUDA from resident weights";
  return r;
}

VulkanBufferDispatchResult run_vulkan_q4_gemv_buffers(VulkanComputeContext& context,
                                                      std::span<const std::uint32_t> packed,
                                                      std::size_t out_dim, std::size_t packed_cols,
                                                      std::span<const float> scales,
                                                      std::span<const float> biases,
                                                      std::size_t group_size,
                                                      const VulkanFloatBuffer& x,
                                                      VulkanFloatBuffer& y) noexcept {
  VulkanBufferDispatchResult r;
  auto w = VulkanQ4ProjectionWeights::create(context, packed, out_dim, packed_cols, scales, biases,
                                             group_size, &r.diagnostic);
  if (!w) return r;
  return run_vulkan_q4_gemv_preloaded(context, *w, x, y);
}

VulkanQ4GemvResult run_vulkan_q4_gemv(VulkanComputeContext& context,
                                      std::span<const std::uint32_t> packed, std::size_t out_dim,
                                      std::size_t packed_cols, std::span<const float> scales,
                                      std::span<const float> biases, std::size_t group_size,
                                      std::span<const float> x) noexcept {
  VulkanQ4GemvResult r;
  if (!context.valid()) {
    r.diagnostic = "Q4 GEMV requires a valid compute context";
    return r;
  }
  if (x.size() != packed_cols * 8) {
    r.diagnostic = "Q4 GEMV: input size disagrees with packed_cols * 8";
    return r;
  }
  std::string d;
  auto xb = VulkanFloatBuffer::create(context, x.size(), &d);
  auto yb = VulkanFloatBuffer::create(context, out_dim, &d);
  if (!xb || !yb || !xb->upload(x, &d)) {
    r.diagnostic = "Q4 GEMV buffers: " + d;
    return r;
  }
  const auto disp = run_vulkan_q4_gemv_buffers(context, packed, out_dim, packed_cols, scales, biases,
                                               group_size, *xb, *yb);
  if (!disp.executed) {
    r.diagnostic = disp.diagnostic;
    return r;
  }
  auto out = yb->download(&d);
  if (!out) {
    r.diagnostic = "Q4 GEMV download: " + d;
    return r;
  }
  r.values = std::move(*out);
  r.executed = true;
  r.diagnostic = disp.diagnostic;
  return r;
}

// ---------------------------------------------------------------------------
// qpack projection binding (the section table of layout.json)
// ---------------------------------------------------------------------------
namespace {

std::size_t shape_product(const std::vector<std::size_t>& shape) {
  std::size_t v = 1;
  for (const auto d : shape) {
    if (d == 0 || v > std::numeric_limits<std::size_t>::max() / d)
      throw std::runtime_error("qpack expert: invalid or overflowing section shape");
    v *= d;
  }
  return v;
}

float half_bits_to_float(std::uint16_t h) {
  const std::uint32_t sign = static_cast<std::uint32_t>(h & 0x8000u) << 16;
  const int e = (h >> 10) & 0x1F;
  const std::uint32_t m = h & 0x3FFu;
  if (e == 0) {  // zero or subnormal: m * 2^-24
    const float mag = std::ldexp(static_cast<float>(m), -24);
    return sign ? -mag : mag;
  }
  if (e == 0x1F) return std::bit_cast<float>(sign | 0x7F800000u | (m << 13));
  return std::bit_cast<float>(sign | (static_cast<std::uint32_t>(e + 112) << 23) | (m << 13));
}

std::vector<float> metadata(std::span<const std::byte> bytes, const QpackSection& s, const char* label) {
  const std::size_t count = shape_product(s.shape);
  if (s.offset > bytes.size() || s.size > bytes.size() - s.offset)
    throw std::runtime_error(std::string("qpack expert: ") + label + " section exceeds the cache slot");
  const std::byte* raw = bytes.data() + s.offset;
  std::vector<float> out(count);
  if (s.dtype == "F32") {
    if (s.size != count * 4)
      throw std::runtime_error(std::string("qpack expert: F32 ") + label + " size disagrees with its shape");
    std::memcpy(out.data(), raw, count * 4);
    return out;
  }
  if (s.dtype == "BF16" || s.dtype == "F16") {
    if (s.size != count * 2)
      throw std::runtime_error("qpack expert: " + s.dtype + " " + label + " size disagrees with its shape");
    for (std::size_t i = 0; i < count; ++i) {
      std::uint16_t h;
      std::memcpy(&h, raw + i * 2, 2);
      out[i] = s.dtype == "BF16" ? std::bit_cast<float>(static_cast<std::uint32_t>(h) << 16)
                                 : half_bits_to_float(h);
    }
    return out;
  }
  throw std::runtime_error(std::string("qpack expert: unsupported ") + label + " dtype " + s.dtype);
}

}  // namespace

QpackExpertQ4View bind_qpack_q4_projection(const QpackReader& reader, const ExpertCacheEntry& entry,
                                           std::string_view projection) {
  const auto& manifest = reader.manifest();
  if (!manifest.quant_bits || !manifest.quant_group_size || *manifest.quant_bits != 4u ||
      *manifest.quant_group_size == 0u)
    throw std::runtime_error("qpack expert: the projection needs affine Q4 manifest metadata");
  const std::string p(projection);
  const auto* w = reader.find_section(p + ".weight");
  const auto* s = reader.find_section(p + ".scales");
  const auto* b = reader.find_section(p + ".biases");
  if (!w || !s || !b) throw std::runtime_error("qpack expert: weight/scales/biases sections incomplete");
  if (w->dtype != "U32") throw std::runtime_error("qpack expert: Q4 weight dtype must be U32");
  if (s->dtype != b->dtype) throw std::runtime_error("qpack expert: scale and bias dtypes must match");
  if (s->dtype != "F32" && s->dtype != "F16" && s->dtype != "BF16")
    throw std::runtime_error("qpack expert: scale/bias dtype must be F32, F16 or BF16");
  if (w->shape.size() != 2 || s->shape.size() != 2 || b->shape.size() != 2)
    throw std::runtime_error("qpack expert: projection sections must be rank-2");
  const std::size_t out_dim = w->shape[0], packed_cols = w->shape[1];
  if (out_dim == 0 || packed_cols == 0)
    throw std::runtime_error("qpack expert: projection dimensions must be non-zero");
  if (packed_cols > std::numeric_limits<std::size_t>::max() / 8)
    throw std::runtime_error("qpack expert: packed projection dimension overflows");
  const std::size_t group = *manifest.quant_group_size;
  if ((packed_cols * 8) % group)
    throw std::runtime_error("qpack expert: logical input dimension not divisible by the group size");
  const std::size_t gpr = packed_cols * 8 / group;
  if (s->shape[0] != out_dim || b->shape[0] != out_dim || s->shape[1] != gpr || b->shape[1] != gpr)
    throw std::runtime_error("qpack expert: scale/bias shapes disagree with the Q4 geometry");
  if (w->offset % alignof(std::uint32_t) || w->size % sizeof(std::uint32_t))
    throw std::runtime_error("qpack expert: misaligned or odd-sized weight section");
  if (w->offset > entry.bytes.size() || w->size > entry.bytes.size() - w->offset)
    throw std::runtime_error("qpack expert: weight section exceeds the cache slot");
  if (w->size / 4 != shape_product(w->shape))
    throw std::runtime_error("qpack expert: weight byte size disagrees with its shape");
  QpackExpertQ4View v;
  v.packed = {reinterpret_cast<const std::uint32_t*>(entry.bytes.data() + w->offset),
              static_cast<std::size_t>(w->size / 4)};
  v.scales = metadata(entry.bytes, *s, "scales");
  v.biases = metadata(entry.bytes, *b, "biases");
  v.out_dim = out_dim;
  v.packed_cols = packed_cols;
  v.group_size = group;
  v.metadata_dtype = s->dtype;
  return v;
}

VulkanQ4GemvResult run_vulkan_qpack_q4_projection(VulkanComputeContext& context,
                                                  const QpackReader& reader,
                                                  const ExpertCacheEntry& entry,
                                                  std::string_view projection,
                                                  std::span<const float> x) noexcept {
  try {
    const auto v = bind_qpack_q4_projection(reader, entry, projection);
    return run_vulkan_q4_gemv(context, v.packed, v.out_dim, v.packed_cols, v.scales, v.biases,
                              v.group_size, x);
  } catch (const std::exception& e) {
    VulkanQ4GemvResult r;
    r.diagnostic = std::string("qpack projection: ") + e.what();
    return r;
  }
}

VulkanBufferDispatchResult run_vulkan_qpack_q4_projection_buffers(VulkanComputeContext& context,
                                                                  const QpackReader& reader,
                                                                  const ExpertCacheEntry& entry,
                                                                  std::string_view projection,
                                                                  const VulkanFloatBuffer& x,
                                                                  VulkanFloatBuffer& y) noexcept {
  try {
    const auto v = bind_qpack_q4_projection(reader, entry, projection);
    return run_vulkan_q4_gemv_buffers(context, v.packed, v.out_dim, v.packed_cols, v.scales, v.biases,
                                      v.group_size, x, y);
  } catch (const std::exception& e) {
    VulkanBufferDispatchResult r;
    r.diagnostic = std::string("qpack projection: ") + e.what();
    return r;
  }
}

}  // namespace orbi::streammoe
