// VulkanResidentExpert, VulkanResidentExpertCache and
// VulkanResidentSharedExpert over libosm_b200's C ABI.
//
// A resident expert of the geometry the fused expert kernels take (group 64,
// hidden a multiple of 64 up to 2048, intermediate a multiple of 64 up to 768,
// down output == hidden) lives in one slot of an expert slab and runs through
// osm_expert_forward (gate/up, SwiGLU and down in two launches).  Any other
// geometry (the reference's tiny fixtures: group 4, hidden 8) keeps three
// VulkanQ4ProjectionWeights and runs three any-geometry GEMVs and a SwiGLU,
// as the reference's src/backend/vulkan_resident_expert.cpp:285-360 does.
//
// Byte accounting is the reference's (vulkan_resident_expert.cpp:258-280:
// packed words + fp32 scales and biases + five fp32 activation buffers), so
// that cache budgets written for the reference hold the same experts.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <map>
#include <stdexcept>
#include <string>
#include <tuple>
#include <unordered_map>
#include <utility>
#include <vector>

#include "orbi/streammoe/backend/vulkan_q4_gemv.hpp"
#include "orbi/streammoe/backend/vulkan_q4_weights.hpp"
#include "orbi/streammoe/backend/vulkan_qpack_expert.hpp"
#include "orbi/streammoe/backend/vulkan_resident_expert.hpp"
#include "orbi/streammoe/backend/vulkan_resident_expert_cache.hpp"
#include "orbi/streammoe/backend/vulkan_resident_shared_expert.hpp"
#include "orbi/streammoe/backend/vulkan_swiglu.hpp"
#include "osm_b200.h"
#include "osm_host_util.hpp"

namespace orbi::streammoe {

namespace {

constexpr std::uint32_t kFillTimeoutMs = 30000;

struct Geometry {
  std::size_t in = 0, inter = 0, out = 0, group = 0;
  std::size_t packed_words = 0;    // gate + up + down
  std::size_t metadata_values = 0; // scales + biases, all projections
};

std::size_t accounted(const Geometry& g) {
  return g.packed_words * 4 + g.metadata_values * 4 + 4 * (g.in + 3 * g.inter + g.out);
}

// The packed slot layout the expert kernels read, when this geometry has one.
bool slab_layout(const Geometry& g, osm_expert_layout* L) {
  if (g.group != 64 || g.out != g.in) return false;
  if (g.in % 64 || g.inter % 64 || g.in > 2048 || g.inter > 768) return false;
  return osm_expert_layout_packed(static_cast<std::uint32_t>(g.in),
                                  static_cast<std::uint32_t>(g.inter), 64, L) == OSM_OK;
}

// One projection's words and bf16 metadata into its sections of a slot image.
bool put_projection(std::vector<unsigned char>& img, std::uint64_t w_off, std::uint64_t s_off,
                    std::uint64_t b_off, const QpackExpertQ4View& v, std::string* d,
                    const char* label) {
  std::vector<std::uint16_t> s16, b16;
  if (!osmh::narrow_bf16(v.scales, s16, d, label) || !osmh::narrow_bf16(v.biases, b16, d, label))
    return false;
  std::memcpy(img.data() + w_off, v.packed.data(), v.packed.size_bytes());
  std::memcpy(img.data() + s_off, s16.data(), s16.size() * 2);
  std::memcpy(img.data() + b_off, b16.data(), b16.size() * 2);
  return true;
}

}  // namespace

// ---------------------------------------------------------------------------
// VulkanResidentExpert
// ---------------------------------------------------------------------------
struct VulkanResidentExpert::Impl {
  osm_context* ctx = nullptr;
  Geometry g;
  // slab mode
  osm_slab* slab = nullptr;
  bool owns_slab = false;
  std::int32_t slot = -1;
  osm_expert_layout layout{};
  // any-geometry mode
  std::optional<VulkanQ4ProjectionWeights> gate_w, up_w, down_w;
  std::optional<VulkanFloatBuffer> gate, up, hidden;
  // both
  std::optional<VulkanFloatBuffer> input, output;

  ~Impl() {
    if (owns_slab && slab) osm_slab_destroy(slab);
  }
  bool slab_mode() const { return slab != nullptr; }
};

VulkanResidentExpert::VulkanResidentExpert() = default;
VulkanResidentExpert::~VulkanResidentExpert() = default;
VulkanResidentExpert::VulkanResidentExpert(VulkanResidentExpert&&) noexcept = default;
VulkanResidentExpert& VulkanResidentExpert::operator=(VulkanResidentExpert&&) noexcept = default;
VulkanResidentExpert::VulkanResidentExpert(std::unique_ptr<Impl> impl) noexcept
    : impl_(std::move(impl)) {}

namespace {

// Binds the three projections of an entry and checks they form an expert
// (the reference's checks, vulkan_resident_expert.cpp:70-105).
bool bind_expert(const QpackReader& reader, const ExpertCacheEntry& entry, QpackExpertQ4View& gate,
                 QpackExpertQ4View& up, QpackExpertQ4View& down, Geometry& g, std::string* d) {
  gate = bind_qpack_q4_projection(reader, entry, "gate_proj");
  up = bind_qpack_q4_projection(reader, entry, "up_proj");
  down = bind_qpack_q4_projection(reader, entry, "down_proj");
  g.in = gate.packed_cols * 8;
  g.inter = gate.out_dim;
  g.out = down.out_dim;
  if (g.in == 0 || g.inter == 0 || g.out == 0) {
    osmh::set(d, "resident expert dimensions must be non-zero");
    return false;
  }
  if (up.packed_cols * 8 != g.in || up.out_dim != g.inter) {
    osmh::set(d, "resident expert gate/up geometry mismatch");
    return false;
  }
  if (down.packed_cols * 8 != g.inter) {
    osmh::set(d, "resident expert down input does not match intermediate dimension");
    return false;
  }
  g.group = gate.group_size;
  g.packed_words = gate.packed.size() + up.packed.size() + down.packed.size();
  g.metadata_values = gate.scales.size() + gate.biases.size() + up.scales.size() +
                      up.biases.size() + down.scales.size() + down.biases.size();
  return true;
}

bool metadata_bf16(const QpackExpertQ4View& v) {
  std::uint16_t b;
  for (const float f : v.scales)
    if (!osmh::bf16_exact(f, &b)) return false;
  for (const float f : v.biases)
    if (!osmh::bf16_exact(f, &b)) return false;
  return true;
}

// Whether the expert can live in a slab slot: a geometry the fused expert
// kernels take and metadata the slot's bf16 format holds exactly.
bool slab_eligible(const QpackExpertQ4View& gate, const QpackExpertQ4View& up,
                   const QpackExpertQ4View& down, const Geometry& g, osm_expert_layout* L) {
  return slab_layout(g, L) && metadata_bf16(gate) && metadata_bf16(up) && metadata_bf16(down);
}

bool slab_eligible(const QpackReader& reader, const ExpertCacheEntry& entry, Geometry* geo,
                   osm_expert_layout* L) {
  QpackExpertQ4View g, u, d;
  std::string ignored;
  return bind_expert(reader, entry, g, u, d, *geo, &ignored) && slab_eligible(g, u, d, *geo, L);
}

}  // namespace

std::optional<VulkanResidentExpert> VulkanResidentExpert::create(VulkanComputeContext& context,
                                                                 const QpackReader& reader,
                                                                 const ExpertCacheEntry& entry,
                                                                 std::string* diagnostic) noexcept {
  return create_in_slab(context, reader, entry, nullptr, 0, diagnostic);
}

std::optional<VulkanResidentExpert> VulkanResidentExpert::create_in_slab(
    VulkanComputeContext& context, const QpackReader& reader, const ExpertCacheEntry& entry,
    osm_slab* slab, std::uint32_t slot, std::string* diagnostic) noexcept {
  if (!context.valid()) {
    osmh::set(diagnostic, "resident expert requires a valid compute context");
    return std::nullopt;
  }
  try {
    QpackExpertQ4View gate, up, down;
    auto impl = std::make_unique<Impl>();
    impl->ctx = context.osm();
    if (!bind_expert(reader, entry, gate, up, down, impl->g, diagnostic)) return std::nullopt;
    const Geometry& g = impl->g;
    std::string local;

    osm_expert_layout L{};
    const bool slab_ok = slab_eligible(gate, up, down, g, &L);
    if (slab && !slab_ok) {
      osmh::set(diagnostic,
                "resident expert: geometry or non-bf16 metadata has no slab slot format");
      return std::nullopt;
    }
    if (slab_ok) {
      if (!slab) {
        const int rc = osm_slab_create(impl->ctx, &L, 1, &impl->slab);
        if (rc != OSM_OK) {
          osmh::set(diagnostic, osmh::err(impl->ctx, rc, "resident expert slab allocation failed"));
          return std::nullopt;
        }
        impl->owns_slab = true;
        slot = 0;
      } else {
        if (slot >= osm_slab_slots(slab)) {
          osmh::set(diagnostic, "resident expert: slab slot out of range");
          return std::nullopt;
        }
        impl->slab = slab;
      }
      impl->slot = static_cast<std::int32_t>(slot);
      impl->layout = L;
      std::vector<unsigned char> img(L.stride, 0);
      if (!put_projection(img, L.gate_w, L.gate_s, L.gate_b, gate, diagnostic, "gate projection") ||
          !put_projection(img, L.up_w, L.up_s, L.up_b, up, diagnostic, "up projection") ||
          !put_projection(img, L.down_w, L.down_s, L.down_b, down, diagnostic, "down projection"))
        return std::nullopt;
      int rc = osm_slab_fill_async(impl->slab, slot, img.data());
      if (rc == OSM_OK) rc = osm_slab_fill_wait(impl->slab, kFillTimeoutMs);
      if (rc != OSM_OK) {
        osmh::set(diagnostic, osmh::err(impl->ctx, rc, "resident expert upload failed"));
        return std::nullopt;
      }
    } else {
      impl->gate_w = VulkanQ4ProjectionWeights::create(context, gate.packed, gate.out_dim,
                                                       gate.packed_cols, gate.scales, gate.biases,
                                                       gate.group_size, &local);
      if (!impl->gate_w) {
        osmh::set(diagnostic, "resident expert gate upload failed: " + local);
        return std::nullopt;
      }
      impl->up_w = VulkanQ4ProjectionWeights::create(context, up.packed, up.out_dim, up.packed_cols,
                                                     up.scales, up.biases, up.group_size, &local);
      if (!impl->up_w) {
        osmh::set(diagnostic, "resident expert up upload failed: " + local);
        return std::nullopt;
      }
      impl->down_w = VulkanQ4ProjectionWeights::create(context, down.packed, down.out_dim,
                                                       down.packed_cols, down.scales, down.biases,
                                                       down.group_size, &local);
      if (!impl->down_w) {
        osmh::set(diagnostic, "resident expert down upload failed: " + local);
        return std::nullopt;
      }
      impl->gate = VulkanFloatBuffer::create(context, g.inter, &local);
      impl->up = VulkanFloatBuffer::create(context, g.inter, &local);
      impl->hidden = VulkanFloatBuffer::create(context, g.inter, &local);
      if (!impl->gate || !impl->up || !impl->hidden) {
        osmh::set(diagnostic, "resident expert activation allocation failed: " + local);
        return std::nullopt;
      }
    }
    impl->input = VulkanFloatBuffer::create(context, g.in, &local);
    impl->output = VulkanFloatBuffer::create(context, g.out, &local);
    if (!impl->input || !impl->output) {
      osmh::set(diagnostic, "resident expert activation allocation failed: " + local);
      return std::nullopt;
    }
    osmh::set(diagnostic, impl->slab_mode()
                              ? "resident expert uploaded into an HBM expert slab slot"
                              : "resident expert created with gate/up/down weights preloaded");
    return VulkanResidentExpert(std::move(impl));
  } catch (const std::exception& e) {
    osmh::set(diagnostic, std::string("resident expert creation exception: ") + e.what());
    return std::nullopt;
  } catch (...) {
    osmh::set(diagnostic, "resident expert creation encountered an unknown exception");
    return std::nullopt;
  }
}

bool VulkanResidentExpert::valid() const noexcept {
  if (!impl_ || !impl_->ctx || !impl_->input || !impl_->output) return false;
  if (impl_->slab_mode()) return impl_->slot >= 0;
  return impl_->gate_w && impl_->up_w && impl_->down_w && impl_->gate && impl_->up &&
         impl_->hidden;
}
std::size_t VulkanResidentExpert::input_dim() const noexcept { return impl_ ? impl_->g.in : 0; }
std::size_t VulkanResidentExpert::intermediate_dim() const noexcept {
  return impl_ ? impl_->g.inter : 0;
}
std::size_t VulkanResidentExpert::output_dim() const noexcept { return impl_ ? impl_->g.out : 0; }
std::size_t VulkanResidentExpert::packed_weight_bytes() const noexcept {
  return valid() ? impl_->g.packed_words * 4 : 0;
}
std::size_t VulkanResidentExpert::accounted_bytes() const noexcept {
  return valid() ? accounted(impl_->g) : 0;
}
std::uintptr_t VulkanResidentExpert::native_device() const noexcept {
  return impl_ ? reinterpret_cast<std::uintptr_t>(impl_->ctx) : 0;
}
std::int32_t VulkanResidentExpert::slab_slot() const noexcept {
  return impl_ && impl_->slab_mode() ? impl_->slot : -1;
}

osm_slab* VulkanResidentExpert::slab() const noexcept { return impl_ ? impl_->slab : nullptr; }
const VulkanFloatBuffer* VulkanResidentExpert::output_buffer() const noexcept {
  return valid() ? &*impl_->output : nullptr;
}

VulkanBufferDispatchResult VulkanResidentExpert::run_from_buffer(VulkanComputeContext& context,
                                                                 const VulkanFloatBuffer& x) noexcept {
  VulkanBufferDispatchResult r;
  if (!valid()) {
    r.diagnostic = "resident expert is not valid";
    return r;
  }
  if (!context.valid() || context.native_device() != native_device()) {
    r.diagnostic = "resident expert belongs to a different compute context";
    return r;
  }
  if (!x.valid() || x.native_device() != native_device() || x.size() != impl_->g.in) {
    r.diagnostic = "resident expert input buffer is invalid or has wrong shape/device";
    return r;
  }
  if (impl_->slab_mode()) {
    osm_context* ctx = impl_->ctx;
    int rc = osm_expert_forward(ctx, osm_slab_slot_ptr(impl_->slab, (uint32_t)impl_->slot),
                                &impl_->layout, x.device_data(), 1, impl_->output->device_data());
    if (rc == OSM_OK) rc = osm_context_synchronize(ctx);
    if (rc != OSM_OK) {
      r.diagnostic = osmh::err(ctx, rc, "resident expert forward failed");
      return r;
    }
    r.executed = true;
    r.diagnostic = "resident expert output remains in its reusable device buffer";
    return r;
  }
  const auto gate = run_vulkan_q4_gemv_preloaded(context, *impl_->gate_w, x, *impl_->gate);
  if (!gate.executed) {
    r.diagnostic = "resident expert gate projection failed: " + gate.diagnostic;
    return r;
  }
  const auto up = run_vulkan_q4_gemv_preloaded(context, *impl_->up_w, x, *impl_->up);
  if (!up.executed) {
    r.diagnostic = "resident expert up projection failed: " + up.diagnostic;
    return r;
  }
  const auto h = run_vulkan_swiglu_buffers(context, *impl_->gate, *impl_->up, *impl_->hidden);
  if (!h.executed) {
    r.diagnostic = "resident expert SwiGLU failed: " + h.diagnostic;
    return r;
  }
  const auto down = run_vulkan_q4_gemv_preloaded(context, *impl_->down_w, *impl_->hidden,
                                                 *impl_->output);
  if (!down.executed) {
    r.diagnostic = "resident expert down projection failed: " + down.diagnostic;
    return r;
  }
  r.executed = true;
  r.diagnostic = "resident expert output remains in its reusable device buffer";
  return r;
}

VulkanResidentExpertResult VulkanResidentExpert::run(VulkanComputeContext& context,
                                                     std::span<const float> x) noexcept {
  VulkanResidentExpertResult r;
  if (!valid()) {
    r.diagnostic = "resident expert is not valid";
    return r;
  }
  if (!context.valid() || context.native_device() != native_device()) {
    r.diagnostic = "resident expert belongs to a different compute context";
    return r;
  }
  if (x.size() != impl_->g.in) {
    r.diagnostic = "resident expert input size mismatch";
    return r;
  }
  std::string d;
  if (!impl_->input->upload(x, &d)) {
    r.diagnostic = "resident expert input upload failed: " + d;
    return r;
  }
  const auto disp = run_from_buffer(context, *impl_->input);
  if (!disp.executed) {
    r.diagnostic = disp.diagnostic;
    return r;
  }
  auto values = impl_->output->download(&d);
  if (!values) {
    r.diagnostic = "resident expert output download failed: " + d;
    return r;
  }
  r.values = std::move(*values);
  r.executed = true;
  r.diagnostic = "resident expert executed through its reusable buffers";
  return r;
}

// ---------------------------------------------------------------------------
// VulkanResidentExpertCache
// ---------------------------------------------------------------------------
struct VulkanResidentExpertCache::Impl {
  VulkanComputeContext& context;
  const QpackReader& reader;
  ExpertCache& host_cache;
  std::size_t budget;

  struct Node {
    std::unique_ptr<VulkanResidentExpert> resident;
    std::size_t accounted = 0;
    std::size_t frequency = 0;
    std::uint64_t last_use = 0;
  };
  std::map<std::uint64_t, Node> entries;  // ordered: deterministic victim ties
  std::unordered_map<std::uint64_t, std::size_t> frequency_history;
  std::uint64_t tick = 0;
  std::size_t hits = 0, misses = 0, loads = 0, evictions = 0, resident_bytes = 0;

  // The slab (created at the first miss whose expert has a slab layout):
  // budget / accounted slots for residents plus one to upload a newcomer
  // into before anything is evicted.
  osm_slab* slab = nullptr;
  osm_expert_layout layout{};
  std::vector<std::uint32_t> free_slots;

  Impl(VulkanComputeContext& c, const QpackReader& r, ExpertCache& h, std::size_t b)
      : context(c), reader(r), host_cache(h), budget(b) {}
  ~Impl() {
    entries.clear();  // residents before the slab they point into
    if (slab) osm_slab_destroy(slab);
  }

  static std::uint64_t key(std::uint32_t layer, std::uint32_t expert) {
    return (static_cast<std::uint64_t>(layer) << 32) | expert;
  }

  std::uint64_t victim() const {
    if (entries.empty()) throw std::runtime_error("resident expert cache: no eviction victim");
    auto best = std::tuple{std::numeric_limits<std::size_t>::max(),
                           std::numeric_limits<std::uint64_t>::max(),
                           std::numeric_limits<std::uint64_t>::max()};
    std::uint64_t v = 0;
    bool have = false;
    for (const auto& [k, n] : entries) {
      const auto score = std::tuple{n.frequency, n.last_use, k};
      if (!have || score < best) {
        best = score;
        v = k;
        have = true;
      }
    }
    return v;
  }

  // Returns a resident's slot to the free list when it lives in this cache's
  // slab (an expert of another geometry holds a one-slot slab of its own).
  void release(const VulkanResidentExpert& r) {
    if (slab && r.slab() == slab && r.slab_slot() >= 0)
      free_slots.push_back(static_cast<std::uint32_t>(r.slab_slot()));
  }

  // Whether this entry goes into a slab slot; creates the slab, sized for
  // its geometry, at the first such entry.
  bool use_slab(const ExpertCacheEntry& entry) {
    Geometry geo;
    osm_expert_layout L{};
    if (!slab_eligible(reader, entry, &geo, &L)) return false;
    if (slab) return std::memcmp(&L, &layout, sizeof(L)) == 0 && !free_slots.empty();
    layout = L;
    const std::size_t per = accounted(geo);
    const std::size_t fit = per ? budget / per : 0;
    const std::size_t slots = std::min<std::size_t>(fit, 1u << 20) + 1;
    const int rc = osm_slab_create(context.osm(), &layout, static_cast<std::uint32_t>(slots), &slab);
    if (rc != OSM_OK) {
      slab = nullptr;
      throw std::runtime_error(
          osmh::err(context.osm(), rc, "resident expert cache: slab allocation failed"));
    }
    free_slots.clear();
    for (std::size_t s = slots; s-- > 0;) free_slots.push_back(static_cast<std::uint32_t>(s));
    return true;
  }
};

VulkanResidentExpertCache::VulkanResidentExpertCache(VulkanComputeContext& context,
                                                     const QpackReader& reader,
                                                     ExpertCache& host_cache,
                                                     std::size_t budget_bytes) {
  if (!context.valid())
    throw std::invalid_argument("resident expert cache: compute context must be valid");
  if (budget_bytes == 0) throw std::invalid_argument("resident expert cache: budget must be non-zero");
  impl_ = std::make_unique<Impl>(context, reader, host_cache, budget_bytes);
}

VulkanResidentExpertCache::~VulkanResidentExpertCache() = default;

VulkanResidentExpert* VulkanResidentExpertCache::get(std::uint32_t layer, std::uint32_t expert,
                                                     std::string* diagnostic) noexcept {
  auto& m = *impl_;
  try {
    ++m.tick;
    const auto k = Impl::key(layer, expert);
    const auto freq = ++m.frequency_history[k];
    if (auto it = m.entries.find(k); it != m.entries.end()) {
      ++m.hits;
      it->second.frequency = freq;
      it->second.last_use = m.tick;
      osmh::set(diagnostic, "resident expert cache hit");
      return it->second.resident.get();
    }
    ++m.misses;

    // Fetch and upload before anything is evicted: a failed fetch or upload
    // leaves every resident in place.
    const std::vector<std::uint32_t> request{expert};
    const auto host_entries = m.host_cache.fetch(layer, request);
    if (host_entries.size() != 1) {
      osmh::set(diagnostic, "resident expert cache: host cache returned unexpected entry count");
      return nullptr;
    }
    std::string local;
    std::optional<VulkanResidentExpert> resident;
    if (m.use_slab(host_entries.front())) {
      const std::uint32_t slot = m.free_slots.back();
      resident = VulkanResidentExpert::create_in_slab(m.context, m.reader, host_entries.front(),
                                                      m.slab, slot, &local);
      if (resident) m.free_slots.pop_back();
    } else {
      resident = VulkanResidentExpert::create(m.context, m.reader, host_entries.front(), &local);
    }
    if (!resident) {
      osmh::set(diagnostic, "resident expert cache: upload failed: " + local);
      return nullptr;
    }
    const auto incoming = resident->accounted_bytes();
    if (incoming == 0) {
      m.release(*resident);
      osmh::set(diagnostic, "resident expert cache: resident expert byte accounting is zero");
      return nullptr;
    }
    if (incoming > m.budget) {
      m.release(*resident);
      osmh::set(diagnostic, "resident expert cache: one expert exceeds the configured budget");
      return nullptr;
    }
    while (!m.entries.empty() && m.resident_bytes + incoming > m.budget) {
      const auto it = m.entries.find(m.victim());
      m.resident_bytes -= it->second.accounted;
      m.release(*it->second.resident);
      m.entries.erase(it);
      ++m.evictions;
    }
    auto owned = std::make_unique<VulkanResidentExpert>(std::move(*resident));
    auto* out = owned.get();
    m.entries.emplace(k, Impl::Node{std::move(owned), incoming, freq, m.tick});
    m.resident_bytes += incoming;
    ++m.loads;
    osmh::set(diagnostic, "resident expert cache miss loaded into HBM");
    return out;
  } catch (const std::exception& e) {
    osmh::set(diagnostic, std::string("resident expert cache exception: ") + e.what());
    return nullptr;
  } catch (...) {
    osmh::set(diagnostic, "resident expert cache encountered an unknown exception");
    return nullptr;
  }
}

VulkanResidentExpertResult VulkanResidentExpertCache::run(std::uint32_t layer, std::uint32_t expert,
                                                          std::span<const float> x) noexcept {
  VulkanResidentExpertResult r;
  std::string d;
  auto* resident = get(layer, expert, &d);
  if (!resident) {
    r.diagnostic = d;
    return r;
  }
  r = resident->run(impl_->context, x);
  if (!r.executed && !d.empty()) r.diagnostic = d + "; execution: " + r.diagnostic;
  return r;
}

bool VulkanResidentExpertCache::contains(std::uint32_t layer, std::uint32_t expert) const noexcept {
  return impl_->entries.contains(Impl::key(layer, expert));
}

VulkanResidentExpertCacheStats VulkanResidentExpertCache::stats() const noexcept {
  const auto& m = *impl_;
  return {m.hits, m.misses, m.loads, m.evictions, m.entries.size(), m.resident_bytes, m.budget};
}

ExpertCacheStats VulkanResidentExpertCache::host_stats() const noexcept {
  return impl_->host_cache.stats();
}

osm_slab* VulkanResidentExpertCache::slab() const noexcept { return impl_->slab; }

VulkanComputeContext& VulkanResidentExpertCache::context() const noexcept { return impl_->context; }

// ---------------------------------------------------------------------------
// VulkanResidentSharedExpert
// ---------------------------------------------------------------------------
struct VulkanResidentSharedExpert::Impl {
  osm_context* ctx = nullptr;
  std::size_t in = 0, inter = 0, out = 0;
  std::optional<VulkanQ4ProjectionWeights> gate_w, up_w, down_w;
  std::optional<VulkanFloatBuffer> gate, up, hidden, output;
  std::vector<float> scalar_gate;
};

VulkanResidentSharedExpert::VulkanResidentSharedExpert() = default;
VulkanResidentSharedExpert::~VulkanResidentSharedExpert() = default;
VulkanResidentSharedExpert::VulkanResidentSharedExpert(VulkanResidentSharedExpert&&) noexcept =
    default;
VulkanResidentSharedExpert& VulkanResidentSharedExpert::operator=(
    VulkanResidentSharedExpert&&) noexcept = default;
VulkanResidentSharedExpert::VulkanResidentSharedExpert(std::unique_ptr<Impl> impl) noexcept
    : impl_(std::move(impl)) {}

namespace {

bool valid_projection(const VulkanSharedExpertProjectionView& v) {
  if (v.out_dim == 0 || v.packed_cols == 0 || v.group_size == 0) return false;
  const std::size_t in = v.packed_cols * 8;
  if (in % v.group_size) return false;
  const std::size_t groups = v.out_dim * (in / v.group_size);
  return v.packed.size() == v.out_dim * v.packed_cols && v.scales.size() == groups &&
         v.biases.size() == groups;
}

}  // namespace

std::optional<VulkanResidentSharedExpert> VulkanResidentSharedExpert::create(
    VulkanComputeContext& context, VulkanSharedExpertWeights w, std::string* diagnostic) noexcept {
  if (!context.valid()) {
    osmh::set(diagnostic, "shared expert requires a valid compute context");
    return std::nullopt;
  }
  try {
    if (!valid_projection(w.gate) || !valid_projection(w.up) || !valid_projection(w.down)) {
      osmh::set(diagnostic, "shared expert Q4 projection geometry is invalid");
      return std::nullopt;
    }
    const std::size_t in = w.gate.packed_cols * 8, inter = w.gate.out_dim, out = w.down.out_dim;
    if (w.up.packed_cols * 8 != in || w.up.out_dim != inter || w.down.packed_cols * 8 != inter ||
        out != in || w.scalar_gate.size() != in) {
      osmh::set(diagnostic, "shared expert gate/up/down/scalar geometry mismatch");
      return std::nullopt;
    }
    auto impl = std::make_unique<Impl>();
    impl->ctx = context.osm();
    impl->in = in;
    impl->inter = inter;
    impl->out = out;
    impl->scalar_gate.assign(w.scalar_gate.begin(), w.scalar_gate.end());
    std::string local;
    auto proj = [&](const VulkanSharedExpertProjectionView& v) {
      return VulkanQ4ProjectionWeights::create(context, v.packed, v.out_dim, v.packed_cols, v.scales,
                                               v.biases, v.group_size, &local);
    };
    impl->gate_w = proj(w.gate);
    if (!impl->gate_w) {
      osmh::set(diagnostic, "shared expert gate upload failed: " + local);
      return std::nullopt;
    }
    impl->up_w = proj(w.up);
    if (!impl->up_w) {
      osmh::set(diagnostic, "shared expert up upload failed: " + local);
      return std::nullopt;
    }
    impl->down_w = proj(w.down);
    if (!impl->down_w) {
      osmh::set(diagnostic, "shared expert down upload failed: " + local);
      return std::nullopt;
    }
    impl->gate = VulkanFloatBuffer::create(context, inter, &local);
    impl->up = VulkanFloatBuffer::create(context, inter, &local);
    impl->hidden = VulkanFloatBuffer::create(context, inter, &local);
    impl->output = VulkanFloatBuffer::create(context, out, &local);
    if (!impl->gate || !impl->up || !impl->hidden || !impl->output) {
      osmh::set(diagnostic, "shared expert activation allocation failed: " + local);
      return std::nullopt;
    }
    osmh::set(diagnostic, "shared expert created with resident Q4 projections");
    return VulkanResidentSharedExpert(std::move(impl));
  } catch (const std::exception& e) {
    osmh::set(diagnostic, std::string("shared expert creation exception: ") + e.what());
    return std::nullopt;
  } catch (...) {
    osmh::set(diagnostic, "shared expert creation encountered an unknown exception");
    return std::nullopt;
  }
}

bool VulkanResidentSharedExpert::valid() const noexcept {
  return impl_ && impl_->ctx && impl_->gate_w && impl_->up_w && impl_->down_w && impl_->gate &&
         impl_->up && impl_->hidden && impl_->output && impl_->scalar_gate.size() == impl_->in;
}
std::size_t VulkanResidentSharedExpert::input_dim() const noexcept { return impl_ ? impl_->in : 0; }
std::size_t VulkanResidentSharedExpert::intermediate_dim() const noexcept {
  return impl_ ? impl_->inter : 0;
}
std::size_t VulkanResidentSharedExpert::output_dim() const noexcept { return impl_ ? impl_->out : 0; }

std::size_t VulkanResidentSharedExpert::accounted_vulkan_bytes() const noexcept {
  if (!valid()) return 0;
  auto proj = [](const VulkanQ4ProjectionWeights& w) {
    return w.packed_size_bytes() + w.scales_buffer().size_bytes() + w.biases_buffer().size_bytes();
  };
  return proj(*impl_->gate_w) + proj(*impl_->up_w) + proj(*impl_->down_w) +
         impl_->gate->size_bytes() + impl_->up->size_bytes() + impl_->hidden->size_bytes() +
         impl_->output->size_bytes();
}

std::uintptr_t VulkanResidentSharedExpert::native_device() const noexcept {
  return impl_ ? reinterpret_cast<std::uintptr_t>(impl_->ctx) : 0;
}

std::optional<float> VulkanResidentSharedExpert::scalar_scale(std::span<const float> hidden,
                                                              std::string* diagnostic) const noexcept {
  if (!valid()) {
    osmh::set(diagnostic, "shared expert is not valid");
    return std::nullopt;
  }
  if (hidden.size() != impl_->in) {
    osmh::set(diagnostic, "shared expert scalar gate input size mismatch");
    return std::nullopt;
  }
  // one sequential fp32 dot, then the logistic function
  float logit = 0.0f;
  for (std::size_t i = 0; i < hidden.size(); ++i) logit += impl_->scalar_gate[i] * hidden[i];
  const float scale = 1.0f / (1.0f + std::exp(-logit));
  if (!std::isfinite(scale)) {
    osmh::set(diagnostic, "shared expert scalar gate is non-finite");
    return std::nullopt;
  }
  osmh::set(diagnostic, "shared expert scalar gate computed");
  return scale;
}

VulkanBufferDispatchResult VulkanResidentSharedExpert::run_from_buffer(
    VulkanComputeContext& context, const VulkanFloatBuffer& hidden) noexcept {
  VulkanBufferDispatchResult r;
  if (!valid()) {
    r.diagnostic = "shared expert is not valid";
    return r;
  }
  if (!context.valid() || context.native_device() != native_device() || !hidden.valid() ||
      hidden.native_device() != native_device() || hidden.size() != impl_->in) {
    r.diagnostic = "shared expert input buffer has wrong device or geometry";
    return r;
  }
  const auto g = run_vulkan_q4_gemv_preloaded(context, *impl_->gate_w, hidden, *impl_->gate);
  if (!g.executed) {
    r.diagnostic = "shared expert gate projection failed: " + g.diagnostic;
    return r;
  }
  const auto u = run_vulkan_q4_gemv_preloaded(context, *impl_->up_w, hidden, *impl_->up);
  if (!u.executed) {
    r.diagnostic = "shared expert up projection failed: " + u.diagnostic;
    return r;
  }
  const auto s = run_vulkan_swiglu_buffers(context, *impl_->gate, *impl_->up, *impl_->hidden);
  if (!s.executed) {
    r.diagnostic = "shared expert SwiGLU failed: " + s.diagnostic;
    return r;
  }
  const auto d = run_vulkan_q4_gemv_preloaded(context, *impl_->down_w, *impl_->hidden,
                                              *impl_->output);
  if (!d.executed) {
    r.diagnostic = "shared expert down projection failed: " + d.diagnostic;
    return r;
  }
  r.executed = true;
  r.diagnostic = "shared expert output remains in its reusable device buffer";
  return r;
}

const VulkanFloatBuffer* VulkanResidentSharedExpert::output_buffer() const noexcept {
  return valid() ? &*impl_->output : nullptr;
}

}  // namespace orbi::streammoe
