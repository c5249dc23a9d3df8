// The drop-in's routed-MoE entry points (src/routed_moe.cpp here) against the
// reference's CPU path on the same inputs: route_qwen_top_k_cpu for the
// routing (ids and logits bit-equal, weights and selected mass within 1e-6
// as the reference's own router tests allow), and the reference's CPU
// expert (cpu::dequantize_affine_rows, cpu::matvec_row_major,
// cpu::swiglu_inplace) plus run_shared_expert_cpu for the values (within
// 1e-4 of the largest magnitude).  It writes its own qpack container (16
// experts, hidden 256, intermediate 128, MLX-affine Q4 with group 64 and
// bf16 scale and bias, so the cache keeps the experts in its slab) and runs
//   * a cache large enough for every expert (all picks in the slab: the one
//     expert call), twice, checking hits and misses;
//   * a cache of one expert, where every pick's load evicts the previous
//     pick of the same call (the picks then run one by one from their slots);
//   * the two routed-only entry points;
//   * a router rewritten in place between calls (a new device router);
//   * non-finite and wrongly sized hidden vectors (executed == false).
// Without a CUDA device it prints the reference tests' "no compute device"
// PASS line, unless ORBI_REQUIRE_VULKAN_COMPUTE=1.
#include <algorithm>
#include <bit>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <iostream>
#include <limits>
#include <stdexcept>
#include <string>
#include <vector>

#include "orbi/streammoe/backend/vulkan_compute_context.hpp"
#include "orbi/streammoe/backend/vulkan_resident_expert_cache.hpp"
#include "orbi/streammoe/backend/vulkan_resident_shared_expert.hpp"
#include "orbi/streammoe/cache/expert_cache.hpp"
#include "orbi/streammoe/cpu/reference_ops.hpp"
#include "orbi/streammoe/model/qwen_router.hpp"
#include "orbi/streammoe/model/routed_moe.hpp"
#include "orbi/streammoe/model/shared_expert.hpp"
#include "orbi/streammoe/storage/qpack_expert_storage.hpp"

namespace fs = std::filesystem;
using namespace orbi::streammoe;

namespace {

constexpr std::size_t kH = 256, kI = 128, kE = 16, kK = 4, kG = 64;
constexpr const char* kName = "routed MoE drop-in (device router, slab experts)";

void require(bool ok, const std::string& what) {
  if (!ok) throw std::runtime_error(what);
}

struct Rng {
  std::uint64_t s;
  std::uint32_t next() {
    s = s * 6364136223846793005ULL + 1442695040888963407ULL;
    return static_cast<std::uint32_t>(s >> 33);
  }
  float uniform() { return (next() & 0xFFFFFF) / 16777216.0F; }  // [0, 1)
  float normal() {
    float a = 0.0F;
    for (int i = 0; i < 12; ++i) a += uniform();
    return a - 6.0F;
  }
};

float bf16_round(float v) {
  auto u = std::bit_cast<std::uint32_t>(v);
  u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
  return std::bit_cast<float>(u);
}

// One Q4 projection [rows][cols]: packed nibbles, bf16-exact scale and bias
// per group of 64 inputs.
struct Proj {
  std::size_t rows = 0, cols = 0;
  std::vector<std::uint32_t> packed;
  std::vector<float> scales, biases;
};

Proj make_proj(Rng& r, std::size_t rows, std::size_t cols) {
  Proj p;
  p.rows = rows;
  p.cols = cols;
  p.packed.resize(rows * cols / 8);
  for (auto& w : p.packed) w = r.next() ^ (r.next() << 16);
  for (std::size_t i = 0; i < rows * cols / kG; ++i) {
    p.scales.push_back(bf16_round(0.004F + 0.002F * r.uniform()));
    p.biases.push_back(bf16_round(-0.03F + 0.0005F * r.normal()));
  }
  return p;
}

std::vector<float> dequant(const Proj& p) {
  return cpu::dequantize_affine_rows(p.packed, p.rows, p.cols / 8, p.scales, p.biases,
                                     cpu::AffineQuantSpec{.bits = 4, .group_size = kG});
}

void put_bf16(std::vector<char>& blob, std::size_t off, std::span<const float> v) {
  for (std::size_t i = 0; i < v.size(); ++i) {
    const auto b = static_cast<std::uint16_t>(std::bit_cast<std::uint32_t>(v[i]) >> 16);
    std::memcpy(blob.data() + off + 2 * i, &b, 2);
  }
}

struct Section {
  std::string name, dtype;
  std::size_t d0, d1, offset, size;
};

// Writes the container: per expert gate_proj, up_proj, down_proj (weight U32,
// scales and biases BF16), 64-byte aligned sections.
fs::path write_qpack(const fs::path& root, const std::vector<std::vector<Proj>>& experts) {
  fs::remove_all(root);
  fs::create_directories(root / "packed_experts");
  std::vector<Section> sections;
  std::size_t off = 0;
  auto add = [&](const std::string& n, const std::string& t, std::size_t d0, std::size_t d1,
                 std::size_t bytes) {
    sections.push_back({n, t, d0, d1, off, bytes});
    off = (off + bytes + 63) / 64 * 64;
  };
  const char* names[3] = {"gate_proj", "up_proj", "down_proj"};
  for (int p = 0; p < 3; ++p) {
    const Proj& q = experts[0][p];
    add(std::string(names[p]) + ".weight", "U32", q.rows, q.cols / 8, q.rows * q.cols / 2);
    add(std::string(names[p]) + ".scales", "BF16", q.rows, q.cols / kG, q.rows * q.cols / kG * 2);
    add(std::string(names[p]) + ".biases", "BF16", q.rows, q.cols / kG, q.rows * q.cols / kG * 2);
  }
  const std::size_t stride = off;
  {
    std::ofstream layer(root / "packed_experts" / "layer_00.bin", std::ios::binary);
    for (const auto& ex : experts) {
      std::vector<char> blob(stride, 0);
      for (int p = 0; p < 3; ++p) {
        const Proj& q = ex[p];
        std::memcpy(blob.data() + sections[3 * p].offset, q.packed.data(), q.packed.size() * 4);
        put_bf16(blob, sections[3 * p + 1].offset, q.scales);
        put_bf16(blob, sections[3 * p + 2].offset, q.biases);
      }
      layer.write(blob.data(), static_cast<std::streamsize>(blob.size()));
    }
  }
  {
    std::ofstream j(root / "packed_experts" / "layout.json");
    j << "{\"expertCount\": " << experts.size() << ", \"layerCount\": 1, \"expertStride\": "
      << stride << ", \"linearLayers\": [false], \"sections\": [";
    for (std::size_t i = 0; i < sections.size(); ++i) {
      const auto& s = sections[i];
      j << (i ? ", " : "") << "{\"name\": \"" << s.name << "\", \"dtype\": \"" << s.dtype
        << "\", \"shape\": [" << s.d0 << ", " << s.d1 << "], \"offset\": " << s.offset
        << ", \"size\": " << s.size << "}";
    }
    j << "]}\n";
  }
  const auto lsz = fs::file_size(root / "packed_experts" / "layout.json");
  const auto bsz = fs::file_size(root / "packed_experts" / "layer_00.bin");
  std::ofstream m(root / "manifest.json");
  m << "{\"magic\": \"QPACK\", \"version\": 1, \"modelName\": \"qwen3_next\", "
       "\"sourceCheckpoint\": \"routed-moe-dropin-fixture\", \"quantBits\": 4, "
       "\"quantGroupSize\": 64, \"files\": {\"packed_experts/layout.json\": "
    << lsz << ", \"packed_experts/layer_00.bin\": " << bsz << "}}\n";
  return root;
}

std::vector<float> cpu_expert(const std::vector<std::vector<float>>& w, std::span<const float> x) {
  auto h = cpu::matvec_row_major(w[0], kI, kH, x);
  const auto u = cpu::matvec_row_major(w[1], kI, kH, x);
  cpu::swiglu_inplace(h, u);
  return cpu::matvec_row_major(w[2], kH, kI, h);
}

void check_close(std::span<const float> got, std::span<const float> want, const std::string& what) {
  require(got.size() == want.size(), what + ": size mismatch");
  float mag = 0.0F, err = 0.0F;
  for (std::size_t i = 0; i < want.size(); ++i) {
    mag = std::max(mag, std::fabs(want[i]));
    err = std::max(err, std::fabs(got[i] - want[i]));
  }
  require(err <= 1e-4F * std::max(mag, 1.0F),
          what + ": max abs error " + std::to_string(err) + " (magnitude " + std::to_string(mag) + ")");
}

void check_routing(const QwenRouterResult& got, const QwenRouterResult& want, const std::string& what) {
  require(got.picks.size() == want.picks.size(), what + ": pick count");
  for (std::size_t j = 0; j < want.picks.size(); ++j) {
    require(got.picks[j].expert == want.picks[j].expert, what + ": pick " + std::to_string(j) + " id");
    require(std::fabs(got.picks[j].weight - want.picks[j].weight) <= 1e-6F,
            what + ": pick " + std::to_string(j) + " weight");
  }
  require(got.logits.size() == want.logits.size(), what + ": logit count");
  for (std::size_t e = 0; e < want.logits.size(); ++e)
    require(std::bit_cast<std::uint32_t>(got.logits[e]) == std::bit_cast<std::uint32_t>(want.logits[e]),
            what + ": logit " + std::to_string(e) + " not bit-equal");
  require(std::fabs(got.selected_probability_mass - want.selected_probability_mass) <= 1e-6F,
          what + ": selected mass");
}

}  // namespace

int main() {
  std::string diagnostic;
  auto context = VulkanComputeContext::create(&diagnostic);
  if (!context) {
    if (const char* v = std::getenv("ORBI_REQUIRE_VULKAN_COMPUTE"); v && std::string(v) == "1") {
      std::cerr << kName << ": FAIL: ORBI_REQUIRE_VULKAN_COMPUTE=1 but no context: " << diagnostic
                << "\n";
      return 1;
    }
    std::cout << kName << ": PASS (no compute device on host)\n";
    return 0;
  }
  const fs::path root = fs::temp_directory_path() / "orbi-streammoe-b200-routed-moe-dropin";
  try {
    Rng rng{0x5EED0001ULL};
    std::vector<std::vector<Proj>> experts(kE);
    std::vector<std::vector<std::vector<float>>> dense(kE);
    for (std::size_t e = 0; e < kE; ++e) {
      experts[e] = {make_proj(rng, kI, kH), make_proj(rng, kI, kH), make_proj(rng, kH, kI)};
      for (const auto& p : experts[e]) dense[e].push_back(dequant(p));
    }
    const std::vector<Proj> shared_q = {make_proj(rng, kI, kH), make_proj(rng, kI, kH),
                                        make_proj(rng, kH, kI)};
    std::vector<float> shared_gate_w(kH), router(kE * kH);
    for (auto& v : shared_gate_w) v = 0.02F * rng.normal();
    for (auto& v : router) v = bf16_round(0.02F * rng.normal());
    // two experts' rows made equal: a tie the router must break to the lower id
    std::copy_n(router.begin() + 3 * kH, kH, router.begin() + 9 * kH);
    std::vector<std::vector<float>> tokens(6, std::vector<float>(kH));
    for (auto& t : tokens)
      for (auto& v : t) v = rng.normal();

    QpackExpertStorage storage(write_qpack(root, experts));
    ExpertCache host_cache(storage, storage.expert_stride_bytes() * kE, kE);

    auto view = [](const Proj& p) {
      return VulkanSharedExpertProjectionView{p.packed, p.scales, p.biases, p.rows, p.cols / 8, kG};
    };
    auto shared = VulkanResidentSharedExpert::create(
        *context,
        VulkanSharedExpertWeights{view(shared_q[0]), view(shared_q[1]), view(shared_q[2]),
                                  shared_gate_w},
        &diagnostic);
    require(shared.has_value(), "shared expert creation failed: " + diagnostic);
    const auto sg = dequant(shared_q[0]), su = dequant(shared_q[1]), sd = dequant(shared_q[2]);

    const QwenRouterConfig cfg{.hidden_size = kH, .expert_count = kE, .top_k = kK,
                               .norm_topk_prob = true};
    auto oracle = [&](std::span<const float> x, const std::vector<float>& rw, bool with_shared,
                      QwenRouterResult* route) {
      *route = route_qwen_top_k_cpu(x, rw, cfg);
      std::vector<float> acc(kH, 0.0F);
      for (const auto& p : route->picks) {
        const auto y = cpu_expert(dense[p.expert], x);
        for (std::size_t i = 0; i < kH; ++i) acc[i] += p.weight * y[i];
      }
      if (with_shared) {
        const auto s = run_shared_expert_cpu(
            x, SharedExpertWeights{sg, su, sd, shared_gate_w},
            SharedExpertConfig{.hidden_size = kH, .intermediate_size = kI});
        require(s.executed, "CPU shared expert failed: " + s.diagnostic);
        for (std::size_t i = 0; i < kH; ++i) acc[i] += s.values[i];
      }
      return acc;
    };

    // 1. every expert fits: the picks run as one expert call
    {
      VulkanResidentExpertCache cache(*context, storage.reader(), host_cache, std::size_t{1} << 30);
      for (int pass = 0; pass < 2; ++pass)
        for (std::size_t t = 0; t < tokens.size(); ++t) {
          QwenRouterResult want;
          const auto ref = oracle(tokens[t], router, true, &want);
          const auto got = run_qwen_sparse_moe_vulkan_accum(*context, cache, *shared, 0, tokens[t],
                                                            router, cfg);
          const std::string what = "large cache, token " + std::to_string(t);
          require(got.executed, what + ": " + got.diagnostic);
          check_routing(got.routing, want, what);
          check_close(got.values, ref, what);
        }
      const auto st = cache.stats();
      require(st.evictions == 0, "large cache evicted");
      require(st.hits + st.misses == 2 * tokens.size() * kK, "one get() per pick");
      require(st.hits >= tokens.size() * kK, "second pass must hit every pick");
    }
    // 2. one expert fits: each pick's load evicts the previous pick
    {
      std::size_t one = 0;
      {
        VulkanResidentExpertCache probe(*context, storage.reader(), host_cache, std::size_t{1} << 30);
        auto* r = probe.get(0, 0, &diagnostic);
        require(r != nullptr, "probe load failed: " + diagnostic);
        one = r->accounted_bytes();
      }
      VulkanResidentExpertCache cache(*context, storage.reader(), host_cache, one);
      for (std::size_t t = 0; t < tokens.size(); ++t) {
        QwenRouterResult want;
        const auto ref = oracle(tokens[t], router, true, &want);
        const auto got = run_qwen_sparse_moe_vulkan_accum(*context, cache, *shared, 0, tokens[t],
                                                          router, cfg);
        const std::string what = "one-expert cache, token " + std::to_string(t);
        require(got.executed, what + ": " + got.diagnostic);
        check_routing(got.routing, want, what);
        check_close(got.values, ref, what);
      }
      const auto st = cache.stats();
      require(st.evictions >= tokens.size() * (kK - 1), "one-expert cache must evict within a call");
      require(st.resident_entries == 1, "one-expert cache holds one expert");
    }
    // 3. the routed-only entry points
    {
      VulkanResidentExpertCache cache(*context, storage.reader(), host_cache, std::size_t{1} << 30);
      for (std::size_t t = 0; t < 3; ++t) {
        QwenRouterResult want;
        const auto ref = oracle(tokens[t], router, false, &want);
        const auto a = run_weighted_routed_moe(cache, 0, tokens[t], router, cfg);
        require(a.executed, "weighted routed MoE: " + a.diagnostic);
        check_routing(a.routing, want, "weighted routed MoE");
        check_close(a.values, ref, "weighted routed MoE");
        const auto b = run_weighted_routed_moe_vulkan_accum(*context, cache, 0, tokens[t], router, cfg);
        require(b.executed, "device-accumulated routed MoE: " + b.diagnostic);
        check_routing(b.routing, want, "device-accumulated routed MoE");
        check_close(b.values, ref, "device-accumulated routed MoE");
      }
    }
    // 4. a router rewritten in place routes by its new contents
    {
      VulkanResidentExpertCache cache(*context, storage.reader(), host_cache, std::size_t{1} << 30);
      auto rw = router;
      QwenRouterResult before;
      oracle(tokens[0], rw, true, &before);
      const auto first = run_qwen_sparse_moe_vulkan_accum(*context, cache, *shared, 0, tokens[0], rw, cfg);
      require(first.executed, "rewrite, first call: " + first.diagnostic);
      const std::uint32_t top = before.picks[0].expert;
      for (std::size_t i = 0; i < kH; ++i) rw[top * kH + i] = -rw[top * kH + i];
      QwenRouterResult want;
      const auto ref = oracle(tokens[0], rw, true, &want);
      require(want.picks[0].expert != top, "fixture: negating the top row must change the top pick");
      const auto got = run_qwen_sparse_moe_vulkan_accum(*context, cache, *shared, 0, tokens[0], rw, cfg);
      require(got.executed, "rewrite, second call: " + got.diagnostic);
      check_routing(got.routing, want, "rewritten router");
      check_close(got.values, ref, "rewritten router");
    }
    // 5. rejected inputs
    {
      VulkanResidentExpertCache cache(*context, storage.reader(), host_cache, std::size_t{1} << 30);
      auto bad = tokens[0];
      bad[7] = std::numeric_limits<float>::quiet_NaN();
      const auto a = run_qwen_sparse_moe_vulkan_accum(*context, cache, *shared, 0, bad, router, cfg);
      require(!a.executed && a.diagnostic.find("non-finite") != std::string::npos,
              "non-finite hidden must fail: " + a.diagnostic);
      const std::vector<float> short_x(kH - 1, 0.5F);
      const auto b = run_weighted_routed_moe_vulkan_accum(*context, cache, 0, short_x, router, cfg);
      require(!b.executed, "a short hidden vector must fail");
      require(cache.stats().misses == 0, "rejected inputs must load nothing");
    }
  } catch (const std::exception& e) {
    std::cerr << kName << ": FAIL: " << e.what() << "\n";
    fs::remove_all(root);
    return 1;
  }
  fs::remove_all(root);
  std::cout << kName << ": PASS\n";
  return 0;
}
