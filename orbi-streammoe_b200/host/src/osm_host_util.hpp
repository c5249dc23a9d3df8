// Helpers shared by the host layer's translation units (not installed).
#pragma once

#include <cstdint>
#include <span>
#include <string>
#include <vector>

#include "osm_b200.h"

namespace orbi::streammoe::osmh {

// *d = v when d is non-null.
void set(std::string* d, std::string v);

// "<what> (osm status <rc>): <the context's last error>".
std::string err(osm_context* ctx, int rc, const char* what);

// The bf16 bits of v when v is exactly representable in bf16.
bool bf16_exact(float v, std::uint16_t* bits);

// Narrows fp32 affine metadata to the device's bf16 format; fails (with a
// diagnostic) on the first value bf16 cannot hold exactly.
bool narrow_bf16(std::span<const float> in, std::vector<std::uint16_t>& out, std::string* d,
                 const char* label);

}  // namespace orbi::streammoe::osmh
