// Scored eviction's profile: the transition counts an engine fitted offline, bound to the model it was fitted on. The
// format is the reference's (its docs' scored eviction section; ss.h "Scored eviction"), little endian:
//   "TSSCPRF1", u32 version 1, u32 n_gated, u32 units[n_gated], identity[32], u32 prov_len (<= 4096),
//   prov[prov_len], per gated layer units^2 u32 counts row-major [previous unit][unit], sha256[32] of all before.
// identity = sha256 of u32 n_gated, then per gated layer u32 model layer index, u32 units, u64 unit_bytes and the
// descriptor's per-unit xxh64 list. SHA-256 is FIPS 180-4's, written here from the standard.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "desc.hpp"

namespace tsb {

// The 32-byte SHA-256 digest of data (raw bytes).
std::string sha256(const void* data, size_t len);

// The profile identity of the gated layers (descriptor layer indices) of d; SS_E_INVALID when a gated layer lacks
// per-unit hashes.
std::string score_identity(const Desc& d, const std::vector<int>& gated);

struct ScoreProfile {
  std::vector<std::vector<uint32_t>> cells;  // per gated layer, units^2 counts
  std::string provenance;
};
// Every rule of the format (exact size, magic, version, layer and unit counts, identity, checksum); throws
// SS_E_INVALID naming the first one broken.
ScoreProfile check_score_profile(const void* data, uint64_t len, const std::vector<uint32_t>& units,
                                 const std::string& identity);

}  // namespace tsb
