// The tier planner: which units are resident on the device, which stream from the pinned host tier, which from their
// files; plus the device bytes of the stream rings and the exclusive mode's spare pinned blocks. The placement rule
// and every total are the reference planner's (plan.cpp), so a descriptor and a budget give the same plan.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "desc.hpp"
#include "json.hpp"
#include "strix_stream/ss.h"

namespace tsb {

struct RingClass {
  uint64_t stride = 0;  // device bytes of one slot (a unit stride)
  uint32_t slots = 0;
};

// Pinned copies packed in model order at 4 KiB strides into chunks of at most 1 GiB (a larger unit gets a chunk alone).
struct PinnedLayout {
  std::vector<uint64_t> chunk_bytes;
  std::vector<int32_t> chunk_of;    // per global unit; -1 = no pinned copy
  std::vector<uint64_t> offset_of;  // per global unit, inside its chunk
  uint64_t total = 0;
};

struct SpareClass {
  uint64_t block_bytes = 0;
  uint32_t asked = 0, blocks = 0;
};

struct Plan {
  std::vector<uint8_t> tier;  // per global unit: ss_tier
  ss_budget budget{};
  uint64_t cap = 0, margin = 0, fixed = 0, dynamic = 0, ring = 0, resident = 0, pinned = 0, disk = 0, peak = 0;
  uint64_t n_resident = 0, n_pinned = 0, n_disk = 0, n_pair = 0, n_backed = 0;
  std::vector<RingClass> rings;
  std::vector<SpareClass> spares;
  uint32_t dynamic_slots_per_layer = 0;
};

constexpr uint64_t kGiB = uint64_t(1) << 30;

uint64_t host_stride(uint64_t bytes);  // pinned bytes of one unit (4 KiB rounded)
uint64_t plan_margin(const ss_budget& b);
bool same_budget(const ss_budget& a, const ss_budget& b);
PinnedLayout pinned_layout(const Desc& d, const std::vector<uint8_t>& tier);
Plan plan_make(const Desc& d, const ss_budget& b, const std::vector<double>& benefit);
Plan plan_from_tiers(const Desc& d, const ss_budget& b, const std::vector<uint8_t>& tiers);
Json plan_to_json(const Desc& d, const Plan& p);
std::vector<uint8_t> tiers_from_json(const Desc& d, const Json& plan_json);

}  // namespace tsb
