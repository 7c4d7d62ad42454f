#include "plan.hpp"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <limits>

#include "errors.hpp"

namespace tsb {
namespace {

constexpr uint64_t kPage = 4096;
constexpr uint64_t kChunkCap = uint64_t(1) << 30;

struct Cand {
  int64_t g;        // global unit index (model order)
  int layer;
  uint64_t bytes;   // device stride
  double benefit;
};

std::string gib(uint64_t n) {
  char b[32];
  std::snprintf(b, sizeof b, "%.3f", double(n) / double(kGiB));
  return b;
}

double density(const Cand& c) {
  return c.bytes ? c.benefit / double(c.bytes) : std::numeric_limits<double>::infinity();
}
// Higher benefit per byte first; ties in model order.
bool denser(const Cand& a, const Cand& b) {
  const double x = density(a), y = density(b);
  return x != y ? x > y : a.g < b.g;
}
bool pinned_copy(uint8_t t) { return t == SS_TIER_PINNED || t == SS_TIER_RESIDENT_BACKED; }
bool exclusive(const ss_budget& b) { return b.tier_mode == SS_TIER_MODE_EXCLUSIVE; }

std::vector<Cand> candidates(const Desc& d, const std::vector<double>& benefit) {
  std::vector<Cand> out;
  for (size_t L = 0; L < d.layers.size(); ++L) {
    const Layer& l = d.layers[L];
    if (!l.streamable) continue;
    for (int u = 0; u < l.n_units; ++u) {
      const int64_t g = d.unit_base[L] + u;
      const double v = !benefit.empty() ? benefit[size_t(g)] : !l.benefit.empty() ? l.benefit[size_t(u)] : 1.0;
      require(std::isfinite(v) && v >= 0, SS_E_INVALID, "plan: benefit must be finite and >= 0");
      out.push_back({g, int(L), d.unit_stride(int(L)), v});
    }
  }
  return out;
}

uint64_t dynamic_upper(const Desc& d, const ss_budget& b) {
  uint64_t t = 0;
  if (!b.dynamic_slots_per_layer) return 0;
  for (size_t L = 0; L < d.layers.size(); ++L) {
    const Layer& l = d.layers[L];
    if (l.streamable && l.n_units > 0)
      t += uint64_t(std::min<uint32_t>(b.dynamic_slots_per_layer, uint32_t(l.n_units))) * d.unit_stride(int(L));
  }
  return t;
}

// One ring per distinct streamed unit stride; slots from the budget, else the descriptor, else twice the most units
// a layer of that stride has.
std::vector<RingClass> rings_of(const Desc& d, const ss_budget& b, const std::vector<Cand>& streamed) {
  std::vector<RingClass> out;
  for (const Cand& c : streamed) {
    if (d.tiers == Tiers::Pair || !c.bytes) continue;
    if (std::any_of(out.begin(), out.end(), [&](const RingClass& r) { return r.stride == c.bytes; })) continue;
    uint32_t slots = b.ring_slots ? b.ring_slots : d.ring_slots;
    if (!slots)
      for (size_t L = 0; L < d.layers.size(); ++L)
        if (d.layers[L].streamable && d.layers[L].n_units && d.unit_stride(int(L)) == c.bytes)
          slots = std::max(slots, uint32_t(2 * d.layers[L].n_units));
    out.push_back({c.bytes, slots});
  }
  std::sort(out.begin(), out.end(), [](const RingClass& x, const RingClass& y) { return x.stride < y.stride; });
  return out;
}

uint64_t ring_total(const std::vector<RingClass>& r) {
  uint64_t t = 0;
  for (const RingClass& c : r) t += c.stride * c.slots;
  return t;
}

std::vector<SpareClass> spares_of(const Desc& d, const ss_budget& b, uint64_t host_left) {
  std::vector<SpareClass> out;
  if (!exclusive(b)) return out;
  std::vector<std::pair<uint64_t, uint64_t>> per;  // host stride -> streamable units
  for (const Layer& l : d.layers) {
    if (!l.streamable || !l.n_units) continue;
    const uint64_t hs = host_stride(l.unit_bytes);
    auto it = std::find_if(per.begin(), per.end(), [&](const auto& x) { return x.first == hs; });
    if (it == per.end()) per.push_back({hs, uint64_t(l.n_units)});
    else it->second += uint64_t(l.n_units);
  }
  for (const auto& [hs, n] : per) {
    const uint64_t want = b.host_spare_units ? b.host_spare_units : 64;
    out.push_back({hs, uint32_t(std::min<uint64_t>(want, n)), 0});
  }
  std::sort(out.begin(), out.end(), [](const SpareClass& x, const SpareClass& y) { return x.block_bytes < y.block_bytes; });
  for (SpareClass& c : out) {
    c.blocks = uint32_t(std::min<uint64_t>(c.asked, host_left / c.block_bytes));
    host_left -= uint64_t(c.blocks) * c.block_bytes;
  }
  return out;
}

// The totals and capacity checks from the tiers alone (every figure is what a context allocates).
void totals(const Desc& d, const ss_budget& b, Plan& p) {
  std::vector<Cand> streamed;
  p.resident = p.pinned = p.disk = p.dynamic = 0;
  p.n_resident = p.n_pinned = p.n_disk = p.n_pair = p.n_backed = 0;
  for (size_t L = 0; L < d.layers.size(); ++L) {
    const Layer& l = d.layers[L];
    int planned = 0;
    for (int u = 0; u < l.n_units; ++u) {
      const int64_t g = d.unit_base[L] + u;
      const uint8_t t = p.tier[size_t(g)];
      require(t <= SS_TIER_RESIDENT_BACKED, SS_E_INVALID, "plan: bad tier value");
      if (!l.streamable) {
        require(t == SS_TIER_RESIDENT, SS_E_INVALID, "plan: a non-streamable layer's units must be resident");
        continue;
      }
      require(!(exclusive(b) && t == SS_TIER_RESIDENT_BACKED), SS_E_INVALID,
              "plan: tier B (resident with a pinned copy) is refused in the exclusive tier mode");
      if (t == SS_TIER_RESIDENT || t == SS_TIER_RESIDENT_BACKED) {
        p.resident += d.unit_stride(int(L));
        ++p.n_resident;
        ++planned;
        if (t == SS_TIER_RESIDENT_BACKED) ++p.n_backed;
        continue;
      }
      if (t != SS_TIER_PAIR) streamed.push_back({g, int(L), d.unit_stride(int(L)), 0.0});
      if (t == SS_TIER_PINNED) ++p.n_pinned;
      else if (t == SS_TIER_DISK) {
        p.disk += l.unit_bytes;
        ++p.n_disk;
      } else {
        ++p.n_pair;
      }
    }
    if (l.streamable && l.n_units > 0 && b.dynamic_slots_per_layer)
      p.dynamic += uint64_t(std::min<uint32_t>(b.dynamic_slots_per_layer, uint32_t(l.n_units - planned))) *
                   d.unit_stride(int(L));
  }
  const uint64_t laid = pinned_layout(d, p.tier).total;
  p.pinned = laid;
  for (const auto& n : d.host_fixed) p.pinned += n.bytes;
  require(p.pinned >= laid, SS_E_INVALID, "plan: host byte total overflows");
  p.spares = spares_of(d, b, b.host_pinned_bytes > p.pinned ? b.host_pinned_bytes - p.pinned : 0);
  for (const SpareClass& c : p.spares) p.pinned += c.block_bytes * c.blocks;
  p.rings = rings_of(d, b, streamed);
  p.ring = ring_total(p.rings);
  require(p.pinned <= b.host_pinned_bytes, SS_E_CAPACITY,
          d.engine + ": " + gib(p.pinned) + " GiB must be pinned on the host, above the host budget " +
              gib(b.host_pinned_bytes) + " GiB; raise the cap or the host budget");
  p.peak = p.fixed + p.dynamic + p.ring + p.resident;
  require(p.peak + p.margin <= p.cap, SS_E_CAPACITY,
          d.engine + ": predicted peak " + gib(p.peak) + " GiB above the cap " + gib(p.cap) + " GiB - margin " +
              gib(p.margin) + " GiB");
}

Plan first_checks(const Desc& d, const ss_budget& b) {
  require(b.device_bytes > 0, SS_E_INVALID, "plan: device budget must be > 0");
  require(b.tier_mode == SS_TIER_MODE_INCLUSIVE || b.tier_mode == SS_TIER_MODE_EXCLUSIVE, SS_E_INVALID,
          "plan: tier_mode must be SS_TIER_MODE_INCLUSIVE or SS_TIER_MODE_EXCLUSIVE");
  if (exclusive(b)) {
    require(!b.pinned_backing, SS_E_INVALID, "plan: pinned_backing is refused in the exclusive tier mode");
    require(d.tiers == Tiers::Pinned || d.tiers == Tiers::PinnedDisk, SS_E_INVALID,
            d.engine + ": the exclusive tier mode needs a descriptor whose tiers allow pinned (it says \"" +
                std::string(tiers_name(d.tiers)) + "\")");
  }
  Plan p;
  p.budget = b;
  p.cap = b.device_bytes;
  p.margin = plan_margin(b);
  p.tier.assign(size_t(d.total_units), SS_TIER_RESIDENT);
  p.dynamic_slots_per_layer = b.dynamic_slots_per_layer;
  p.fixed = d.fixed_total() + b.workspace_bytes;
  p.dynamic = dynamic_upper(d, b);
  require(p.cap >= p.margin + p.fixed + p.dynamic, SS_E_CAPACITY,
          d.engine + ": fixed device memory " + gib(p.fixed) + " GiB + dynamic slots " + gib(p.dynamic) +
              " GiB + margin " + gib(p.margin) + " GiB exceeds the " + gib(p.cap) + " GiB cap");
  return p;
}

void backing(const Desc& d, const ss_budget& b, const std::vector<double>& benefit, std::vector<uint8_t>& tier) {
  uint64_t left = b.host_pinned_bytes;
  for (const auto& n : d.host_fixed) left = left > n.bytes ? left - n.bytes : 0;
  std::vector<Cand> res;
  for (const Cand& c : candidates(d, benefit)) {
    const uint8_t t = tier[size_t(c.g)];
    if (t == SS_TIER_PINNED) {
      const uint64_t hb = host_stride(d.layers[size_t(c.layer)].unit_bytes);
      left = left > hb ? left - hb : 0;
    } else if (t == SS_TIER_RESIDENT) {
      res.push_back(c);
    }
  }
  std::stable_sort(res.begin(), res.end(), [](const Cand& x, const Cand& y) { return denser(y, x); });
  for (const Cand& c : res) {
    const uint64_t hb = host_stride(d.layers[size_t(c.layer)].unit_bytes);
    if (hb > left) break;
    tier[size_t(c.g)] = SS_TIER_RESIDENT_BACKED;
    left -= hb;
  }
}

}  // namespace

uint64_t host_stride(uint64_t bytes) {
  require(bytes <= UINT64_MAX - (kPage - 1), SS_E_INVALID, "plan: unit bytes overflow the host stride");
  return (bytes + kPage - 1) / kPage * kPage;
}

uint64_t plan_margin(const ss_budget& b) {
  return uint64_t(std::max(b.margin_gib * double(kGiB), b.margin_fraction * double(b.device_bytes)));
}

bool same_budget(const ss_budget& a, const ss_budget& b) {
  return a.device_bytes == b.device_bytes && a.host_pinned_bytes == b.host_pinned_bytes &&
         a.workspace_bytes == b.workspace_bytes && a.margin_gib == b.margin_gib &&
         a.margin_fraction == b.margin_fraction && a.dynamic_slots_per_layer == b.dynamic_slots_per_layer &&
         a.ring_slots == b.ring_slots && a.pinned_backing == b.pinned_backing && a.tier_mode == b.tier_mode &&
         a.host_spare_units == b.host_spare_units;
}

PinnedLayout pinned_layout(const Desc& d, const std::vector<uint8_t>& tier) {
  PinnedLayout pl;
  pl.chunk_of.assign(size_t(d.total_units), -1);
  pl.offset_of.assign(size_t(d.total_units), 0);
  uint64_t used = 0;
  bool open = false;
  for (size_t L = 0; L < d.layers.size(); ++L) {
    const uint64_t stride = host_stride(d.layers[L].unit_bytes);
    for (int u = 0; u < d.layers[L].n_units; ++u) {
      const int64_t g = d.unit_base[L] + u;
      if (!pinned_copy(tier[size_t(g)])) continue;
      if (!open || (used > 0 && used + stride > kChunkCap)) {
        if (open) pl.chunk_bytes.push_back(used);
        used = 0;
        open = true;
      }
      pl.chunk_of[size_t(g)] = int32_t(pl.chunk_bytes.size());
      pl.offset_of[size_t(g)] = used;
      used += stride;
    }
  }
  if (open) pl.chunk_bytes.push_back(used);
  for (uint64_t c : pl.chunk_bytes) {
    require(pl.total <= UINT64_MAX - c, SS_E_INVALID, "plan: pinned layout overflows");
    pl.total += c;
  }
  return pl;
}

Plan plan_make(const Desc& d, const ss_budget& b, const std::vector<double>& benefit) {
  require(benefit.empty() || int64_t(benefit.size()) == d.total_units, SS_E_INVALID,
          "plan: benefit needs one value per unit (ss_desc_total_units)");
  Plan p = first_checks(d, b);
  const std::vector<Cand> units = candidates(d, benefit);
  uint64_t room = p.cap - p.margin - p.fixed - p.dynamic;
  std::vector<char> chosen(units.size(), 0);
  uint64_t total = 0;
  for (const Cand& c : units) total += c.bytes;
  bool ok = false;
  if (d.order == Order::Prefix) {
    // the longest prefix whose bytes plus the rings of the units after it fit
    for (size_t k = units.size() + 1; k-- > 0;) {
      const std::vector<Cand> rest(units.begin() + std::ptrdiff_t(k), units.end());
      if (total + ring_total(rings_of(d, b, rest)) <= room) {
        std::fill(chosen.begin(), chosen.begin() + std::ptrdiff_t(k), char(1));
        ok = true;
        break;
      }
      if (k) total -= units[k - 1].bytes;
    }
  } else if (total <= room) {
    std::fill(chosen.begin(), chosen.end(), char(1));
    ok = true;
  } else {
    // rings for every unit size first, then the densest units while they fit (ties in model order)
    const uint64_t ring = ring_total(rings_of(d, b, units));
    if (ring <= room) {
      room -= ring;
      std::vector<size_t> order(units.size());
      for (size_t i = 0; i < order.size(); ++i) order[i] = i;
      std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t c) { return denser(units[a], units[c]); });
      uint64_t used = 0;
      for (size_t i : order)
        if (used + units[i].bytes <= room) {
          chosen[i] = 1;
          used += units[i].bytes;
        }
      ok = true;
    }
  }
  require(ok, SS_E_CAPACITY,
          d.engine + ": nothing fits under the " + gib(p.cap) + " GiB cap: fixed " + gib(p.fixed) + " GiB + margin " +
              gib(p.margin) + " GiB + the stream rings exceed it");
  uint64_t host_left = b.host_pinned_bytes;
  for (const auto& n : d.host_fixed) host_left = host_left > n.bytes ? host_left - n.bytes : 0;
  std::vector<Cand> spill;
  for (size_t i = 0; i < units.size(); ++i) {
    if (chosen[i]) continue;
    const Cand& c = units[i];
    uint8_t& t = p.tier[size_t(c.g)];
    switch (d.tiers) {
      case Tiers::Pinned: {
        t = SS_TIER_PINNED;
        const uint64_t hb = host_stride(d.layers[size_t(c.layer)].unit_bytes);
        host_left = host_left > hb ? host_left - hb : 0;
        break;
      }
      case Tiers::Disk: t = SS_TIER_DISK; break;
      case Tiers::Pair: t = SS_TIER_PAIR; break;
      case Tiers::PinnedDisk: spill.push_back(c); break;
    }
  }
  std::stable_sort(spill.begin(), spill.end(), denser);
  for (const Cand& c : spill) {
    const uint64_t hb = host_stride(d.layers[size_t(c.layer)].unit_bytes);
    if (hb <= host_left) {
      p.tier[size_t(c.g)] = SS_TIER_PINNED;
      host_left -= hb;
    } else {
      p.tier[size_t(c.g)] = SS_TIER_DISK;
    }
  }
  if (b.pinned_backing) backing(d, b, benefit, p.tier);
  totals(d, b, p);
  return p;
}

Plan plan_from_tiers(const Desc& d, const ss_budget& b, const std::vector<uint8_t>& tiers) {
  require(int64_t(tiers.size()) == d.total_units, SS_E_INVALID, "plan: one tier per unit (ss_desc_total_units)");
  Plan p = first_checks(d, b);
  p.tier = tiers;
  totals(d, b, p);
  return p;
}

Json plan_to_json(const Desc& d, const Plan& p) {
  Json j = Json::object();
  j["schema"] = Json::string("strix-stream/plan-v1");
  j["engine"] = Json::string(d.engine);
  j["cap_bytes"] = Json::number(p.cap);
  j["margin_bytes"] = Json::number(p.margin);
  j["fixed_bytes"] = Json::number(p.fixed);
  j["dynamic_bytes"] = Json::number(p.dynamic);
  j["dynamic_slots_per_layer"] = Json::number(uint64_t(p.dynamic_slots_per_layer));
  j["ring_bytes"] = Json::number(p.ring);
  Json rings = Json::array();
  for (const RingClass& c : p.rings) {
    Json r = Json::object();
    r["slot_bytes"] = Json::number(c.stride);
    r["slots"] = Json::number(uint64_t(c.slots));
    rings.push(r);
  }
  j["rings"] = rings;
  j["resident_bytes"] = Json::number(p.resident);
  j["pinned_bytes"] = Json::number(p.pinned);
  j["disk_bytes"] = Json::number(p.disk);
  j["peak_bytes"] = Json::number(p.peak);
  j["n_resident"] = Json::number(p.n_resident);
  j["n_pinned"] = Json::number(p.n_pinned);
  j["n_disk"] = Json::number(p.n_disk);
  j["n_pair"] = Json::number(p.n_pair);
  j["n_backed"] = Json::number(p.n_backed);
  if (exclusive(p.budget)) {
    j["tier_mode"] = Json::string("exclusive");
    Json sp = Json::array();
    for (const SpareClass& c : p.spares) {
      Json x = Json::object();
      x["block_bytes"] = Json::number(c.block_bytes);
      x["asked"] = Json::number(uint64_t(c.asked));
      x["blocks"] = Json::number(uint64_t(c.blocks));
      sp.push(x);
    }
    j["spare_blocks"] = sp;
  }
  Json layers = Json::array();
  for (size_t L = 0; L < d.layers.size(); ++L) {
    std::string s;
    for (int u = 0; u < d.layers[L].n_units; ++u) s += "RPDXB"[p.tier[size_t(d.unit_base[L] + u)]];
    layers.push(Json::string(s));
  }
  j["tiers"] = layers;
  return j;
}

std::vector<uint8_t> tiers_from_json(const Desc& d, const Json& j) {
  static const char kLetters[] = "RPDXB";
  const Json* t = j.find("tiers");
  require(t && t->is_array() && t->arr.size() == d.layers.size(), SS_E_DESC,
          "plan json: \"tiers\" needs one string per layer");
  std::vector<uint8_t> out;
  for (size_t L = 0; L < d.layers.size(); ++L) {
    const std::string s = json_str(t->arr[L], "plan.tiers");
    require(s.size() == size_t(d.layers[L].n_units), SS_E_DESC,
            "plan json: tiers[" + std::to_string(L) + "] needs one letter per unit");
    for (char c : s) {
      const char* k = c ? std::strchr(kLetters, c) : nullptr;
      require(k != nullptr, SS_E_DESC, "plan json: tier letters are R P D X B");
      out.push_back(uint8_t(k - kLetters));
    }
  }
  return out;
}

}  // namespace tsb
