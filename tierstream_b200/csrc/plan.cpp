// The tier planner (plan.hpp). Rules that decide a plan, each the reference planner's so the same descriptor and
// budget give the same tiers and totals (plan.cpp:104-408 there):
//   - a unit's benefit: the caller's array, else its layer's, else 1; finite and >= 0;
//   - the device room: cap - margin - fixed - the dynamic slots' upper bound;
//   - order "prefix": the longest model-order prefix resident whose bytes plus the rings of the rest fit;
//     otherwise all resident when they fit, else the rings of every unit size first and then the densest units
//     (benefit per device byte, ties in model order) greedily while they fit;
//   - units left over: pinned, on disk or paired as the descriptor's tiers say; "pinned+disk" spills the densest
//     into the pinned budget first;
//   - pinned_backing: the least dense residents (ties: the later unit) lose nothing but gain a pinned copy (tier B)
//     while the host budget lasts;
//   - rings: one per streamed device stride, slots from the budget, the descriptor, or twice the most units of a layer
//     of that stride; spare blocks (exclusive mode): per host stride min(asked, its units), granted smallest first;
//   - pinned copies packed in model order into chunks of at most 1 GiB.
#include "plan.hpp"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <limits>
#include <map>
#include <tuple>

#include "errors.hpp"

namespace tsb {
namespace {

constexpr uint64_t kPage = 4096;
constexpr uint64_t kChunkMax = uint64_t(1) << 30;

// One streamable unit as the planner sees it.
struct Item {
  int64_t key;        // global unit index, model order
  int layer;
  uint64_t dev;       // device bytes (its stride)
  double benefit;
  double per_byte() const { return dev ? benefit / double(dev) : std::numeric_limits<double>::infinity(); }
};

// The planner's preference: more benefit per byte first, model order among equals.
bool preferred(const Item& a, const Item& b) {
  const double x = a.per_byte(), y = b.per_byte();
  if (x != y) return x > y;
  return a.key < b.key;
}

std::string gib(uint64_t n) {
  char buf[32];
  std::snprintf(buf, sizeof buf, "%.3f", double(n) / double(kGiB));
  return buf;
}

uint64_t less_floor(uint64_t a, uint64_t b) { return a > b ? a - b : 0; }

bool has_pinned_copy(uint8_t t) { return t == SS_TIER_PINNED || t == SS_TIER_RESIDENT_BACKED; }

class Planner {
 public:
  Planner(const Desc& d, const ss_budget& b) : d_(d), b_(b) {}

  // The budget's own checks and the device room before any unit is placed.
  Plan open() const {
    require(b_.device_bytes > 0, SS_E_INVALID, "plan: device budget must be > 0");
    require(b_.tier_mode == SS_TIER_MODE_INCLUSIVE || b_.tier_mode == SS_TIER_MODE_EXCLUSIVE, SS_E_INVALID,
            "plan: tier_mode must be SS_TIER_MODE_INCLUSIVE or SS_TIER_MODE_EXCLUSIVE");
    if (exclusive()) {
      require(!b_.pinned_backing, SS_E_INVALID, "plan: pinned_backing is refused in the exclusive tier mode");
      require(d_.tiers == Tiers::Pinned || d_.tiers == Tiers::PinnedDisk, SS_E_INVALID,
              d_.engine + ": the exclusive tier mode needs a descriptor whose tiers allow pinned (it says \"" +
                  std::string(tiers_name(d_.tiers)) + "\")");
    }
    Plan p;
    p.budget = b_;
    p.cap = b_.device_bytes;
    p.margin = plan_margin(b_);
    p.tier.assign(size_t(d_.total_units), SS_TIER_RESIDENT);
    p.dynamic_slots_per_layer = b_.dynamic_slots_per_layer;
    p.fixed = d_.fixed_total() + b_.workspace_bytes;
    p.dynamic = 0;
    if (b_.dynamic_slots_per_layer)
      for_each_streamable_layer([&](int L, const Layer& l) {
        p.dynamic += uint64_t(std::min<uint32_t>(b_.dynamic_slots_per_layer, uint32_t(l.n_units))) *
                     d_.unit_stride(L);
      });
    require(p.cap >= p.margin + p.fixed + p.dynamic, SS_E_CAPACITY,
            d_.engine + ": fixed device memory " + gib(p.fixed) + " GiB + dynamic slots " + gib(p.dynamic) +
                " GiB + margin " + gib(p.margin) + " GiB exceeds the " + gib(p.cap) + " GiB cap");
    return p;
  }

  std::vector<Item> items(const std::vector<double>& benefit) const {
    std::vector<Item> out;
    for (size_t L = 0; L < d_.layers.size(); ++L) {
      const Layer& l = d_.layers[L];
      if (!l.streamable) continue;
      for (int u = 0; u < l.n_units; ++u) {
        const int64_t key = d_.unit_base[L] + u;
        double v = 1.0;
        if (!benefit.empty()) v = benefit[size_t(key)];
        else if (!l.benefit.empty()) v = l.benefit[size_t(u)];
        require(std::isfinite(v) && v >= 0, SS_E_INVALID, "plan: benefit must be finite and >= 0");
        out.push_back(Item{key, int(L), d_.unit_stride(int(L)), v});
      }
    }
    return out;
  }

  // The rings the units `streamed` need: stride -> slots (a map: ordered by stride).
  std::map<uint64_t, uint32_t> rings(const std::vector<Item>& streamed) const {
    std::map<uint64_t, uint32_t> out;
    if (d_.tiers == Tiers::Pair) return out;
    for (const Item& it : streamed) {
      if (!it.dev || out.count(it.dev)) continue;
      uint32_t slots = b_.ring_slots ? b_.ring_slots : d_.ring_slots;
      if (!slots)
        for_each_streamable_layer([&](int L, const Layer& l) {
          if (d_.unit_stride(L) == it.dev) slots = std::max(slots, uint32_t(2 * l.n_units));
        });
      out[it.dev] = slots;
    }
    return out;
  }
  static uint64_t ring_bytes(const std::map<uint64_t, uint32_t>& r) {
    uint64_t t = 0;
    for (const auto& [stride, slots] : r) t += stride * slots;
    return t;
  }

  // Every total and the two capacity checks, from the tiers alone.
  void close(Plan& p) const {
    std::vector<Item> streamed;
    p.resident = p.pinned = p.disk = p.dynamic = 0;
    p.n_resident = p.n_pinned = p.n_disk = p.n_pair = p.n_backed = 0;
    for (size_t L = 0; L < d_.layers.size(); ++L) {
      const Layer& l = d_.layers[L];
      const uint64_t stride = l.streamable ? d_.unit_stride(int(L)) : 0;
      uint32_t kept = 0;
      for (int u = 0; u < l.n_units; ++u) {
        const int64_t key = d_.unit_base[L] + u;
        const uint8_t t = p.tier[size_t(key)];
        require(t <= SS_TIER_RESIDENT_BACKED, SS_E_INVALID, "plan: bad tier value");
        if (!l.streamable) {
          require(t == SS_TIER_RESIDENT, SS_E_INVALID, "plan: a non-streamable layer's units must be resident");
          continue;
        }
        require(!(exclusive() && t == SS_TIER_RESIDENT_BACKED), SS_E_INVALID,
                "plan: tier B (resident with a pinned copy) is refused in the exclusive tier mode");
        switch (t) {
          case SS_TIER_RESIDENT_BACKED:
            ++p.n_backed;
            [[fallthrough]];
          case SS_TIER_RESIDENT:
            p.resident += stride;
            ++p.n_resident;
            ++kept;
            break;
          case SS_TIER_PINNED:
            ++p.n_pinned;
            streamed.push_back(Item{key, int(L), stride, 0.0});
            break;
          case SS_TIER_DISK:
            p.disk += l.unit_bytes;
            ++p.n_disk;
            streamed.push_back(Item{key, int(L), stride, 0.0});
            break;
          default:  // paired
            ++p.n_pair;
            break;
        }
      }
      if (l.streamable && l.n_units > 0 && b_.dynamic_slots_per_layer)
        p.dynamic += uint64_t(std::min<uint32_t>(b_.dynamic_slots_per_layer, uint32_t(l.n_units) - kept)) * stride;
    }
    const uint64_t packed = pinned_layout(d_, p.tier).total;
    p.pinned = packed;
    for (const auto& h : d_.host_fixed) p.pinned += h.bytes;
    require(p.pinned >= packed, SS_E_INVALID, "plan: host byte total overflows");
    grant_spares(p, less_floor(b_.host_pinned_bytes, p.pinned));
    const std::map<uint64_t, uint32_t> r = rings(streamed);
    p.rings.clear();
    for (const auto& [stride, slots] : r) p.rings.push_back(RingClass{stride, slots});
    p.ring = ring_bytes(r);
    require(p.pinned <= b_.host_pinned_bytes, SS_E_CAPACITY,
            d_.engine + ": " + gib(p.pinned) + " GiB must be pinned on the host, above the host budget " +
                gib(b_.host_pinned_bytes) + " GiB; raise the cap or the host budget");
    p.peak = p.fixed + p.dynamic + p.ring + p.resident;
    require(p.peak + p.margin <= p.cap, SS_E_CAPACITY,
            d_.engine + ": predicted peak " + gib(p.peak) + " GiB above the cap " + gib(p.cap) + " GiB - margin " +
                gib(p.margin) + " GiB");
  }

  // The host budget after the descriptor's fixed host bytes.
  uint64_t host_room() const {
    uint64_t left = b_.host_pinned_bytes;
    for (const auto& h : d_.host_fixed) left = less_floor(left, h.bytes);
    return left;
  }
  uint64_t host_bytes(const Item& it) const { return host_stride(d_.layers[size_t(it.layer)].unit_bytes); }
  bool exclusive() const { return b_.tier_mode == SS_TIER_MODE_EXCLUSIVE; }

 private:
  template <typename F>
  void for_each_streamable_layer(F&& f) const {
    for (size_t L = 0; L < d_.layers.size(); ++L)
      if (d_.layers[L].streamable && d_.layers[L].n_units > 0) f(int(L), d_.layers[L]);
  }
  // Exclusive mode: per host stride, the blocks asked (host_spare_units or 64, at most that stride's units), granted
  // in ascending block size while the host budget lasts.
  void grant_spares(Plan& p, uint64_t host_left) const {
    p.spares.clear();
    if (!exclusive()) return;
    std::map<uint64_t, uint64_t> units_of;  // host stride -> streamable units
    for_each_streamable_layer([&](int, const Layer& l) { units_of[host_stride(l.unit_bytes)] += uint64_t(l.n_units); });
    const uint64_t want = b_.host_spare_units ? b_.host_spare_units : 64;
    for (const auto& [block, units] : units_of) {
      SpareClass c;
      c.block_bytes = block;
      c.asked = uint32_t(std::min(want, units));
      c.blocks = uint32_t(std::min<uint64_t>(c.asked, host_left / block));
      host_left -= uint64_t(c.blocks) * block;
      p.spares.push_back(c);
      p.pinned += block * c.blocks;
    }
  }

  const Desc& d_;
  const ss_budget& b_;
};

// Which units stay resident: true per item (items in model order).
std::vector<char> choose_residents(const Desc& d, const Planner& pl, const std::vector<Item>& items, uint64_t room,
                                   bool* fits) {
  std::vector<char> on(items.size(), 0);
  uint64_t all = 0;
  for (const Item& it : items) all += it.dev;
  *fits = true;
  if (d.order == Order::Prefix) {
    // shrink the prefix from the whole model until it and the rest's rings fit
    uint64_t prefix = all;
    for (size_t k = items.size();; --k) {
      const std::vector<Item> rest(items.begin() + std::ptrdiff_t(k), items.end());
      if (prefix + Planner::ring_bytes(pl.rings(rest)) <= room) {
        std::fill(on.begin(), on.begin() + std::ptrdiff_t(k), char(1));
        return on;
      }
      if (k == 0) break;
      prefix -= items[k - 1].dev;
    }
    *fits = false;
    return on;
  }
  if (all <= room) {
    std::fill(on.begin(), on.end(), char(1));
    return on;
  }
  const uint64_t ring = Planner::ring_bytes(pl.rings(items));
  if (ring > room) {
    *fits = false;
    return on;
  }
  std::vector<size_t> by_pref(items.size());
  for (size_t i = 0; i < by_pref.size(); ++i) by_pref[i] = i;
  std::stable_sort(by_pref.begin(), by_pref.end(), [&](size_t a, size_t b) { return preferred(items[a], items[b]); });
  uint64_t used = 0;
  const uint64_t budget = room - ring;
  for (size_t i : by_pref) {
    if (used + items[i].dev > budget) continue;
    on[i] = 1;
    used += items[i].dev;
  }
  return on;
}

}  // namespace

uint64_t host_stride(uint64_t bytes) {
  require(bytes <= UINT64_MAX - (kPage - 1), SS_E_INVALID, "plan: unit bytes overflow the host stride");
  return (bytes + kPage - 1) & ~(kPage - 1);
}

uint64_t plan_margin(const ss_budget& b) {
  const double by_gib = b.margin_gib * double(kGiB), by_share = b.margin_fraction * double(b.device_bytes);
  return uint64_t(by_gib < by_share ? by_share : by_gib);
}

bool same_budget(const ss_budget& a, const ss_budget& b) {
  return std::make_tuple(a.device_bytes, a.host_pinned_bytes, a.workspace_bytes, a.margin_gib, a.margin_fraction,
                         a.dynamic_slots_per_layer, a.ring_slots, a.pinned_backing, a.tier_mode, a.host_spare_units) ==
         std::make_tuple(b.device_bytes, b.host_pinned_bytes, b.workspace_bytes, b.margin_gib, b.margin_fraction,
                         b.dynamic_slots_per_layer, b.ring_slots, b.pinned_backing, b.tier_mode, b.host_spare_units);
}

PinnedLayout pinned_layout(const Desc& d, const std::vector<uint8_t>& tier) {
  PinnedLayout out;
  out.chunk_of.assign(size_t(d.total_units), -1);
  out.offset_of.assign(size_t(d.total_units), 0);
  // chunk_bytes.back() is the chunk being filled; a unit that does not fit after others opens the next one (a unit
  // larger than a chunk's maximum gets one alone)
  for (size_t L = 0; L < d.layers.size(); ++L) {
    const uint64_t stride = host_stride(d.layers[L].unit_bytes);
    for (int u = 0; u < d.layers[L].n_units; ++u) {
      const size_t key = size_t(d.unit_base[L] + u);
      if (!has_pinned_copy(tier[key])) continue;
      if (out.chunk_bytes.empty() || (out.chunk_bytes.back() > 0 && out.chunk_bytes.back() + stride > kChunkMax))
        out.chunk_bytes.push_back(0);
      out.chunk_of[key] = int32_t(out.chunk_bytes.size() - 1);
      out.offset_of[key] = out.chunk_bytes.back();
      out.chunk_bytes.back() += stride;
    }
  }
  for (uint64_t c : out.chunk_bytes) {
    require(out.total <= UINT64_MAX - c, SS_E_INVALID, "plan: pinned layout overflows");
    out.total += c;
  }
  return out;
}

Plan plan_make(const Desc& d, const ss_budget& b, const std::vector<double>& benefit) {
  require(benefit.empty() || int64_t(benefit.size()) == d.total_units, SS_E_INVALID,
          "plan: benefit needs one value per unit (ss_desc_total_units)");
  const Planner pl(d, b);
  Plan p = pl.open();
  const std::vector<Item> items = pl.items(benefit);
  bool fits = false;
  const std::vector<char> resident =
      choose_residents(d, pl, items, p.cap - p.margin - p.fixed - p.dynamic, &fits);
  require(fits, SS_E_CAPACITY,
          d.engine + ": nothing fits under the " + gib(p.cap) + " GiB cap: fixed " + gib(p.fixed) + " GiB + margin " +
              gib(p.margin) + " GiB + the stream rings exceed it");
  // the others go where the descriptor's tiers say; "pinned+disk" spills the preferred ones into the host budget
  uint64_t host_left = pl.host_room();
  std::vector<Item> spill;
  for (size_t i = 0; i < items.size(); ++i) {
    if (resident[i]) continue;
    uint8_t& t = p.tier[size_t(items[i].key)];
    if (d.tiers == Tiers::Pinned) {
      t = SS_TIER_PINNED;
      host_left = less_floor(host_left, pl.host_bytes(items[i]));
    } else if (d.tiers == Tiers::Disk) {
      t = SS_TIER_DISK;
    } else if (d.tiers == Tiers::Pair) {
      t = SS_TIER_PAIR;
    } else {
      spill.push_back(items[i]);
    }
  }
  std::stable_sort(spill.begin(), spill.end(), preferred);
  for (const Item& it : spill) {
    const uint64_t hb = pl.host_bytes(it);
    const bool pin = hb <= host_left;
    p.tier[size_t(it.key)] = pin ? SS_TIER_PINNED : SS_TIER_DISK;
    if (pin) host_left -= hb;
  }
  if (b.pinned_backing) {
    // residents gain a pinned copy, least preferred first (among equals the later unit), while the host budget lasts
    uint64_t left = pl.host_room();
    std::vector<Item> res;
    for (const Item& it : pl.items(benefit)) {
      const uint8_t t = p.tier[size_t(it.key)];
      if (t == SS_TIER_PINNED) left = less_floor(left, pl.host_bytes(it));
      else if (t == SS_TIER_RESIDENT) res.push_back(it);
    }
    std::stable_sort(res.begin(), res.end(), [](const Item& x, const Item& y) { return preferred(y, x); });
    for (const Item& it : res) {
      const uint64_t hb = pl.host_bytes(it);
      if (hb > left) break;
      p.tier[size_t(it.key)] = SS_TIER_RESIDENT_BACKED;
      left -= hb;
    }
  }
  pl.close(p);
  return p;
}

Plan plan_from_tiers(const Desc& d, const ss_budget& b, const std::vector<uint8_t>& tiers) {
  require(int64_t(tiers.size()) == d.total_units, SS_E_INVALID, "plan: one tier per unit (ss_desc_total_units)");
  const Planner pl(d, b);
  Plan p = pl.open();
  p.tier = tiers;
  pl.close(p);
  return p;
}

namespace {
// plan-v1 tier letters: R resident, P pinned, D disk, X paired, B resident with a pinned copy.
char tier_letter(uint8_t t) {
  switch (t) {
    case SS_TIER_RESIDENT: return 'R';
    case SS_TIER_PINNED: return 'P';
    case SS_TIER_DISK: return 'D';
    case SS_TIER_PAIR: return 'X';
    default: return 'B';
  }
}
int tier_of_letter(char c) {
  switch (c) {
    case 'R': return SS_TIER_RESIDENT;
    case 'P': return SS_TIER_PINNED;
    case 'D': return SS_TIER_DISK;
    case 'X': return SS_TIER_PAIR;
    case 'B': return SS_TIER_RESIDENT_BACKED;
    default: return -1;
  }
}
}  // namespace

Json plan_to_json(const Desc& d, const Plan& p) {
  Json j = Json::object();
  j["schema"] = Json::string("strix-stream/plan-v1");
  j["engine"] = Json::string(d.engine);
  const std::pair<const char*, uint64_t> head[] = {{"cap_bytes", p.cap},
                                                   {"margin_bytes", p.margin},
                                                   {"fixed_bytes", p.fixed},
                                                   {"dynamic_bytes", p.dynamic},
                                                   {"dynamic_slots_per_layer", p.dynamic_slots_per_layer},
                                                   {"ring_bytes", p.ring}};
  for (const auto& [k, v] : head) j[k] = Json::number(v);
  Json rings = Json::array();
  for (const RingClass& r : p.rings) {
    Json o = Json::object();
    o["slot_bytes"] = Json::number(r.stride);
    o["slots"] = Json::number(uint64_t(r.slots));
    rings.push(o);
  }
  j["rings"] = rings;
  const std::pair<const char*, uint64_t> sums[] = {
      {"resident_bytes", p.resident}, {"pinned_bytes", p.pinned}, {"disk_bytes", p.disk},   {"peak_bytes", p.peak},
      {"n_resident", p.n_resident},   {"n_pinned", p.n_pinned},   {"n_disk", p.n_disk},     {"n_pair", p.n_pair},
      {"n_backed", p.n_backed}};
  for (const auto& [k, v] : sums) j[k] = Json::number(v);
  if (p.budget.tier_mode == SS_TIER_MODE_EXCLUSIVE) {  // inclusive plans carry no spare blocks
    j["tier_mode"] = Json::string("exclusive");
    Json spare = Json::array();
    for (const SpareClass& c : p.spares) {
      Json o = Json::object();
      o["block_bytes"] = Json::number(c.block_bytes);
      o["asked"] = Json::number(uint64_t(c.asked));
      o["blocks"] = Json::number(uint64_t(c.blocks));
      spare.push(o);
    }
    j["spare_blocks"] = spare;
  }
  Json per_layer = Json::array();
  for (size_t L = 0; L < d.layers.size(); ++L) {
    std::string letters(size_t(d.layers[L].n_units), 'R');
    for (size_t u = 0; u < letters.size(); ++u) letters[u] = tier_letter(p.tier[size_t(d.unit_base[L]) + u]);
    per_layer.push(Json::string(letters));
  }
  j["tiers"] = per_layer;
  return j;
}

std::vector<uint8_t> tiers_from_json(const Desc& d, const Json& j) {
  const Json* t = j.find("tiers");
  require(t && t->is_array() && t->arr.size() == d.layers.size(), SS_E_DESC,
          "plan json: \"tiers\" needs one string per layer");
  std::vector<uint8_t> out;
  out.reserve(size_t(d.total_units));
  for (size_t L = 0; L < d.layers.size(); ++L) {
    const std::string letters = json_str(t->arr[L], "plan.tiers");
    require(letters.size() == size_t(d.layers[L].n_units), SS_E_DESC,
            "plan json: tiers[" + std::to_string(L) + "] needs one letter per unit");
    for (char c : letters) {
      const int tier = tier_of_letter(c);
      require(tier >= 0, SS_E_DESC, "plan json: tier letters are R P D X B");
      out.push_back(uint8_t(tier));
    }
  }
  return out;
}

}  // namespace tsb
