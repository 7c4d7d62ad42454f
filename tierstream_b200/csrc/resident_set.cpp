// The host forward mode's per-layer resident set; the rules are stated in resident_set.hpp.
#include "resident_set.hpp"

#include <algorithm>
#include <numeric>
#include <tuple>

#include "errors.hpp"

namespace tsb {

namespace {

// The scored cut's order: a higher score first, then the later last use, then the lower unit id.
struct CutKey {
  double score;
  uint64_t stamp;
  int32_t unit;
  bool before(const CutKey& o) const {
    return std::make_tuple(o.score, o.stamp, unit) < std::make_tuple(score, stamp, o.unit);
  }
};

std::vector<int32_t> ascending_unique(std::vector<int32_t> v) {
  std::sort(v.begin(), v.end());
  v.erase(std::unique(v.begin(), v.end()), v.end());
  return v;
}

}  // namespace

ResidentSet::ResidentSet(int n_units, int capacity, bool scored, uint32_t window)
    : n_units_(n_units), scored_(scored), window_(window ? window : 16) {
  require(capacity >= 0 && capacity <= n_units, SS_E_INVALID, "resident set: capacity must be 0..n_units");
  slots_.resize(size_t(capacity));
  home_.assign(size_t(n_units), -1);
  free_bits_.assign((size_t(capacity) + 63) / 64, 0);
  for (int s = 0; s < capacity; ++s) free_bits_[size_t(s) / 64] |= uint64_t(1) << (s % 64);
  stamp_.assign(size_t(n_units), 0);
  if (scored_) {
    h_.pair.assign(size_t(n_units) * size_t(n_units), 0);
    h_.from.assign(size_t(n_units), 0);
    h_.in_ring.assign(size_t(n_units), 0);
    h_.ring.resize(window_);
  }
}

int ResidentSet::first_free() const {
  for (size_t w = 0; w < free_bits_.size(); ++w)
    if (free_bits_[w]) return int(w * 64 + size_t(__builtin_ctzll(free_bits_[w])));
  return -1;
}

void ResidentSet::occupy(int slot, int32_t unit, bool pin) {
  slots_[size_t(slot)] = Slot{unit, pin};
  home_[size_t(unit)] = slot;
  free_bits_[size_t(slot) / 64] &= ~(uint64_t(1) << (slot % 64));
  ++occupied_;
}

void ResidentSet::vacate(int slot) {
  Slot& s = slots_[size_t(slot)];
  home_[size_t(s.unit)] = -1;
  s = Slot{};
  free_bits_[size_t(slot) / 64] |= uint64_t(1) << (slot % 64);
  --occupied_;
}

// The terms and their order of operations are fixed: the cut compares these doubles exactly.
double ResidentSet::score(int unit) const {
  if (!scored_) return 0.0;
  double trans = 0.0;
  if (!h_.last.empty()) {
    for (int32_t p : h_.last) {
      const uint32_t n = h_.from[size_t(p)];
      if (n) trans += double(h_.pair[size_t(p) * size_t(n_units_) + size_t(unit)]) / double(n);
    }
    trans /= double(h_.last.size());
  }
  const double freq = h_.count ? double(h_.in_ring[size_t(unit)]) / double(h_.count) : 0.0;
  const uint64_t st = stamp_[size_t(unit)];
  const double rec = st ? 1.0 / (1.0 + double(now_ - st)) : 0.0;
  return 0.7 * trans + 0.2 * freq + 0.1 * rec;
}

int ResidentSet::place(int unit, bool pin) {
  require(unit >= 0 && unit < n_units_, SS_E_INVALID, "resident set: unit out of range");
  if (const int at = home_[size_t(unit)]; at >= 0) {
    if (pin) slots_[size_t(at)].pinned = true;
    return at;
  }
  const int s = first_free();
  if (s >= 0) occupy(s, unit, pin);
  return s;
}

void ResidentSet::drop(int unit) {
  if (const int at = home_[size_t(unit)]; at >= 0) vacate(at);
}

Admission ResidentSet::admit(const std::vector<int32_t>& routed_in, const std::vector<char>& busy, bool admit_misses,
                             int max_evictions) {
  Admission out;
  const std::vector<int32_t> routed = ascending_unique(routed_in);
  // protected this forward: the routed units and the busy ones (their copies are in flight)
  std::vector<char> hold(size_t(n_units_), 0);
  std::vector<int32_t> misses;
  for (int32_t u : routed) {
    require(u >= 0 && u < n_units_, SS_E_INVALID, "routes: unit id out of range");
    hold[size_t(u)] = 1;
    if (home_[size_t(u)] >= 0) out.hits.push_back(u);
    else misses.push_back(u);
  }
  for (size_t u = 0; u < std::min(busy.size(), hold.size()); ++u) hold[u] |= busy[u] ? 1 : 0;
  if (!admit_misses || slots_.empty()) {
    out.transient = misses;
    return out;
  }
  // the residents that may be evicted: unpinned and not held
  std::vector<int32_t> evictable;
  int n_free = 0;
  for (const Slot& s : slots_) {
    if (s.unit < 0) ++n_free;
    else if (!s.pinned && !hold[size_t(s.unit)]) evictable.push_back(s.unit);
  }
  std::vector<int32_t> order = misses;  // the misses that get a slot, in admission order (LRU: ascending ids)
  if (scored_) {
    // the cut: evictable residents and misses ranked together for the n_free + evictable rows; misses inside are
    // admitted in rank order, and only residents outside may be evicted
    std::vector<CutKey> keys;
    for (int32_t u : evictable) keys.push_back({score(u), stamp_[size_t(u)], u});
    const size_t n_res = keys.size(), rows = size_t(n_free) + n_res;
    for (int32_t u : misses) keys.push_back({score(u), stamp_[size_t(u)], u});
    std::vector<size_t> rank(keys.size());
    std::iota(rank.begin(), rank.end(), size_t(0));
    std::sort(rank.begin(), rank.end(), [&](size_t a, size_t b) { return keys[a].before(keys[b]); });
    order.clear();
    std::vector<char> outside(size_t(n_units_), 0);
    for (size_t r = 0; r < rank.size(); ++r) {
      const bool is_miss = rank[r] >= n_res;
      if (r < rows && is_miss) order.push_back(keys[rank[r]].unit);
      if (r >= rows && !is_miss) outside[size_t(keys[rank[r]].unit)] = 1;
    }
    evictable.erase(std::remove_if(evictable.begin(), evictable.end(),
                                   [&](int32_t u) { return !outside[size_t(u)]; }),
                    evictable.end());
  }
  // victims in eviction order: the least recent first, ties to the lower id
  std::sort(evictable.begin(), evictable.end(), [&](int32_t a, int32_t b) {
    return std::make_pair(stamp_[size_t(a)], a) < std::make_pair(stamp_[size_t(b)], b);
  });
  size_t next_victim = 0;
  std::vector<char> got(size_t(n_units_), 0);
  std::vector<std::pair<int32_t, int32_t>> admitted, evicted;  // (unit, slot)
  for (int32_t u : order) {
    int s = first_free();
    if (s < 0) {
      if (max_evictions >= 0 && int(evicted.size()) >= max_evictions) {
        ++out.deferred;  // no free slot and no eviction allowed: stays transient
        continue;
      }
      if (next_victim == evictable.size()) break;  // everything resident is pinned or held this forward
      const int32_t v = evictable[next_victim++];
      s = home_[size_t(v)];
      vacate(s);
      evicted.push_back({v, s});
    }
    occupy(s, u, false);
    got[size_t(u)] = 1;
    admitted.push_back({u, s});
  }
  for (int32_t u : misses)
    if (!got[size_t(u)]) out.transient.push_back(u);
  std::sort(admitted.begin(), admitted.end());
  std::sort(evicted.begin(), evicted.end());
  for (const auto& [u, s] : admitted) {
    out.admitted.push_back(u);
    out.slot_of.push_back(s);
  }
  for (const auto& [u, s] : evicted) {
    out.evicted.push_back(u);
    out.evicted_slot.push_back(s);
  }
  return out;
}

void ResidentSet::observe(const std::vector<int32_t>& routed_in, const std::vector<int32_t>& misses) {
  const std::vector<int32_t> routed = ascending_unique(routed_in);
  ++now_;
  if (!scored_) {
    for (int32_t u : routed) stamp_[size_t(u)] = now_;
    return;
  }
  // SCORED: a miss (admitted or not) and a first use refresh a unit's recency; a hit does not
  for (int32_t u : misses) stamp_[size_t(u)] = now_;
  for (int32_t u : routed) stamp_[size_t(u)] = stamp_[size_t(u)] ? stamp_[size_t(u)] : now_;
  for (int32_t p : h_.last) {
    h_.from[size_t(p)] += 1;
    uint32_t* row = h_.pair.data() + size_t(p) * size_t(n_units_);
    for (int32_t u : routed) row[u] += 1;
  }
  h_.last = routed;
  // the window ring: the oldest forward leaves once the ring is full
  if (h_.count == window_) {
    for (int32_t u : h_.ring[h_.head]) h_.in_ring[size_t(u)] -= 1;
  } else {
    ++h_.count;
  }
  h_.ring[h_.head] = routed;
  for (int32_t u : routed) h_.in_ring[size_t(u)] += 1;
  h_.head = (h_.head + 1) % window_;
}

}  // namespace tsb
