#include "resident_set.hpp"

#include <algorithm>
#include <numeric>

#include "errors.hpp"

namespace tsb {

ResidentSet::ResidentSet(int n_units, int capacity, bool scored, uint32_t window)
    : n_units_(n_units), scored_(scored), window_(window) {
  require(capacity >= 0 && capacity <= n_units, SS_E_INVALID, "resident set: capacity must be 0..n_units");
  slot_of_.assign(size_t(n_units), -1);
  unit_in_.assign(size_t(capacity), -1);
  pinned_.assign(size_t(capacity), 0);
  last_use_.assign(size_t(n_units), 0);
  if (scored_) {
    trans_.assign(size_t(n_units) * size_t(n_units), 0);
    trans_n_.assign(size_t(n_units), 0);
    freq_.assign(size_t(n_units), 0);
  }
}

// In double precision, in this order of operations (the decisions compare these values exactly).
double ResidentSet::score(int unit) const {
  if (!scored_) return 0.0;
  double trans = 0.0;
  if (!prev_.empty()) {
    for (int32_t p : prev_) {
      const uint32_t n = trans_n_[size_t(p)];
      if (n) trans += double(trans_[size_t(p) * size_t(n_units_) + size_t(unit)]) / double(n);
    }
    trans /= double(prev_.size());
  }
  const double freq = recent_.empty() ? 0.0 : double(freq_[size_t(unit)]) / double(recent_.size());
  const uint64_t lu = last_use_[size_t(unit)];
  const double rec = lu ? 1.0 / (1.0 + double(tick_ - lu)) : 0.0;
  return 0.7 * trans + 0.2 * freq + 0.1 * rec;
}

int ResidentSet::place(int unit, bool pin) {
  require(unit >= 0 && unit < n_units_, SS_E_INVALID, "resident set: unit out of range");
  int& s = slot_of_[size_t(unit)];
  if (s >= 0) {
    if (pin) pinned_[size_t(s)] = 1;
    return s;
  }
  const auto it = std::find(unit_in_.begin(), unit_in_.end(), -1);
  if (it == unit_in_.end()) return -1;
  s = int32_t(it - unit_in_.begin());
  *it = unit;
  pinned_[size_t(s)] = pin;
  ++n_resident_;
  return s;
}

void ResidentSet::drop(int unit) {
  const int s = slot_of_[size_t(unit)];
  if (s < 0) return;
  unit_in_[size_t(s)] = -1;
  pinned_[size_t(s)] = 0;
  slot_of_[size_t(unit)] = -1;
  --n_resident_;
}

int ResidentSet::lru_victim(const std::vector<char>& keep) const {
  int best = -1;
  for (size_t s = 0; s < unit_in_.size(); ++s) {
    const int32_t u = unit_in_[s];
    if (u < 0 || pinned_[s] || keep[size_t(u)]) continue;
    if (best >= 0) {
      const int32_t b = unit_in_[size_t(best)];
      const uint64_t lu = last_use_[size_t(u)], lb = last_use_[size_t(b)];
      if (!(lu < lb || (lu == lb && u < b))) continue;
    }
    best = int(s);
  }
  return best;
}

Admission ResidentSet::admit(const std::vector<int32_t>& routed_in, const std::vector<char>& busy, bool admit_misses,
                             int max_evictions) {
  Admission a;
  std::vector<int32_t> routed = routed_in;
  std::sort(routed.begin(), routed.end());
  routed.erase(std::unique(routed.begin(), routed.end()), routed.end());
  std::vector<char> keep(size_t(n_units_), 0);
  std::vector<int32_t> misses;
  for (int32_t u : routed) {
    require(u >= 0 && u < n_units_, SS_E_INVALID, "routes: unit id out of range");
    keep[size_t(u)] = 1;
    (slot_of_[size_t(u)] >= 0 ? a.hits : misses).push_back(u);
  }
  for (size_t u = 0; u < busy.size() && u < keep.size(); ++u)
    if (busy[u]) keep[u] = 1;
  if (!admit_misses || unit_in_.empty()) {
    a.transient = misses;
    return a;
  }
  std::vector<int32_t> take = misses;  // the misses that get a slot, in admission order
  if (scored_) {
    // the scored cut: the unpinned residents outside this forward and the misses compete for the rows they can hold
    struct Cand {
      int32_t unit;
      double score;
      uint64_t last;
      bool resident;
    };
    std::vector<Cand> comp;
    size_t free_slots = 0;
    for (size_t s = 0; s < unit_in_.size(); ++s) {
      const int32_t u = unit_in_[s];
      if (u < 0) ++free_slots;
      else if (!pinned_[s] && !keep[size_t(u)]) comp.push_back({u, score(u), last_use_[size_t(u)], true});
    }
    const size_t rows = free_slots + comp.size();
    for (int32_t u : misses) comp.push_back({u, score(u), last_use_[size_t(u)], false});
    std::sort(comp.begin(), comp.end(), [](const Cand& x, const Cand& y) {
      if (x.score != y.score) return x.score > y.score;
      if (x.last != y.last) return x.last > y.last;
      return x.unit < y.unit;
    });
    take.clear();
    for (size_t i = 0; i < comp.size() && i < rows; ++i)
      if (!comp[i].resident) take.push_back(comp[i].unit);
    std::vector<char> below(size_t(n_units_), 0);  // residents below the cut: the only eviction candidates
    for (size_t i = rows; i < comp.size(); ++i)
      if (comp[i].resident) below[size_t(comp[i].unit)] = 1;
    for (size_t u = 0; u < keep.size(); ++u)
      if (!below[u] && slot_of_[u] >= 0) keep[u] = 1;
  }
  std::vector<char> taken(size_t(n_units_), 0);
  std::vector<std::pair<int32_t, int32_t>> adm, ev;  // (unit, slot)
  for (int32_t u : take) {
    int s = -1;
    const auto it = std::find(unit_in_.begin(), unit_in_.end(), -1);
    if (it != unit_in_.end()) {
      s = int(it - unit_in_.begin());
    } else {
      if (max_evictions >= 0 && int(ev.size()) >= max_evictions) {
        ++a.deferred;
        continue;
      }
      s = lru_victim(keep);
      if (s < 0) break;  // everything resident is pinned or in use this forward
      const int32_t old = unit_in_[size_t(s)];
      slot_of_[size_t(old)] = -1;
      ev.push_back({old, s});
      --n_resident_;
    }
    unit_in_[size_t(s)] = u;
    pinned_[size_t(s)] = 0;
    slot_of_[size_t(u)] = s;
    keep[size_t(u)] = 1;
    taken[size_t(u)] = 1;
    ++n_resident_;
    adm.push_back({u, s});
  }
  for (int32_t u : misses)
    if (!taken[size_t(u)]) a.transient.push_back(u);
  std::sort(adm.begin(), adm.end());
  std::sort(ev.begin(), ev.end());
  for (const auto& x : adm) {
    a.admitted.push_back(x.first);
    a.slot_of.push_back(x.second);
  }
  for (const auto& x : ev) {
    a.evicted.push_back(x.first);
    a.evicted_slot.push_back(x.second);
  }
  return a;
}

void ResidentSet::observe(const std::vector<int32_t>& routed_in, const std::vector<int32_t>& misses) {
  ++tick_;
  if (!scored_) {
    for (int32_t u : routed_in) last_use_[size_t(u)] = tick_;
    return;
  }
  std::vector<int32_t> routed = routed_in;
  std::sort(routed.begin(), routed.end());
  routed.erase(std::unique(routed.begin(), routed.end()), routed.end());
  for (int32_t u : misses) last_use_[size_t(u)] = tick_;  // a miss and a first use refresh recency, a hit does not
  for (int32_t u : routed)
    if (last_use_[size_t(u)] == 0) last_use_[size_t(u)] = tick_;
  for (int32_t p : prev_) {
    ++trans_n_[size_t(p)];
    for (int32_t u : routed) ++trans_[size_t(p) * size_t(n_units_) + size_t(u)];
  }
  prev_ = routed;
  recent_.push_back(routed);
  for (int32_t u : routed) ++freq_[size_t(u)];
  if (recent_.size() > window_) {
    for (int32_t u : recent_.front()) --freq_[size_t(u)];
    recent_.pop_front();
  }
}

}  // namespace tsb
