// Host forward mode: one layer's persistent device slots and the admission of a forward's routed units. Pure host
// logic; the decisions are the reference's (resident_set.cpp:25-217 there): a miss takes the lowest free slot, else
// evicts the least recently used unpinned unit not routed or busy this forward (ties to the lower unit id).
//   - LRU: misses are admitted in ascending id order; a forward's routed units all become the most recent.
//   - SCORED: every unit has a score, 0.7 x the one-step transition estimate from the previous forward's routed units
//     + 0.2 x its share of the last `window` forwards + 0.1 / (1 + forwards since its last miss or first use); the
//     misses and the unpinned residents outside this forward compete for the rows free slots and those residents
//     hold (higher score first, then the more recent, then the lower id): misses above the cut are admitted in that
//     order, only residents below it may be evicted; a hit does not refresh recency.
#pragma once

#include <cstdint>
#include <deque>
#include <vector>

namespace tsb {

struct Admission {
  std::vector<int32_t> hits, admitted, slot_of, evicted, evicted_slot, transient;  // ascending unit ids
  int deferred = 0;
};

class ResidentSet {
 public:
  ResidentSet(int n_units, int capacity, bool scored = false, uint32_t window = 16);
  int capacity() const { return int(unit_in_.size()); }
  int slot(int unit) const { return slot_of_[size_t(unit)]; }
  int n_resident() const { return n_resident_; }
  int place(int unit, bool pin);  // at open / seed: the lowest free slot, -1 when full
  void drop(int unit);
  // max_evictions >= 0 caps the evictions (misses past the cap that need a victim stay transient)
  Admission admit(const std::vector<int32_t>& routed, const std::vector<char>& busy, bool admit_misses,
                  int max_evictions = -1);
  // The forward's routed units and which of them missed (prefetched or not resident: SCORED refreshes their recency).
  void observe(const std::vector<int32_t>& routed, const std::vector<int32_t>& misses);
  double score(int unit) const;  // SCORED (0 under LRU)

 private:
  int lru_victim(const std::vector<char>& keep) const;
  int n_units_;
  bool scored_ = false;
  uint32_t window_ = 16;
  std::vector<uint32_t> trans_, trans_n_, freq_;  // SCORED: transition counts [prev][unit], row totals, window counts
  std::vector<int32_t> prev_;                     // the previous forward's routed units (ascending)
  std::deque<std::vector<int32_t>> recent_;
  std::vector<int32_t> slot_of_, unit_in_;
  std::vector<char> pinned_;
  std::vector<uint64_t> last_use_;
  uint64_t tick_ = 0;
  int n_resident_ = 0;
};

}  // namespace tsb
