// Host forward mode: one layer's persistent device slots and the admission of a forward's routed units. Pure host
// logic. The decision rules are the reference's (resident_set.cpp:25-217 there), so the same routes give the same
// slots:
//   - a miss takes the lowest free slot; with none free, the least recently used unpinned unit that is not routed or
//     busy this forward is evicted (ties to the lower unit id);
//   - LRU: misses are admitted in ascending id order; a forward's routed units all become the most recent;
//   - SCORED: every unit has a score, 0.7 x the one-step transition estimate from the previous forward's routed units
//     + 0.2 x its share of the last `window` forwards + 0.1 / (1 + forwards since its last miss or first use); the
//     misses and the unpinned residents outside this forward compete for the rows free slots and those residents hold
//     (higher score first, then the more recent, then the lower id): misses above the cut are admitted in that order,
//     only residents below it may be evicted; a hit does not refresh recency.
// Here the free slots are a bitset searched lowest first, and an admission builds its victims once, as a queue in
// eviction order (no slot frees while misses are admitted, so the queue equals a fresh search per miss).
#pragma once

#include <cstdint>
#include <vector>

namespace tsb {

struct Admission {
  std::vector<int32_t> hits, admitted, slot_of, evicted, evicted_slot, transient;  // ascending unit ids
  int deferred = 0;
};

class ResidentSet {
 public:
  ResidentSet(int n_units, int capacity, bool scored = false, uint32_t window = 16);
  int capacity() const { return int(slots_.size()); }
  int slot(int unit) const { return home_[size_t(unit)]; }
  int n_resident() const { return occupied_; }
  int place(int unit, bool pin);  // at open / seed: the lowest free slot, -1 when full
  void drop(int unit);
  // max_evictions >= 0 caps the evictions (misses past the cap that need a victim stay transient)
  Admission admit(const std::vector<int32_t>& routed, const std::vector<char>& busy, bool admit_misses,
                  int max_evictions = -1);
  // The forward's routed units and which of them missed (prefetched or not resident: SCORED refreshes their recency).
  void observe(const std::vector<int32_t>& routed, const std::vector<int32_t>& misses);
  double score(int unit) const;  // SCORED (0 under LRU)

 private:
  struct Slot {
    int32_t unit = -1;
    bool pinned = false;
  };
  int first_free() const;
  void occupy(int slot, int32_t unit, bool pin);
  void vacate(int slot);
  // SCORED: the forwards' routed sets, a fixed ring of the last `window`
  struct History {
    std::vector<uint32_t> pair;     // [previous unit][unit]: forwards that routed unit right after previous
    std::vector<uint32_t> from;     // [previous unit]: forwards that followed one routing it
    std::vector<uint32_t> in_ring;  // [unit]: forwards of the ring that routed it
    std::vector<std::vector<int32_t>> ring;
    size_t head = 0, count = 0;
    std::vector<int32_t> last;      // the previous forward's routed units (ascending)
  };
  int n_units_;
  bool scored_;
  uint32_t window_;
  std::vector<Slot> slots_;
  std::vector<int32_t> home_;           // per unit: its slot, -1 when not resident
  std::vector<uint64_t> free_bits_;     // bit s: slot s is free
  std::vector<uint64_t> stamp_;         // per unit: the forward that last refreshed it (0: never)
  uint64_t now_ = 0;
  int occupied_ = 0;
  History h_;
};

}  // namespace tsb
