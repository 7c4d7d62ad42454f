// Host forward mode: one layer's persistent device slots and the LRU admission of a forward's routed units. Pure host
// logic; the decisions are the reference's (resident_set.cpp:25-217 there, its LRU policy): a miss takes the lowest
// free slot, else evicts the least recently used unpinned unit not routed or busy this forward (ties to the lower unit
// id); misses are admitted in ascending id order; a forward's routed units all become the most recent.
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
  ResidentSet(int n_units, int capacity);
  int capacity() const { return int(unit_in_.size()); }
  int slot(int unit) const { return slot_of_[size_t(unit)]; }
  int n_resident() const { return n_resident_; }
  int place(int unit, bool pin);  // at open / seed: the lowest free slot, -1 when full
  void drop(int unit);
  // max_evictions >= 0 caps the evictions (misses past the cap that need a victim stay transient)
  Admission admit(const std::vector<int32_t>& routed, const std::vector<char>& busy, bool admit_misses,
                  int max_evictions = -1);
  void observe(const std::vector<int32_t>& routed);

 private:
  int lru_victim(const std::vector<char>& keep) const;
  int n_units_;
  std::vector<int32_t> slot_of_, unit_in_;
  std::vector<char> pinned_;
  std::vector<uint64_t> last_use_;
  uint64_t tick_ = 0;
  int n_resident_ = 0;
};

}  // namespace tsb
