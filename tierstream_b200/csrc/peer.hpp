// The peer tier: gated units partitioned over the GPUs' HBM. Each GPU keeps the units it owns in a store (one device
// allocation, unit-major: unit i of the store at base + i * unit_bytes, its parts back to back in descriptor order); a
// device-gated miss on an owned unit is copied from its owner's store (over NVLink for a peer, inside HBM for the
// GPU's own) instead of from pinned RAM. The slot cache's decisions do not change: an owned unit keeps its Host home
// and its block number; only the source of its bytes does. When every unit is owned, no pinned block is allocated
// (blocks are bookkeeping only) and write-backs move no bytes, since every unit's bytes live in a store.
//
// The striped layout instead cuts every owned unit into `world` stripes (stripe_bytes below), stripe r of each in rank
// r's store: a miss then reads 1/world of the unit from every GPU at once, so the ranks' pulls spread over all links
// instead of queueing on the few owners of the units they happen to miss. The owner map then only says which units
// are in the tier.
//
// There is no counterpart in the reference (it declares SS_TIER_PAIR, ss.h:103, and never fetches from it).
#pragma once

#include <algorithm>
#include <cstdint>
#include <memory>
#include <vector>

#include "desc.hpp"

namespace tsb {

// Gated layers in ordinal order (layers with units, every one streamable) and the unit base of each (G + 1 entries):
// the key space the device-gated context and the peer tier share.
struct GatedKeys {
  std::vector<int> layers;
  std::vector<uint32_t> base;
  uint64_t unit_bytes = 0;
  uint32_t keys() const { return base.empty() ? 0 : base.back(); }
};
GatedKeys gated_keys(const Desc& d);

// The owner of every key, by routing counts summed over the ranks: keys in descending count (ties: lower key first),
// each to the rank with the least count assigned so far (ties: fewer units, then the lower rank) among those below
// their unit capacity; -1 when every rank is full (the key stays in pinned RAM). Deterministic: every rank that
// plans from the same counts gets the same owners.
std::vector<int32_t> plan_owners(const uint64_t* counts, uint32_t keys, uint32_t world, const uint64_t* cap_units);

// index[k]: the position of key k in its owner's store (keys of one owner in key order); -1 for unowned keys.
std::vector<int64_t> store_index(const std::vector<int32_t>& owner, uint32_t world, std::vector<uint64_t>* per_rank);

enum PeerLayout : uint32_t { kWholeUnits = 0, kStriped = 1 };

// Striped layout: the bytes of one stripe, ceil(unit_bytes / world) rounded up to 256 (stripes start 256-byte
// aligned in every store); stripe r covers [r * stripe, min(unit_bytes, (r + 1) * stripe)) of the unit, so the last
// stripes may be shorter or empty.
uint64_t stripe_bytes(uint64_t unit_bytes, uint32_t world);
inline uint64_t stripe_len(uint64_t unit_bytes, uint64_t stripe, uint32_t r) {
  const uint64_t lo = uint64_t(r) * stripe;
  return lo >= unit_bytes ? 0 : std::min(stripe, unit_bytes - lo);
}
// Striped layout: index[k] = the position of key k among all owned keys (key order, the same in every store); -1 for
// unowned keys.
std::vector<int64_t> striped_index(const std::vector<int32_t>& owner, uint64_t* owned);

// f(part, unit offset, bytes) for each part that [off, off + n) of a unit's bytes overlaps (parts back to back at
// part_offset[p], part_bytes[p] long): how one piece of a unit is split into copies into the arena's part slots.
template <class F>
void split_parts(const std::vector<uint64_t>& part_offset, const std::vector<uint64_t>& part_bytes, uint64_t off,
                 uint64_t n, F&& f) {
  for (uint32_t p = 0; p < part_bytes.size(); ++p) {
    const uint64_t a = std::max(off, part_offset[p]), b = std::min(off + n, part_offset[p] + part_bytes[p]);
    if (a < b) f(p, a, b - a);
  }
}

struct PeerTier {
  uint32_t world = 0;
  int32_t rank = -1;
  std::vector<int32_t> owner;   // per gated key
  std::vector<int64_t> index;   // per gated key (store_index, or striped_index for the striped layout)
  std::vector<char*> base;      // per rank: its store's device address in this process
  bool all_owned = false;
  int copy = 0;                 // 0 = land kernel, 1 = copy engines
  uint32_t layout = kWholeUnits;
  uint64_t stripe = 0;          // striped: stripe_bytes(unit_bytes, world)
  bool owned(uint32_t key) const { return owner[key] >= 0; }
  // Calls f(src, unit_offset, bytes, from_rank) for the pieces that make up an owned unit's bytes: the whole unit from
  // its owner's store, or (striped) each non-empty stripe from its rank's store, the next rank's first and this
  // rank's own last, so that ranks issuing their pulls at the same moment start on different GPUs.
  template <class F>
  void pieces(uint32_t key, uint64_t unit_bytes, F&& f) const {
    const uint64_t i = uint64_t(index[key]);
    if (layout == kWholeUnits) {
      f(static_cast<const char*>(base[size_t(owner[key])] + i * unit_bytes), uint64_t(0), unit_bytes, owner[key]);
      return;
    }
    for (uint32_t j = 1; j <= world; ++j) {
      const uint32_t r = (uint32_t(rank) + j) % world;
      const uint64_t n = stripe_len(unit_bytes, stripe, r);
      if (n) f(static_cast<const char*>(base[r] + i * stripe), uint64_t(r) * stripe, n, int32_t(r));
    }
  }
};

// CUDA IPC for the stores: the handle of a store (64 bytes), a mapping of another process's store on `device` with
// peer access enabled, and its release.
void ipc_export(const void* base, void* handle);
void* ipc_map(const void* handle, int device);
void ipc_unmap(void* base);

// This rank's store: cudaMalloc'd on `device`, filled from the descriptor's sources, checked on the device against
// the descriptor's hashes (K3) when verify is set and the descriptor has them; with fill = false only allocated (the
// caller writes every unit's bytes).
//
// Striped (layout kStriped, world ranks): stripe `rank` of every owned unit, unit i (striped_index) at base + i *
// stripe_bytes; the bytes are read from the sources with fill, but a stripe cannot be checked against its unit's
// hash on its own: verify_tier checks the units once every store is mapped.
class PeerStore {
 public:
  PeerStore(const Desc& d, const std::vector<int32_t>& owner, int32_t rank, int device, bool verify, bool fill = true,
            uint32_t layout = kWholeUnits, uint32_t world = 1);
  ~PeerStore();
  PeerStore(const PeerStore&) = delete;
  PeerStore& operator=(const PeerStore&) = delete;
  char* base() const { return base_; }
  uint64_t bytes() const { return bytes_; }
  uint64_t units() const { return units_; }
  int device() const { return device_; }
  uint64_t unit_bytes() const { return unit_bytes_; }
  int32_t rank() const { return rank_; }
  const std::vector<int32_t>& owner() const { return owner_; }
  double fill_seconds() const { return fill_s_; }
  uint32_t layout() const { return layout_; }

 private:
  char* base_ = nullptr;
  uint64_t bytes_ = 0, units_ = 0, unit_bytes_ = 0;
  uint32_t layout_ = kWholeUnits;
  int device_ = 0;
  int32_t rank_ = -1;
  std::vector<int32_t> owner_;  // the owner map the store was made for
  double fill_s_ = 0;
};

// A re-plan's migration: fills `dst` (allocated for `new_owner`, this rank's units of it in key order) with every
// unit from where it lives now, `old_owner` / `old_base` (each rank's current store as seen from this process: a
// peer's over NVLink, this rank's own in HBM), by the land kernel on `stream`; returns after the copies landed. Every
// unit of dst must be owned under old_owner (a unit joining the tier is read from its file by a new store instead).
struct Migration {
  uint64_t units = 0, peer_units = 0, bytes = 0;
  double seconds = 0;
};
Migration migrate_store(PeerStore& dst, const std::vector<int32_t>& old_owner, const std::vector<char*>& old_base,
                        void* stream);

// This rank's share of a tier's check against the descriptor's hashes: the owned units whose position among the
// owned keys is rank modulo world, each gathered whole from the stores (t.pieces) into a scratch buffer on `device`
// and hashed there by K3, in batches of at most 2 GiB. Returns the units checked; SS_E_HASH names the mismatches.
// Every rank calls it once all stores are filled and mapped; together they check every owned unit once.
uint64_t verify_tier(const Desc& d, const PeerTier& t, int device);

}  // namespace tsb
