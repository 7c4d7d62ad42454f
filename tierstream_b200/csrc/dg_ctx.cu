// Device-gated decode on a B200: the context behind ss_open(forward_mode = SS_FORWARD_DEVICE_GATED).
//
// Memory (one context, one device):
//   HBM    arena: one array per part, `slots` entries of part bytes each (residents, spares, 2 banks, zeroed guard);
//          slot_of[keys]; control words (seq, abort, errors, any_miss[G], ready[G], unit_base[G + 1], absent_err)
//          and one completion counter per copy stream for the land kernel.
//   pinned blocks: P + Q units at a 4 KiB host stride, mapped (the land kernel reads them over PCIe), <= 1 GiB chunks;
//          one staging unit for reset cycles; a mapped control area with the export records and flags.
// Per token the engine's graph runs begin / export / wait / end (kernels.cu); a service thread spins on the mapped
// export flags and drives the slot cache (dg_core.cpp) whose copies, entries and ready words go to the CudaMover: one
// land-kernel launch per batch (copies, then entries, then ready, published by its last block), or the copy engines
// plus stream writes when a part is large enough for them to be faster.
#include <cuda.h>
#include <cuda_runtime.h>
#include <immintrin.h>

#include <algorithm>
#include <numeric>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <memory>
#include <condition_variable>
#include <deque>
#include <mutex>
#include <thread>

#include "ctx.hpp"
#include "dg_core.hpp"
#include "errors.hpp"
#include "kernels.hpp"
#include "loader.hpp"
#include "peer.hpp"
#include "pinned.hpp"
#include "score_profile.hpp"
#include "source_file.hpp"
#include "xxh64.hpp"

namespace tsb {
namespace {

using Clock = std::chrono::steady_clock;

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    fail(e == cudaErrorMemoryAllocation ? SS_E_NOMEM : SS_E_BACKEND,
         std::string(what) + ": " + cudaGetErrorString(e));
  }
}
// The few driver functions used here, resolved through the runtime (cudaGetDriverEntryPoint) at the first open: the
// library links no libcuda, so it loads on a machine without a driver (the CPU tests).
struct Driver {
  CUresult (*write_value32)(CUstream, CUdeviceptr, cuuint32_t, unsigned int) = nullptr;
  CUresult (*error_string)(CUresult, const char**) = nullptr;
  CUresult (*loading_mode)(CUmoduleLoadingMode*) = nullptr;
};
const Driver& driver() {
  static const Driver d = [] {
    Driver x;
    cudaDriverEntryPointQueryResult q{};
    auto get = [&](const char* name, void** fn) {
      if (cudaGetDriverEntryPoint(name, fn, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
        *fn = nullptr;
    };
    get("cuStreamWriteValue32", reinterpret_cast<void**>(&x.write_value32));
    get("cuGetErrorString", reinterpret_cast<void**>(&x.error_string));
    get("cuModuleGetLoadingMode", reinterpret_cast<void**>(&x.loading_mode));
    return x;
  }();
  return d;
}
void ck_drv(CUresult r, const char* what) {
  if (r != CUDA_SUCCESS) {
    const char* s = nullptr;
    if (driver().error_string) driver().error_string(r, &s);
    fail(SS_E_BACKEND, std::string(what) + ": " + (s ? s : "CUDA driver error"));
  }
}
CUresult write_value32(CUstream s, CUdeviceptr p, cuuint32_t v) {
  require(driver().write_value32 != nullptr, SS_E_BACKEND, "cuStreamWriteValue32 is not available from the driver");
  return driver().write_value32(s, p, v, CU_STREAM_WRITE_VALUE_DEFAULT);
}
void ck_launch(int e, const char* what) { ck(cudaError_t(e), what); }

inline uint32_t load_acquire(const uint32_t* p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }
inline void store_release(uint32_t* p, uint32_t v) { __atomic_store_n(p, v, __ATOMIC_RELEASE); }
inline void cpu_relax() { _mm_pause(); }

double us_between(Clock::time_point a, Clock::time_point b) {
  return std::chrono::duration<double, std::micro>(b - a).count();
}

// ---------------------------------------------------------------------------------------------------------------
// Layout: what an open needs from the descriptor, the plan and the options, with the reference's refusals
// (dg_layout.cpp:183-411) for everything this build supports.
// ---------------------------------------------------------------------------------------------------------------
struct Layout {
  std::vector<int> gated;           // descriptor layer of each gated ordinal
  std::vector<int> ordinal;         // per descriptor layer, -1 when not gated
  std::vector<uint32_t> unit_base;  // G + 1
  std::vector<uint64_t> part_bytes, part_offset;
  uint64_t unit_bytes = 0, host_stride = 0;
  uint32_t keys = 0, R = 0, D = 0, B = 0, P = 0, Q = 0, I = 0;
  uint32_t persistent_slots = 0, slots = 0, guard_slot = 0, blocks = 0;
  std::vector<uint32_t> residents;  // keys of tier R, key order
  // file tier (dg_disk_tier): F units of tier DISK (flagged per key in `disk`), S staging buffers after the blocks
  bool disk_tier = false, disk_prefetch = false;
  uint32_t F = 0, S = 0, disk_queue = 0;
  std::vector<uint8_t> disk;
  // landing blocks (dg_landing_blocks, file tier only): L blocks after the staging buffers; the landing reads at once
  // (dg_landing_max_queued, 0 = 1), the TTL and the chunk size (0 = whole reads)
  uint32_t L = 0, landing_queued = 1, landing_ttl = 0, landing_chunk = 0;
  // scored eviction (SS_POLICY_SCORED / SCORED_AUTO): the weights and a profile's counts (empty: none)
  bool scored = false, scored_auto = false;
  uint32_t w_trans = 700, w_freq = 200, w_rec = 100;
  std::vector<std::vector<uint32_t>> profile;
  std::string provenance;
};

[[noreturn]] void dg_refuse(ss_status st, const std::string& why) { fail(st, "device-gated: " + why); }

// The options an open checks before it reads the descriptor. Every SS_E_INVALID refusal comes before the
// SS_E_UNSUPPORTED ones, so a set of options with several faults gets the reference's status (dg_layout.cpp:183-215).
void check_dg_options(const ss_budget& b, const ss_options& o, const PeerTier* peer) {
  constexpr uint32_t kQueueAuto = 0xFFFFFFFFu;
  struct Need {
    bool ok;
    const char* why;
  };
  const Need invalid[] = {
      {b.tier_mode == SS_TIER_MODE_EXCLUSIVE, "needs tier_mode EXCLUSIVE"},
      {!b.pinned_backing, "pinned_backing is refused (each unit has one home)"},
      {o.policy == SS_POLICY_LRU || o.policy == SS_POLICY_SCORED || o.policy == SS_POLICY_SCORED_AUTO,
       "policy must be LRU, SCORED or SCORED_AUTO"},
      {!(o.dg_score_profile_len || o.dg_score_profile) || o.policy != SS_POLICY_LRU,
       "dg_score_profile needs policy SCORED"},
      {!o.pin_planned, "needs pin_planned = 0 (planned residents are a warm start)"},
      {o.fill_residents != 0, "needs fill_residents = 1 (a resident's slot is its only copy)"},
      {!o.readahead_units, "readahead_units must be 0 (no gated unit is read from its file)"},
      {!o.spec_persistent, "spec_persistent is refused (prediction is the service's)"},
      {o.dg_max_ids >= 1 && o.dg_max_ids <= dev::kMaxIds, "dg_max_ids must be 1..64 (rows x top_k)"},
      {o.dg_wait_timeout_ms >= 1, "dg_wait_timeout_ms must be >= 1"},
      {o.dg_disk_tier <= 1 && o.dg_disk_prefetch <= 1, "dg_disk_tier / dg_disk_prefetch must be 0 or 1"},
      {o.dg_disk_tier || !(o.dg_disk_prefetch || o.dg_disk_staging || (o.dg_disk_queue && o.dg_disk_queue != kQueueAuto)),
       "dg_disk_prefetch / dg_disk_staging / dg_disk_queue need dg_disk_tier = 1"},
      {o.dg_disk_staging <= 256, "dg_disk_staging must be 0..256"},
      {o.dg_disk_queue <= 64 || o.dg_disk_queue == kQueueAuto, "dg_disk_queue must be 0..64 or SS_DG_DISK_QUEUE_AUTO"},
      {o.dg_bank_keep <= 2, "dg_bank_keep must be 0, 1 or 2"},
      {o.dg_landing_blocks <= 4096, "dg_landing_blocks must be 0..4096"},
      {o.dg_landing_blocks || !(o.dg_landing_max_queued || o.dg_landing_ttl || o.dg_landing_chunk),
       "dg_landing_max_queued / dg_landing_ttl / dg_landing_chunk need dg_landing_blocks > 0"},
      {o.dg_landing_max_queued <= 64, "dg_landing_max_queued must be 0..64"},
      {o.dg_landing_ttl <= 1024, "dg_landing_ttl must be 0..1024"},
      {o.dg_landing_chunk == 0xFFFFFFFFu || o.dg_landing_chunk % 4096 == 0,
       "dg_landing_chunk must be 0, a multiple of 4096 or 0xFFFFFFFF (no chunks)"},
      {!o.dg_landing_blocks || o.dg_disk_tier, "dg_landing_blocks needs dg_disk_tier = 1"},
      {!o.dg_landing_blocks || o.dg_disk_queue > 1,
       "dg_landing_blocks needs dg_disk_queue > 1 (the landing reads run on the read pool)"},
      {o.dg_disk_queue_adapt <= 1, "dg_disk_queue_adapt must be 0 or 1"},
      {!o.dg_disk_queue_adapt || (o.dg_disk_tier && o.dg_disk_queue == kQueueAuto),
       "dg_disk_queue_adapt needs dg_disk_tier = 1 and dg_disk_queue = SS_DG_DISK_QUEUE_AUTO"},
  };
  for (const Need& n : invalid)
    if (!n.ok) dg_refuse(SS_E_INVALID, n.why);
  // switches that are 0 or 1
  const std::pair<uint32_t, const char*> flags[] = {
      {o.dg_wb_defer, "dg_wb_defer"},         {o.dg_wb_stream, "dg_wb_stream"},
      {o.dg_no_admit, "dg_no_admit"},         {o.dg_clean_evict, "dg_clean_evict"},
      {o.dg_pf_revert_unused, "dg_pf_revert_unused"}, {o.dg_pf_strict_admit, "dg_pf_strict_admit"},
  };
  for (const auto& f : flags)
    if (f.first > 1) dg_refuse(SS_E_INVALID, std::string(f.second) + " must be 0 or 1");
  if (o.dg_disk_tier && peer) dg_refuse(SS_E_UNSUPPORTED, "the file tier with the peer tier is not in this build");
  if (o.dg_prior_len)
    dg_refuse(SS_E_UNSUPPORTED, "dg_prior_len (window prefetch priors) is not in this build");
}

// The gated layers (every layer with units; each must be streamable) and the one part shape they share: the arena
// is a single array of slots, each the concatenation of the parts (each a multiple of 256 bytes).
void gate_layers(const Desc& d, Layout& x) {
  x.ordinal.assign(d.layers.size(), -1);
  for (size_t L = 0; L < d.layers.size(); ++L) {
    const Layer& l = d.layers[L];
    if (l.n_units == 0) continue;
    const std::string name = "layer " + std::to_string(l.index);
    if (!l.streamable) dg_refuse(SS_E_UNSUPPORTED, name + " has non-streamable units (every unit is gated)");
    if (x.gated.empty()) {  // the shape
      if (l.parts.size() > SS_DG_MAX_PARTS)
        dg_refuse(SS_E_UNSUPPORTED, "more than " + std::to_string(SS_DG_MAX_PARTS) + " parts per unit");
      uint64_t at = 0;
      for (const Part& part : l.parts) {
        if (part.bytes % 256)
          dg_refuse(SS_E_UNSUPPORTED, "part " + part.name + " is " + std::to_string(part.bytes) +
                                          " bytes, not a multiple of 256 (the arena stride equals the part bytes)");
        x.part_offset.push_back(at);
        x.part_bytes.push_back(part.bytes);
        at += part.bytes;
      }
      x.unit_bytes = l.unit_bytes;
    } else {
      const std::vector<Part>& first = d.layers[size_t(x.gated[0])].parts;
      const bool same = std::equal(l.parts.begin(), l.parts.end(), first.begin(), first.end(),
                                   [](const Part& a, const Part& c) { return a.bytes == c.bytes; });
      if (!same) dg_refuse(SS_E_UNSUPPORTED, name + " has another part shape (one arena)");
    }
    x.ordinal[L] = int(x.gated.size());
    x.gated.push_back(int(L));
  }
  if (x.gated.empty()) dg_refuse(SS_E_INVALID, "the descriptor has no streamable units");
  x.host_stride = host_stride(x.unit_bytes);
}

// Every gated unit's home from the plan (resident, pinned, or with the file tier its file), keys in descriptor order;
// the spare slots the plan billed: per layer its dynamic slots, never more than its non-resident units.
void place_homes(const Desc& d, const Plan& p, const ss_options& o, Layout& x) {
  const bool files = o.dg_disk_tier != 0;
  uint64_t key = 0;
  x.unit_base.assign(1, 0);
  for (int L : x.gated) {
    const Layer& l = d.layers[size_t(L)];
    const size_t first = size_t(d.unit_base[size_t(L)]);
    uint32_t resident_here = 0;
    for (int u = 0; u < l.n_units; ++u, ++key) {
      const uint8_t tier = p.tier[first + size_t(u)];
      const bool to_file = files && tier == SS_TIER_DISK;
      if (tier == SS_TIER_RESIDENT) {
        x.residents.push_back(uint32_t(key));
        ++resident_here;
      } else if (tier == SS_TIER_PINNED || to_file) {
        ++(to_file ? x.F : x.P);
      } else {
        dg_refuse(SS_E_CAPACITY, "unit (" + std::to_string(l.index) + ", " + std::to_string(u) +
                                     ") is not resident or pinned (no gated unit is read from its file)");
      }
      if (files) x.disk.push_back(uint8_t(to_file));
    }
    x.D += std::min<uint32_t>(p.budget.dynamic_slots_per_layer, uint32_t(l.n_units) - resident_here);
    require(key < 0x7fffffffull, SS_E_INVALID, "device-gated: more than 2^31 - 1 gated units");
    x.unit_base.push_back(uint32_t(key));
  }
  x.keys = uint32_t(key);
  x.R = uint32_t(x.residents.size());
  // file reads in flight and their staging buffers (dg_layout.cpp:159-181, one location per source here): AUTO is
  // 4 bounded by an explicit staging count, an explicit 0 means 1; staging defaults to 8 buffers
  x.disk_tier = files;
  x.disk_prefetch = o.dg_disk_prefetch != 0;
  if (files) {
    const uint32_t staging = o.dg_disk_staging;
    x.disk_queue = o.dg_disk_queue == 0xFFFFFFFFu ? std::min<uint32_t>(4, staging ? staging : 4)
                                                  : std::max<uint32_t>(1, o.dg_disk_queue);
    x.S = staging ? staging : 8u;
  }
  // landing blocks only with file units (nothing to land otherwise: dg_layout.cpp:343-347)
  x.L = files ? o.dg_landing_blocks : 0u;
  x.landing_queued = o.dg_landing_max_queued ? o.dg_landing_max_queued : 1u;
  x.landing_ttl = o.dg_landing_ttl;
  x.landing_chunk = o.dg_landing_chunk == 0xFFFFFFFFu ? 0u : o.dg_landing_chunk ? o.dg_landing_chunk : 4u << 20;
}

// Scored eviction (dg_layout.cpp:349-371): the three weights (per mille, summing to 1000, or all 0 for the
// defaults), at most 65536 units per gated layer, and a profile checked against this descriptor's identity.
void resolve_scoring(const Desc& d, const ss_options& o, Layout& x) {
  if (o.policy != SS_POLICY_SCORED && o.policy != SS_POLICY_SCORED_AUTO) return;
  x.scored = true;
  x.scored_auto = o.policy == SS_POLICY_SCORED_AUTO;
  const uint32_t w[3] = {o.dg_score_w_trans, o.dg_score_w_freq, o.dg_score_w_recency};
  if (w[0] || w[1] || w[2]) {
    const bool each = w[0] <= 1000 && w[1] <= 1000 && w[2] <= 1000;
    if (!each || w[0] + w[1] + w[2] != 1000)
      dg_refuse(SS_E_INVALID, "dg_score_w_trans / _freq / _recency must each be 0..1000 and sum to 1000");
    x.w_trans = w[0];
    x.w_freq = w[1];
    x.w_rec = w[2];
  }
  std::vector<uint32_t> units;
  units.reserve(x.gated.size());
  for (int L : x.gated) {
    const Layer& l = d.layers[size_t(L)];
    if (l.n_units > 65536)
      dg_refuse(SS_E_INVALID, "scored eviction needs at most 65536 units per gated layer (layer " +
                                  std::to_string(l.index) + ")");
    units.push_back(uint32_t(l.n_units));
  }
  if (!o.dg_score_profile && !o.dg_score_profile_len) return;
  if (!o.dg_score_profile || !o.dg_score_profile_len)
    dg_refuse(SS_E_INVALID, "dg_score_profile and dg_score_profile_len must be given together");
  ScoreProfile prof = check_score_profile(o.dg_score_profile, o.dg_score_profile_len, units, score_identity(d, x.gated));
  x.profile = std::move(prof.cells);
  x.provenance = std::move(prof.provenance);
}

// Slots and blocks: R + D persistent slots (D the billed spare slots, or dg_spare_slots), then two banks of B and the
// guard; P + Q pinned blocks (Q the plan's spare blocks, at least one kept free of the inclusive share); and the two
// admissions - the arena against the device cap less the margin, the staging units against the pinned budget.
void size_arena(const Desc& d, const Plan& p, const ss_options& o, const PeerTier* peer, Layout& x) {
  const ss_budget& b = p.budget;
  if (o.dg_spare_slots) {
    if (o.dg_spare_slots > x.P + x.F)
      dg_refuse(SS_E_INVALID, "dg_spare_slots " + std::to_string(o.dg_spare_slots) + " above the non-resident units (" +
                                  std::to_string(x.P + x.F) + ")");
    x.D = o.dg_spare_slots;
  }
  if (x.D == 0) dg_refuse(SS_E_INVALID, "needs dynamic_slots_per_layer > 0 or dg_spare_slots > 0 (the spare slots)");
  const uint64_t want_ring = 2ull * x.B + 1;
  const uint64_t stride = d.unit_stride(x.gated[0]);
  uint32_t ring_slots = 0;  // (of the ring class with the gated units' stride)
  for (const RingClass& rc : p.rings)
    if (rc.stride == stride) ring_slots = rc.slots;
  if (ring_slots < want_ring)
    dg_refuse(SS_E_CAPACITY, "the plan bills " + std::to_string(ring_slots) + " ring slots, the banks and the guard need " +
                                 std::to_string(want_ring) + " (set ring_slots = 2 x dg_max_ids + 1)");
  for (const SpareClass& sc : p.spares)
    if (sc.block_bytes == x.host_stride) x.Q = sc.blocks;
  if (x.Q == 0)
    dg_refuse(SS_E_CAPACITY, "the plan granted no spare blocks (host_spare_units asked " +
                                 std::to_string(b.host_spare_units) + "): a write-back needs a free block");
  x.blocks = x.P + x.Q;
  x.I = o.dg_inclusive_blocks;
  if (x.I && x.I >= x.Q)
    dg_refuse(SS_E_CAPACITY, "dg_inclusive_blocks " + std::to_string(x.I) + " must stay below the spare blocks (" +
                                 std::to_string(x.Q) + "): raise host_spare_units by the inclusive share");
  x.persistent_slots = x.R + x.D;
  const uint64_t all_slots = uint64_t(x.persistent_slots) + want_ring;
  require(all_slots < 0x7fffffffull, SS_E_INVALID, "device-gated: more than 2^31 - 1 slots");
  x.slots = uint32_t(all_slots);
  x.guard_slot = x.slots - 1;
  // device: the arena and the published table in place of what the plan billed for gated slots
  const uint64_t slot_bytes = std::accumulate(x.part_bytes.begin(), x.part_bytes.end(), uint64_t(0));
  const uint64_t arena = all_slots * slot_bytes + uint64_t(x.keys) * 4 + 4096;
  const uint64_t billed = p.resident + p.dynamic + p.ring;
  const uint64_t rest = p.peak >= billed ? p.peak - billed : 0;
  const uint64_t room = p.cap > p.margin ? p.cap - p.margin : 0;
  if (rest + arena > room)
    dg_refuse(SS_E_CAPACITY, "the arena needs " + std::to_string(arena) + " bytes where the plan billed " +
                                 std::to_string(billed) + "; with the rest of the plan that is above the cap - margin");
  // host: the plan's pinned bytes, one reset unit and S staging units, and 1 MiB of mapped control words (none of
  // the blocks when every unit lives in a peer store)
  const bool no_blocks = peer && peer->all_owned;
  const uint64_t pinned = p.pinned + (1ull + x.S + x.L) * x.host_stride + (uint64_t(1) << 20);
  if (!no_blocks && pinned > b.host_pinned_bytes)
    dg_refuse(SS_E_CAPACITY, "the plan's pinned bytes plus the staging units, the landing blocks and the mapped "
                             "control area exceed the host budget (" + std::to_string(b.host_pinned_bytes) + ")");
}

Layout make_layout(const Desc& d, const Plan& p, const ss_options& o, const PeerTier* peer) {
  check_dg_options(p.budget, o, peer);
  Layout x;
  x.B = o.dg_max_ids;
  gate_layers(d, x);
  place_homes(d, p, o, x);
  resolve_scoring(d, o, x);
  size_arena(d, p, o, peer, x);
  return x;
}

// ---------------------------------------------------------------------------------------------------------------
// The CUDA mover: copies, entries, ready words and events on the three streams.
// ---------------------------------------------------------------------------------------------------------------
class CudaMover final : public Mover {
 public:
  struct Buffers {
    std::vector<char*> arena;     // per part, device
    std::vector<char*> blocks;    // host addresses (mapped)
    std::vector<char*> blocks_d;  // the same blocks, device addresses
    char* staging = nullptr;
    char* staging_d = nullptr;
    int32_t* slot_of = nullptr;   // device
    uint32_t* ready = nullptr;    // device, [G]
    uint32_t* counters = nullptr; // device, 3 (one per stream)
  };

  CudaMover(const Layout& x, const Buffers& b, const PeerTier* peer) : x_(x), b_(b), peer_(peer) {
    int lo = 0, hi = 0;
    ck(cudaDeviceGetStreamPriorityRange(&lo, &hi), "cudaDeviceGetStreamPriorityRange");
    ck(cudaStreamCreateWithPriority(&s_[kDem], cudaStreamNonBlocking, hi), "cudaStreamCreate (demand)");
    ck(cudaStreamCreateWithPriority(&s_[kPf], cudaStreamNonBlocking, lo), "cudaStreamCreate (prefetch)");
    ck(cudaStreamCreateWithFlags(&s_[kD2h], cudaStreamNonBlocking), "cudaStreamCreate (write-back)");
    ck(cudaHostAlloc(reinterpret_cast<void**>(&table_pin_), size_t(std::max<uint32_t>(x_.keys, 1)) * 4,
                     cudaHostAllocPortable),
       "cudaHostAlloc (table staging)");
    for (int i = 0; i < 3; ++i) batch_[i] = std::make_unique<dev::Batch>();
    // copy engines for parts at least this large (they measured faster there), the land kernel below it;
    // TSB_COPY_MODE=kernel | ce forces one mover, TSB_CE_MIN_BYTES moves the threshold
    ce_min_ = uint64_t(8) << 20;
    if (const char* e = std::getenv("TSB_CE_MIN_BYTES")) ce_min_ = std::strtoull(e, nullptr, 10);
    if (const char* e = std::getenv("TSB_LAND_INTERLEAVE")) interleave_ = std::strcmp(e, "0") != 0;
    if (const char* e = std::getenv("TSB_COPY_MODE")) {
      if (!std::strcmp(e, "kernel")) ce_min_ = UINT64_MAX;
      else if (!std::strcmp(e, "ce")) ce_min_ = 0;
    }
    deterministic_ = std::getenv("TSB_DG_DETERMINISTIC") && std::getenv("TSB_DG_DETERMINISTIC")[0] == '1';
  }
  ~CudaMover() override {
    for (cudaStream_t s : s_)
      if (s) cudaStreamSynchronize(s);
    for (cudaStream_t s : chk_.vs)
      if (s) cudaStreamSynchronize(s);
    for (cudaEvent_t e : chk_.land_ev)
      if (e) cudaEventDestroy(e);
    for (cudaStream_t s : chk_.vs)
      if (s) cudaStreamDestroy(s);
    if (table_pin_) cudaFreeHost(table_pin_);
    for (cudaEvent_t e : ev_a_)
      if (e) cudaEventDestroy(e);
    for (cudaEvent_t e : ev_b_)
      if (e) cudaEventDestroy(e);
    for (cudaStream_t s : s_)
      if (s) cudaStreamDestroy(s);
  }
  cudaStream_t stream(Stream s) const { return s_[s]; }
  bool deterministic() const { return deterministic_; }
  bool kernel_copies() const {
    return (peer_ && peer_->all_owned && peer_->copy == 0) || ce_min_ > x_.part_bytes[0];
  }
  uint64_t kernel_launches() const { return launches_; }
  uint64_t peer_units() const { return peer_units_; }
  uint64_t self_units() const { return self_units_; }
  uint64_t peer_bytes() const { return peer_bytes_; }
  uint64_t self_bytes() const { return self_bytes_; }

  uint32_t parts() const override { return uint32_t(x_.part_bytes.size()); }
  uint64_t part_bytes(uint32_t p) const override { return x_.part_bytes[p]; }

  void h2d(Stream s, int32_t slot, int32_t block, uint32_t key) override {
    check_hold(s, slot);
    if (peer_ && peer_->owned(key)) {  // from the stores: NVLink for a peer's, HBM for this GPU's own
      bool self = true;
      peer_->pieces(key, x_.unit_bytes, [&](const char* src, uint64_t off, uint64_t n, int32_t from) {
        for_parts(off, n, [&](uint32_t p, uint64_t a, uint64_t len) {  // the piece's span within part p
          char* dst = arena(p, slot) + (a - x_.part_offset[p]);
          if (peer_->copy == 1) {
            flush(s);
            ck(cudaMemcpyAsync(dst, src + (a - off), size_t(len), cudaMemcpyDefault, s_[s]),
               "cudaMemcpyAsync (store part)");
          } else {
            add_copy(s, src + (a - off), dst, len);
          }
        });
        self = self && from == peer_->rank;
        (from == peer_->rank ? self_bytes_ : peer_bytes_) += n;
      });
      ++(self ? self_units_ : peer_units_);
      // not hashed again on landing: the store was hashed on the device against the descriptor when it was filled and
      // nothing writes it while decoding; a unit hashes in ~75 ms (four serial lane chains) while a peer-tier token
      // lasts ~10 ms, so hashing store copies would hold their slots across several tokens
      return;
    }
    for (uint32_t p = 0; p < parts(); ++p)
      copy(s, block_dev(block) + x_.part_offset[p], arena(p, slot), x_.part_bytes[p], cudaMemcpyHostToDevice);
    check_add(s, key, slot);
  }
  void d2h(Stream s, int32_t slot, int32_t block, int32_t part, uint32_t key) override {
    if (peer_ && peer_->owned(key)) return;  // its store keeps its bytes: the block is bookkeeping only
    for (uint32_t p = 0; p < parts(); ++p) {
      if (part >= 0 && uint32_t(part) != p) continue;
      copy(s, arena(p, slot), block_dev(block) + x_.part_offset[p], x_.part_bytes[p], cudaMemcpyDeviceToHost);
    }
  }
  void d2d_moves(const std::vector<std::pair<int32_t, int32_t>>& moves, const std::vector<uint32_t>& wave) override {
    flush(kDem);
    check_fence(kDem);  // no move overwrites a slot whose landing is still being hashed
    uint32_t max_wave = 0;
    for (uint32_t w : wave) max_wave = std::max(max_wave, w);
    // K4 (TMA bulk copies through shared memory) per wave, stream-ordered on kDem; the arena's parts are 256-byte
    // multiples, so every move fits it (the land kernel takes one that does not, on the same stream)
    auto mb = std::make_unique<dev::Batch>();
    uint64_t chunks = 0;
    auto launch = [&] {
      if (!mb->n_copies) return;
      ck_launch(dev::launch_move(*mb, int(std::min<uint64_t>(std::max<uint64_t>(chunks, 1), 148)), s_[kDem]),
                "move kernel");
      ++launches_;
      mb->n_copies = 0;
      chunks = 0;
    };
    for (uint32_t w = 0; w <= max_wave; ++w) {
      for (size_t i = 0; i < moves.size(); ++i) {
        if (wave[i] != w) continue;
        for (uint32_t p = 0; p < parts(); ++p) {
          const char* src = arena(p, moves[i].first);
          char* dst = arena(p, moves[i].second);
          if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | x_.part_bytes[p]) & 15u) != 0) {
            add_copy(kDem, src, dst, x_.part_bytes[p]);
            continue;
          }
          if (mb->n_copies == dev::kMaxCopies) launch();
          mb->copies[mb->n_copies++] = {src, dst, x_.part_bytes[p]};
          chunks += (x_.part_bytes[p] + (64u << 10) - 1) >> 16;
        }
      }
      flush(kDem);  // the wave's copies, if any, that the move kernel cannot take
      launch();
    }
    sync(kDem);
    uint32_t timeouts = 0;
    ck_launch(dev::move_take_timeouts(&timeouts), "move kernel timeout word");
    require(!timeouts, SS_E_BACKEND, "device-gated: a staging copy of the move kernel did not complete");
  }
  // File tier: the unit from its file into a block or staging buffer (the context's checked read), synchronously.
  void read_unit(uint32_t key, int32_t block) override {
    require(reader_ != nullptr, SS_E_BACKEND, "device-gated: no file reader");
    reader_(key, block_host(block));
  }
  void set_reader(std::function<void(uint32_t, char*)> f) { reader_ = std::move(f); }
  void set_async(AsyncReads* a) { async_ = a; }
  void* read_begin(uint32_t key, int32_t block) override {
    if (!async_) {
      read_unit(key, block);
      return nullptr;
    }
    return async_->begin(key, block_host(block));
  }
  uint64_t read_end(void* h) override { return async_ && h ? async_->end(h) : 0; }
  bool read_done(void* h) override {
    if (!async_ || !h) return true;
    if (deterministic_) {  // the reference's immediate transport: every read complete when asked
      async_->wait(h);
      return true;
    }
    return async_->done(h);
  }
  // Landing reads: on the pool behind the demand reads (whole-unit reads), or the synchronous read with one reader.
  void* read_landing_begin(uint32_t key, int32_t block) override {
    if (!async_) {
      read_unit(key, block);
      return nullptr;
    }
    return async_->begin_landing(key, block_host(block));
  }
  uint64_t read_landing_end(void* h, LandingEnd* end) override {
    *end = LandingEnd{};
    return read_end(h);
  }
  bool read_landing_cancel(void* h, LandingEnd* end) noexcept override {
    *end = LandingEnd{};
    return async_ && h && !deterministic_ && async_->cancel(h);  // (immediate reads: nothing left to cancel)
  }
  void h2h(int32_t src, int32_t dst, uint32_t key) override {
    if (peer_ && peer_->owned(key)) return;
    std::memcpy(block_host(dst), block_host(src), size_t(x_.unit_bytes));
  }
  void publish(Stream s, uint32_t key, int32_t v) override {
    if (kernel_copies()) {
      dev::Batch& b = *batch_[s];
      if (b.n_entries == dev::kMaxEntries) flush(s);
      b.entry_key[b.n_entries] = key;
      b.entry_val[b.n_entries] = v;
      ++b.n_entries;
      return;
    }
    flush(s);
    ck_drv(write_value32(reinterpret_cast<CUstream>(s_[s]), reinterpret_cast<CUdeviceptr>(b_.slot_of + key),
                         cuuint32_t(v)),
           "cuStreamWriteValue32 (entry)");
  }
  void ready(uint32_t g, uint32_t seq) override {
    if (kernel_copies()) {
      dev::Batch& b = *batch_[kDem];
      b.ready_word = b_.ready + g;
      b.ready_val = seq;
      flush(kDem, true);
    } else {
      flush(kDem);
      ck_drv(write_value32(reinterpret_cast<CUstream>(s_[kDem]), reinterpret_cast<CUdeviceptr>(b_.ready + g),
                           cuuint32_t(seq)),
             "cuStreamWriteValue32 (ready)");
    }
    check_submit(kDem);  // behind the ready word: the engine never waits for the check
  }
  void* event_create() override {
    cudaEvent_t e = nullptr;
    ck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
    return e;
  }
  void event_destroy(void* ev) override {
    if (ev) cudaEventDestroy(static_cast<cudaEvent_t>(ev));
  }
  void record(void* ev, Stream s) override {
    flush(s);
    ck(cudaEventRecord(static_cast<cudaEvent_t>(ev), s_[s]), "cudaEventRecord");
    check_submit(s);
  }
  void wait(Stream s, void* ev) override {
    flush(s);
    ck(cudaStreamWaitEvent(s_[s], static_cast<cudaEvent_t>(ev), 0), "cudaStreamWaitEvent");
  }
  bool done(void* ev) override {
    if (deterministic_) {  // the reference's immediate transport: every event complete when asked
      ck(cudaEventSynchronize(static_cast<cudaEvent_t>(ev)), "cudaEventSynchronize");
      return true;
    }
    const cudaError_t e = cudaEventQuery(static_cast<cudaEvent_t>(ev));
    if (e == cudaErrorNotReady) return false;
    ck(e, "cudaEventQuery");
    return true;
  }
  void event_sync(void* ev) override { ck(cudaEventSynchronize(static_cast<cudaEvent_t>(ev)), "cudaEventSynchronize"); }
  void sync(Stream s) override {
    flush(s);
    check_submit(s);
    ck(cudaStreamSynchronize(s_[s]), "cudaStreamSynchronize");
  }
  void upload_table(const int32_t* t, uint32_t n) override {
    flush(kDem);
    std::memcpy(table_pin_, t, size_t(n) * 4);
    ck(cudaMemcpyAsync(b_.slot_of, table_pin_, size_t(n) * 4, cudaMemcpyHostToDevice, s_[kDem]), "cudaMemcpyAsync (table)");
    ck(cudaStreamSynchronize(s_[kDem]), "cudaStreamSynchronize (table)");
  }
  // Each range staged in the pinned mirror and copied on its own; the rest of the device table is never written. A
  // copy that fails to enqueue lets those already enqueued finish first (they read the staging the retry refills).
  void upload_table_ranges(const int32_t* t, const uint32_t* ranges, uint32_t n) override {
    flush(kDem);
    try {
      for (uint32_t i = 0; i < n; ++i) {
        const size_t first = ranges[2 * i], count = ranges[2 * i + 1];
        std::memcpy(table_pin_ + first, t + first, count * 4);
        ck(cudaMemcpyAsync(b_.slot_of + first, table_pin_ + first, count * 4, cudaMemcpyHostToDevice, s_[kDem]),
           "cudaMemcpyAsync (table range)");
      }
    } catch (...) {
      cudaStreamSynchronize(s_[kDem]);
      throw;
    }
    ck(cudaStreamSynchronize(s_[kDem]), "cudaStreamSynchronize (table)");
  }
  void drain_all() noexcept {
    for (cudaStream_t s : s_)
      if (s) cudaStreamSynchronize(s);
  }
  void gate(Stream s, cudaEvent_t ev) {
    flush(s);
    ck(cudaStreamWaitEvent(s_[s], ev, 0), "cudaStreamWaitEvent (test gate)");
  }
  // dg_diag: timing events around each layer's demand work on kDem (its copies, entries and ready)
  void enable_diag(uint32_t G) {
    ev_a_.assign(G, nullptr);
    ev_b_.assign(G, nullptr);
    used_.assign(G, 0);
    dma_ms_.assign(G, -1.0);
    for (uint32_t g = 0; g < G; ++g) {
      ck(cudaEventCreate(&ev_a_[g]), "cudaEventCreate (diag)");
      ck(cudaEventCreate(&ev_b_[g]), "cudaEventCreate (diag)");
    }
  }
  void diag_mark(uint32_t g, int which) override {
    if (g >= ev_a_.size()) return;
    flush(kDem);
    ck(cudaEventRecord(which == 0 ? ev_a_[g] : ev_b_[g], s_[kDem]), "cudaEventRecord (diag)");
    if (which == 1) used_[g] = 1;
  }
  // After the boundary synced kDem: each marked layer's demand device time; their sum is kept since open.
  void diag_collect() {
    for (size_t g = 0; g < used_.size(); ++g) {
      dma_ms_[g] = -1;
      if (!used_[g]) continue;
      float ms = 0;
      if (cudaEventElapsedTime(&ms, ev_a_[g], ev_b_[g]) == cudaSuccess) {
        dma_ms_[g] = ms;
        dma_total_ms_ += ms;
      }
      used_[g] = 0;
    }
  }
  double dma_ms(uint32_t g) const { return g < dma_ms_.size() ? dma_ms_[g] : -1; }
  double dma_total_ms() const { return dma_total_ms_; }

  // ---- The landing check (verify_hash with descriptor hashes) ----
  // Every unit copied into a slot from host memory (demand, prefetch, placement round, kept-resident set; from a pinned
  // block or a file's staging buffer) is hashed on the device by K3 over the landed slot, after the copies of its stream
  // (a copy from a peer store is not: the store was hashed on the device when it was filled, see h2d) (after
  // the layer's ready word for demand copies, so the engine never waits for it), and compared with its descriptor hash;
  // a mismatch is logged in mapped memory for the host. One unit's hash is a serial chain (about 70 ms for a 99 MB
  // unit), so launches run side by side on a pool of low-priority streams, a launch on a stream whose last launch has
  // finished. When every stream is busy, landings stay pending and join the next launch (a launch hashes all its units
  // at once), so the hashing keeps up with any landing rate without the host waiting: the boundary submits what is left.
  // Launches are numbered; each one's last CTA writes its number to its word of a mapped ring when it finished (no event
  // is recorded after a hash: an event record behind a 70 ms kernel would hold every stream that shares its hardware
  // queue). slot_gen[slot] is the last launch that reads a slot; a copy into a slot whose landing is pending or being
  // hashed first submits it and waits for it on the host, so a hash never reads a slot being overwritten. Nothing here
  // changes a decision of the slot cache.
  struct CheckWords {
    const uint64_t* expect;  // [keys], device
    uint32_t* bad_count;     // device
    uint32_t* bad_log;       // mapped, device address
    uint32_t* bad_flag;      // mapped, device address
    uint32_t* timeouts;      // device
    uint32_t* done_cnt;      // device, kCheckRing words (zeroed)
    uint32_t* done_dev;      // mapped, kCheckRing words: device address
    const uint32_t* done_host;  // the same words: host address
  };
  static constexpr uint32_t kCheckRing = 256;
  struct CheckStats {
    uint64_t units = 0, bytes = 0, launches = 0, hold_waits = 0, merged = 0;
  };
  void enable_check(const CheckWords& w) {
    int lo = 0, hi = 0;
    ck(cudaDeviceGetStreamPriorityRange(&lo, &hi), "cudaDeviceGetStreamPriorityRange");
    chk_.vs.assign(kCheckStreams, nullptr);
    chk_.last_on.assign(kCheckStreams, 0);
    for (cudaStream_t& v : chk_.vs)
      ck(cudaStreamCreateWithPriority(&v, cudaStreamNonBlocking, lo), "cudaStreamCreate (landing check)");
    chk_.land_ev.assign(kCheckRing, nullptr);
    for (uint32_t i = 0; i < kCheckRing; ++i)
      ck(cudaEventCreateWithFlags(&chk_.land_ev[i], cudaEventDisableTiming), "cudaEventCreate (landing check)");
    chk_.slot_gen.assign(x_.slots, 0);
    chk_.slot_pending.assign(x_.slots, 0);
    chk_.w = w;
    chk_.on = true;
  }
  bool check_on() const { return chk_.on; }
  const CheckStats& check_stats() const { return chk_.st; }
  // Every landing so far submitted (on busy streams too), and the number of the last launch (a mark for check_wait).
  uint64_t check_mark() {
    for (Stream st : {kDem, kPf, kD2h}) check_submit(st, true);
    return chk_.launched;
  }
  // Host wait until every launch up to `mark` finished; returns the seconds waited.
  double check_wait(uint64_t mark) {
    if (!chk_.on || mark <= chk_.completed) return 0;
    check_poll();
    if (mark <= chk_.completed) return 0;
    const auto t0 = Clock::now();
    check_complete_through(mark);
    return std::chrono::duration<double>(Clock::now() - t0).count();
  }
  // Every landing submitted and hashed.
  void check_drain() {
    if (!chk_.on) return;
    check_wait(check_mark());
    for (cudaStream_t v : chk_.vs) ck(cudaStreamSynchronize(v), "cudaStreamSynchronize (landing check)");
  }

 private:
  static constexpr uint32_t kCheckStreams = 32;
  // Launch i finished: its done word holds i (or a later launch of the same ring entry).
  bool check_done(uint64_t i) const {
    return int32_t(load_acquire(chk_.w.done_host + i % kCheckRing) - uint32_t(i)) >= 0;
  }
  // Host wait until launch i finished (its hash waits are bounded, so it does: a launch silent for 30 s is a device
  // failure).
  void check_wait_one(uint64_t i) {
    if (check_done(i)) return;
    const auto deadline = Clock::now() + std::chrono::seconds(30);
    for (uint32_t spins = 0; !check_done(i); ++spins) {
      if ((spins & 1023u) == 0) {
        require(Clock::now() < deadline, SS_E_BACKEND, "device-gated: a landing check launch did not finish in 30 s");
        ck(cudaGetLastError(), "landing check");
      }
      if (spins < 4096) cpu_relax();
      else std::this_thread::yield();
    }
  }
  // Host wait for launches completed + 1 .. last.
  void check_complete_through(uint64_t last) {
    for (uint64_t i = chk_.completed + 1; i <= last; ++i) check_wait_one(i);
    chk_.completed = std::max(chk_.completed, last);
  }
  void check_poll() {
    while (chk_.completed < chk_.launched && check_done(chk_.completed + 1)) ++chk_.completed;
  }
  // Before a copy into `slot` on s: the slot's last landing has been hashed (its pending landing is submitted first; a
  // host wait, rare: a slot is reused long after its unit landed unless it is a bank slot).
  void check_hold(Stream s, int32_t slot) {
    if (!chk_.on) return;
    if (const uint8_t ps = chk_.slot_pending[size_t(slot)]) check_submit(Stream(ps - 1), true);
    const uint64_t g = chk_.slot_gen[size_t(slot)];
    if (g <= chk_.completed) return;
    check_poll();
    if (g <= chk_.completed || check_done(g)) return;
    ++chk_.st.hold_waits;
    flush(s);  // copies already batched on s do not wait
    check_wait_one(g);
  }
  // Before copies that may overwrite any slot (reset moves): every landing hashed.
  void check_fence(Stream s) {
    (void)s;
    if (!chk_.on) return;
    check_complete_through(check_mark());
  }
  void check_add(Stream s, uint32_t key, int32_t slot) {
    if (!chk_.on) return;
    chk_.pending[s].push_back({key, slot});
    chk_.slot_pending[size_t(slot)] = uint8_t(s + 1);
    if (chk_.pending[s].size() == dev::kMaxVerify) check_submit(s, true);
  }
  // One K3 launch over the landings pending on s, behind everything enqueued on s so far, on a check stream whose last
  // launch finished; with none free the landings stay pending unless `force` (then the stream whose last launch is the
  // oldest takes it, queued behind that launch).
  void check_submit(Stream s, bool force = false) {
    auto& p = chk_.pending[s];
    if (!chk_.on || p.empty()) return;
    uint32_t pick = kCheckStreams;
    for (uint32_t k = 0; k < kCheckStreams && pick == kCheckStreams; ++k) {
      const uint32_t i = (chk_.rr + k) % kCheckStreams;
      if (!chk_.last_on[i] || check_done(chk_.last_on[i])) pick = i;
    }
    if (pick == kCheckStreams) {
      if (!force) {
        ++chk_.st.merged;
        return;
      }
      pick = 0;
      for (uint32_t i = 1; i < kCheckStreams; ++i)
        if (chk_.last_on[i] < chk_.last_on[pick]) pick = i;
    }
    chk_.rr = (pick + 1) % kCheckStreams;
    flush(s);
    const uint64_t n = chk_.launched + 1;
    if (n > kCheckRing && chk_.completed < n - kCheckRing) {  // the ring's words of launch n - R are reused for n
      check_poll();
      if (chk_.completed < n - kCheckRing) check_complete_through(n - kCheckRing);
    }
    cudaStream_t vs = chk_.vs[pick];
    cudaEvent_t le = chk_.land_ev[n % kCheckRing];
    ck(cudaEventRecord(le, s_[s]), "cudaEventRecord (landing check)");
    ck(cudaStreamWaitEvent(vs, le, 0), "cudaStreamWaitEvent (landing check)");
    dev::VerifyBatch& b = *chk_.batch;
    b.n_parts = parts();
    for (uint32_t q = 0; q < b.n_parts; ++q) {
      b.arena[q] = reinterpret_cast<const uint8_t*>(b_.arena[q]);
      b.part_bytes[q] = x_.part_bytes[q];
    }
    b.n = uint32_t(p.size());
    b.expect = chk_.w.expect;
    b.bad_count = chk_.w.bad_count;
    b.bad_log = chk_.w.bad_log;
    b.bad_flag = chk_.w.bad_flag;
    b.timeouts = chk_.w.timeouts;
    b.done_cnt = chk_.w.done_cnt + n % kCheckRing;
    b.done_word = chk_.w.done_dev + n % kCheckRing;
    b.done_val = uint32_t(n);
    for (uint32_t i = 0; i < b.n; ++i) {
      b.key[i] = p[i].first;
      b.slot[i] = p[i].second;
    }
    ck_launch(dev::launch_xxh64_landed(b, vs), "xxh64 kernel (landing check)");
    chk_.launched = n;
    chk_.last_on[pick] = n;
    for (const auto& [key, slot] : p) {
      chk_.slot_gen[size_t(slot)] = n;
      chk_.slot_pending[size_t(slot)] = 0;
    }
    chk_.st.units += p.size();
    chk_.st.bytes += p.size() * x_.unit_bytes;
    ++chk_.st.launches;
    p.clear();
  }
  struct Check {
    bool on = false;
    std::vector<cudaStream_t> vs;
    std::vector<uint64_t> last_on;  // per check stream: its last launch (0: none)
    uint32_t rr = 0;                // where the search for a free stream starts
    CheckWords w{};
    std::vector<cudaEvent_t> land_ev;
    std::vector<uint64_t> slot_gen;
    std::vector<uint8_t> slot_pending;  // per slot: 1 + the copy stream of its pending landing, 0 = none
    std::vector<std::pair<uint32_t, int32_t>> pending[3];
    uint64_t launched = 0, completed = 0;
    std::unique_ptr<dev::VerifyBatch> batch = std::make_unique<dev::VerifyBatch>();
    CheckStats st;
  } chk_;

  char* arena(uint32_t p, int32_t slot) const { return b_.arena[p] + uint64_t(slot) * x_.part_bytes[p]; }
  // f(part, unit offset, bytes) for each part that [off, off + n) of the unit's bytes overlaps
  template <class F>
  void for_parts(uint64_t off, uint64_t n, F&& f) const {
    split_parts(x_.part_offset, x_.part_bytes, off, n, f);
  }
  char* block_dev(int32_t b) const { return b < 0 ? b_.staging_d : b_.blocks_d[size_t(b)]; }
  char* block_host(int32_t b) const { return b < 0 ? b_.staging : b_.blocks[size_t(b)]; }

  void copy(Stream s, const char* src, char* dst, uint64_t bytes, cudaMemcpyKind kind) {
    if (bytes >= ce_min_) {
      flush(s);
      ck(cudaMemcpyAsync(dst, src, size_t(bytes), kind, s_[s]), "cudaMemcpyAsync (part)");
      return;
    }
    add_copy(s, src, dst, bytes);
  }
  // The land kernel's blocks take a batch's 64 KiB chunks in list order, so at any moment nearly all of them read the
  // first copy. With copies from different sources (peers' stores over NVLink, this GPU's own store, pinned memory),
  // that leaves one source busy and the others idle for this batch while other GPUs contend for it; cutting the
  // copies into 4 MiB pieces taken round-robin keeps every source of the batch in flight at once. Left as it is when
  // the pieces would not fit the batch. (Measured in the 8-GPU Mixtral decode, 1.4 misses a layer: 7.31 against
  // 7.35 ms per token without it, within the noise.)
  static void interleave(dev::Batch& b) {
    constexpr uint64_t kPiece = uint64_t(4) << 20;
    if (b.n_copies < 2) return;
    uint64_t pieces = 0;
    for (uint32_t c = 0; c < b.n_copies; ++c) pieces += (b.copies[c].bytes + kPiece - 1) / kPiece;
    if (pieces <= b.n_copies || pieces > dev::kMaxCopies) return;
    dev::Copy whole[dev::kMaxCopies];
    std::copy(b.copies, b.copies + b.n_copies, whole);
    const uint32_t n = b.n_copies;
    uint64_t off[dev::kMaxCopies] = {};
    uint32_t out = 0;
    for (bool more = true; more;) {
      more = false;
      for (uint32_t c = 0; c < n; ++c) {
        if (off[c] >= whole[c].bytes) continue;
        const uint64_t len = std::min(kPiece, whole[c].bytes - off[c]);
        b.copies[out++] = {static_cast<const char*>(whole[c].src) + off[c], static_cast<char*>(whole[c].dst) + off[c],
                           len};
        off[c] += len;
        more = true;
      }
    }
    b.n_copies = out;
  }
  void add_copy(Stream s, const char* src, char* dst, uint64_t bytes) {
    dev::Batch& b = *batch_[s];
    if (b.n_copies == dev::kMaxCopies) flush(s);
    b.copies[b.n_copies++] = {src, dst, bytes};
    chunks_[s] += (bytes + (64u << 10) - 1) >> 16;
  }
  void flush(Stream s, bool force = false) {
    dev::Batch& b = *batch_[s];
    if (!b.n_copies && !b.n_entries && !b.ready_word && !force) return;
    b.slot_of = b_.slot_of;
    b.done_counter = b_.counters + s;
    if (interleave_) interleave(b);
    const int blocks = int(std::min<uint64_t>(std::max<uint64_t>(chunks_[s], 1), 296));
    ck_launch(dev::launch_batch(b, blocks, s_[s]), "land kernel");
    ++launches_;
    b.n_copies = b.n_entries = 0;
    b.ready_word = nullptr;
    chunks_[s] = 0;
  }

  const Layout& x_;
  Buffers b_;
  const PeerTier* peer_ = nullptr;
  std::function<void(uint32_t, char*)> reader_;
  AsyncReads* async_ = nullptr;
  uint64_t peer_units_ = 0, self_units_ = 0;  // owned units landed wholly from peers' stores / this GPU's own
  uint64_t peer_bytes_ = 0, self_bytes_ = 0;  // their bytes by source
  cudaStream_t s_[3] = {nullptr, nullptr, nullptr};
  int32_t* table_pin_ = nullptr;
  std::unique_ptr<dev::Batch> batch_[3];
  uint64_t chunks_[3] = {0, 0, 0};
  uint64_t ce_min_ = 0;
  bool interleave_ = true;  // a batch's large copies cut in 4 MiB pieces, taken round-robin (TSB_LAND_INTERLEAVE=0: off)
  uint64_t launches_ = 0;
  bool deterministic_ = false;
  std::vector<cudaEvent_t> ev_a_, ev_b_;
  std::vector<uint8_t> used_;
  std::vector<double> dma_ms_;
  double dma_total_ms_ = 0;
};

// ---------------------------------------------------------------------------------------------------------------
// The mapped control area: records, flags and words shared with the kernels (host and device addresses).
// ---------------------------------------------------------------------------------------------------------------
struct Mapped {
  dev::DgRecord* rec = nullptr;
  dev::DgPredRecord* prec = nullptr;
  uint32_t* flag = nullptr;
  uint32_t* pflag = nullptr;
  uint32_t* done = nullptr;
  uint32_t* err_code = nullptr;
  uint32_t* err_aux = nullptr;
  uint32_t* host_abort = nullptr;
  uint32_t* host_seq = nullptr;
  uint32_t* began = nullptr;
  uint32_t* err_count = nullptr;
};

struct LayerTimes {
  double seen_us = -1, demand_us = -1, pred_wait_us = -1, prefetch_us = -1, serve_us = -1;
  uint32_t ids = 0, misses = 0, covered = 0, fetched = 0, prefetched = 0, predicted_true = 0, covered_waits = 0;
};

// ---------------------------------------------------------------------------------------------------------------
// The service thread: waits for each exported layer's flag, serves it through the cache, publishes a terminal word.
// The protocol and its checks follow the reference's DgService (dg_service.cpp:116-365).
// ---------------------------------------------------------------------------------------------------------------
class Service {
 public:
  enum State : uint32_t { kIdle = 0, kServed = 1, kFailed = 2, kStopped = 3 };
  Service(SlotCache* core, const Mapped& m, uint32_t max_ids, uint32_t timeout_ms, int device, bool deterministic,
          bool diag)
      : core_(core), m_(m), max_ids_(max_ids), timeout_(std::chrono::milliseconds(timeout_ms)), device_(device),
        deterministic_(deterministic), diag_(diag) {
    const uint32_t G = core_->gated();
    run_.assign(G, 1);
    run_next_.assign(G, 1);
    last_flag_.assign(G, 0);
    times_.assign(G, LayerTimes{});
    ids_.reserve(dev::kMaxIds);
    pred_.reserve(dev::kMaxIds);
  }
  ~Service() { stop_join(); }
  void start() { th_ = std::thread([this] { run(); }); }
  void stop_join() {
    stop_.store(true, std::memory_order_release);
    if (th_.joinable()) th_.join();
  }
  // The engine thread, at ss_begin (release: the run flags, then the sequence).
  void begin(uint32_t seq, const std::vector<uint8_t>& run) {
    std::copy(run.begin(), run.end(), run_next_.begin());
    host_seq_.store(seq, std::memory_order_release);
  }
  // Waits (bounded) until the service published a terminal word for seq; returns its state.
  State wait_terminal(uint32_t seq, std::chrono::milliseconds left) {
    const auto deadline = Clock::now() + left;
    for (uint32_t spins = 0;; ++spins) {
      const uint64_t t = term_.load(std::memory_order_acquire);
      if (uint32_t(t) == seq && (t >> 32) != kIdle) return State(t >> 32);
      if ((t >> 32) == kStopped || (t >> 32) == kFailed) return State(t >> 32);
      if (Clock::now() > deadline) return kIdle;
      if (spins < 2000) cpu_relax();
      else std::this_thread::yield();
    }
  }
  std::string error() {
    std::lock_guard<std::mutex> lk(err_mu_);
    return err_;
  }
  const std::vector<LayerTimes>& times() const { return times_done_; }

 private:
  struct Stop {};
  void publish(State s, uint32_t seq) { term_.store(uint64_t(s) << 32 | seq, std::memory_order_release); }
  void fail_with(const std::string& msg) {
    {
      std::lock_guard<std::mutex> lk(err_mu_);
      if (err_.empty()) err_ = msg;
    }
    store_release(m_.host_abort, 1);  // every later wait kernel of the token returns at once
  }
  void wait_word(const uint32_t* w, uint32_t seq, const char* what, uint32_t g, bool strict, uint32_t last) {
    const auto start = Clock::now();
    for (uint32_t spins = 0;; ++spins) {
      const uint32_t v = load_acquire(w);
      if (v == seq) return;
      if (strict && v != last)
        fail(SS_E_BACKEND, std::string("device-gated: sequence desync: ") + what + " of gated layer " +
                               std::to_string(g) + " holds " + std::to_string(v) + " while serving token " +
                               std::to_string(seq));
      if ((spins & 4095u) == 0) {
        if (stop_.load(std::memory_order_acquire)) throw Stop{};
        if (Clock::now() - start > timeout_)
          fail(SS_E_BACKEND, std::string("device-gated: ") + what + " of gated layer " + std::to_string(g) +
                                 " never came (token " + std::to_string(seq) + ")");
      }
      cpu_relax();
    }
  }
  void wait_began(uint32_t seq) {
    for (uint32_t spins = 0;; ++spins) {
      const uint32_t v = load_acquire(m_.began);
      if (v == seq) return;
      if (int32_t(v - seq) > 0)
        fail(SS_E_BACKEND, "device-gated: sequence desync: a gated step began with seq " + std::to_string(v) +
                               " while serving token " + std::to_string(seq) +
                               " (a step ran outside ss_begin / ss_end)");
      if ((spins & 1023u) == 0) {
        if (stop_.load(std::memory_order_acquire)) throw Stop{};
        if (load_acquire(m_.host_abort)) throw Stop{};
      }
      if (spins < 20000) cpu_relax();
      else std::this_thread::yield();
    }
  }
  void serve_token(uint32_t seq) {
    const uint32_t G = core_->gated();
    std::copy(run_next_.begin(), run_next_.end(), run_.begin());
    core_->begin_token(seq, &run_);
    if (diag_) std::fill(times_.begin(), times_.end(), LayerTimes{});
    wait_began(seq);
    auto t_prev = Clock::now();
    for (uint32_t g = 0; g < G; ++g) {
      if (!run_[g]) continue;
      uint32_t nx = g + 1;
      while (nx < G && !run_[nx]) ++nx;
      wait_word(&m_.flag[g], seq, "export flag", g, true, last_flag_[g]);
      last_flag_[g] = seq;
      const auto t_seen = Clock::now();
      const dev::DgRecord& r = m_.rec[g];
      require(r.seq == seq, SS_E_BACKEND,
              "device-gated: sequence desync: the record of gated layer " + std::to_string(g) + " is for token " +
                  std::to_string(r.seq) + ", serving " + std::to_string(seq));
      const uint32_t n = r.n_ids, n_pred = r.n_pred_promised;
      require(n >= 1 && n <= max_ids_, SS_E_BACKEND,
              "device-gated: gated layer " + std::to_string(g) + " exported " + std::to_string(n) + " ids");
      require(n_pred <= dev::kMaxIds && (n_pred == 0 || g + 1 < G), SS_E_BACKEND,
              "device-gated: gated layer " + std::to_string(g) + " promised " + std::to_string(n_pred) +
                  " predicted ids");
      const uint64_t mask = uint64_t(r.mask_lo) | uint64_t(r.mask_hi) << 32;
      ids_.assign(r.ids, r.ids + n);
      const CacheStats before = core_->stats();
      core_->serve_demand(g, ids_.data(), n, mask);
      const auto t_demand = Clock::now();
      core_->serve_use(g, ids_.data(), n, mask);
      LayerTimes t;
      t.seen_us = us_between(t_prev, t_seen);
      t.demand_us = us_between(t_seen, t_demand);
      if (n_pred > 0 && run_[g + 1]) {
        wait_word(&m_.pflag[g], seq, "prediction flag", g, false, 0);
        const auto t_pw = Clock::now();
        t.pred_wait_us = us_between(t_demand, t_pw);
        const dev::DgPredRecord& pr = m_.prec[g];
        require(pr.n_pred == n_pred, SS_E_BACKEND,
                "device-gated: gated layer " + std::to_string(g) + " predicted " + std::to_string(pr.n_pred) +
                    " ids, its export promised " + std::to_string(n_pred));
        pred_.assign(pr.pred, pr.pred + n_pred);
        const bool ahead = !deterministic_ && load_acquire(&m_.flag[g + 1]) == seq;
        core_->serve_prediction(g + 1, pred_.data(), n_pred, ahead);
        t.prefetch_us = us_between(t_pw, Clock::now());
      }
      if (core_->deferred() && nx < G)
        core_->issue_writebacks(g, [&] { return !deterministic_ && load_acquire(&m_.flag[nx]) == seq; });
      if (core_->scored()) core_->score_layer(g);  // scored eviction: layer g is final for this token
      const auto t_end = Clock::now();
      t.serve_us = us_between(t_seen, t_end);
      if (diag_) {
        const CacheStats& a = core_->stats();
        t.ids = uint32_t(a.lookups - before.lookups);
        t.misses = uint32_t(a.misses - before.misses);
        t.covered = uint32_t(a.covered - before.covered);
        t.covered_waits = uint32_t(a.covered_waits - before.covered_waits);
        t.fetched = uint32_t(a.fetched - before.fetched);
        t.prefetched = uint32_t(a.prefetched - before.prefetched);
        t.predicted_true = uint32_t(a.predicted_true - before.predicted_true);
        times_[g] = t;
      }
      t_prev = t_end;
    }
  }
  void run() {
    if (cudaSetDevice(device_) != cudaSuccess) {
      fail_with("device-gated: the service thread cannot bind the device");
      publish(kFailed, 0);
      return;
    }
    uint32_t seen = 0;
    for (;;) {
      uint32_t seq = 0;
      for (uint32_t spins = 0;; ++spins) {
        seq = host_seq_.load(std::memory_order_acquire);
        if (seq != seen) break;
        if (stop_.load(std::memory_order_acquire)) {
          publish(kStopped, seen);
          return;
        }
        if (spins < 20000) cpu_relax();
        else std::this_thread::yield();
      }
      seen = seq;
      try {
        serve_token(seq);
        if (diag_) times_done_ = times_;
      } catch (const Stop&) {
        publish(kStopped, seq);
        return;
      } catch (const std::exception& e) {
        fail_with(e.what());
        publish(kFailed, seq);
        return;
      }
      publish(kServed, seq);
    }
  }

  SlotCache* core_;
  Mapped m_;
  uint32_t max_ids_;
  std::chrono::milliseconds timeout_;
  int device_;
  bool deterministic_, diag_;
  std::thread th_;
  std::atomic<bool> stop_{false};
  std::atomic<uint32_t> host_seq_{0};
  std::atomic<uint64_t> term_{0};
  std::mutex err_mu_;
  std::string err_;
  std::vector<uint8_t> run_, run_next_;
  std::vector<uint32_t> last_flag_, ids_, pred_;
  std::vector<LayerTimes> times_, times_done_;
};

// ---------------------------------------------------------------------------------------------------------------
// The context.
// ---------------------------------------------------------------------------------------------------------------
class CudaDgContext final : public DgContext {
 public:
  CudaDgContext(const Desc& d, const Plan& p, const ss_options& o, const PeerTier* peer)
      : d_(d), o_(o), peer_(peer ? std::make_unique<PeerTier>(*peer) : nullptr), x_(make_layout(d, p, o, peer)) {
    try {
      init();
    } catch (...) {
      close();
      throw;
    }
  }
  ~CudaDgContext() override { close(); }

  bool poisoned() const override { return poisoned_; }
  void poison() override { poisoned_ = true; }
  int device() const override { return o_.device; }
  int n_sources() const override { return int(files_.size()); }
  bool source_direct(int i) const override { return files_[size_t(i)]->direct(); }
  int gated_index(int layer) const override {
    return layer >= 0 && size_t(layer) < x_.ordinal.size() ? x_.ordinal[size_t(layer)] : -1;
  }

  void begin(const uint32_t* rows, int n_layers) override {
    require(!in_token_, SS_E_INVALID, "ss_begin: a gated token is already open (call ss_end)");
    if (rows) require(n_layers == int(d_.layers.size()), SS_E_INVALID, "ss_begin: rows_per_layer must cover every layer");
    const uint32_t G = uint32_t(x_.gated.size());
    for (uint32_t g = 0; g < G; ++g)  // (a held layer is not exported)
      run_[g] = uint8_t((rows ? rows[x_.gated[g]] != 0 : true) && !held_[g]);
    // no step ran outside a pair: every word still holds the last token's sequence
    bool clean = load_acquire(m_.done) == seq_ && load_acquire(m_.began) == seq_;
    for (uint32_t g = 0; clean && g < G; ++g)
      clean = int32_t(load_acquire(m_.flag + g) - seq_) <= 0 && int32_t(load_acquire(m_.pflag + g) - seq_) <= 0;
    if (!clean) {
      store_release(m_.host_abort, 1);
      svc_->stop_join();
      poisoned_ = true;
      fail(SS_E_BACKEND, "device-gated: sequence desync at ss_begin: a gated step ran outside ss_begin / ss_end (done " +
                             std::to_string(load_acquire(m_.done)) + ", began " + std::to_string(load_acquire(m_.began)) +
                             ", last token " + std::to_string(seq_) + "; the context is poisoned)");
    }
    ++seq_;
    in_token_ = true;
    store_release(m_.host_seq, seq_);
    svc_->begin(seq_, run_);
  }

  void end(uint32_t rows) override {
    require(in_token_, SS_E_INVALID, "ss_end: no gated token is open");
    in_token_ = false;
    const auto deadline = Clock::now() + std::chrono::milliseconds(uint64_t(o_.dg_wait_timeout_ms) + 5000);
    auto left = [&] {
      const auto now = Clock::now();
      return now < deadline ? std::chrono::duration_cast<std::chrono::milliseconds>(deadline - now)
                            : std::chrono::milliseconds(0);
    };
    if (!skip_edge_) {  // the end kernel ran after every reader of the token
      uint32_t v = 0;
      for (uint32_t spins = 0;; ++spins) {
        v = load_acquire(m_.done);
        if (v == seq_ || int32_t(v - seq_) > 0 || Clock::now() > deadline) break;
        if (spins < 20000) cpu_relax();
        else std::this_thread::yield();
      }
      const uint32_t began = load_acquire(m_.began);
      if (v != seq_ || began != seq_) {
        const std::string dev = device_error();
        store_release(m_.host_abort, 1);
        svc_->stop_join();
        poisoned_ = true;
        fail(SS_E_BACKEND, token_failure(dev, v == seq_ || int32_t(v - seq_) > 0
                                                  ? "sequence desync at ss_end: another gated step ran in it"
                                                  : "the device did not finish it (no end kernel)"));
      }
    }
    const Service::State st = svc_->wait_terminal(seq_, left());
    if (st != Service::kServed) {
      const std::string dev = device_error();
      store_release(m_.host_abort, 1);
      svc_->stop_join();
      poisoned_ = true;
      const std::string why = svc_->error();
      fail(SS_E_BACKEND, token_failure(dev, "the service: " + (why.empty() ? std::string("it did not finish") : why)));
    }
    const std::string dev = device_error();
    if (!dev.empty()) {
      poisoned_ = true;
      fail(SS_E_BACKEND, token_failure(dev, ""));
    }
    const auto t0 = Clock::now();
    core_->end_token(keep_all(), rows);
    boundary_.writebacks = uint32_t(core_->stats().evicted - evicted_before_);
    evicted_before_ = core_->stats().evicted;
    boundary_.sync_us = 0;
    boundary_.select_us = us_between(t0, Clock::now());
    if (o_.dg_diag) collect_diag();
    timeline_valid_ = true;
    if (mover_->check_on()) end_check();
  }

  // The landing check at ss_end: this token's landings are submitted, and those of the token before the previous one
  // have been hashed before the call returns, so a unit that landed wrong fails the ss_end of its own token or of one
  // of the next two (a 99 MB unit's hash takes longer than a token: waiting for the previous token's would stall). A
  // mismatch fails it with SS_E_HASH (a library error: the context stays usable) once every unit logged has been read
  // again from its file into its slot and, when it has one, its pinned block; the outputs of both tokens must be
  // discarded. A staging copy of the check that did not complete, or more mismatches than the log holds, is a device
  // failure (SS_E_BACKEND).
  void end_check() {
    const uint64_t mark = mover_->check_mark();
    check_wait_s_ += mover_->check_wait(check_marks_[0]);
    check_marks_[0] = check_marks_[1];
    check_marks_[1] = mark;
    if (!load_acquire(bad_flag_h_)) return;
    mover_->check_drain();  // every check issued so far has finished: the log is complete and nothing writes it
    uint32_t count = 0, touts = 0;
    ck(cudaMemcpy(&count, ctl_ + 6, 4, cudaMemcpyDeviceToHost), "cudaMemcpy (landing check)");
    ck(cudaMemcpy(&touts, ctl_ + 7, 4, cudaMemcpyDeviceToHost), "cudaMemcpy (landing check)");
    std::vector<std::pair<uint32_t, int32_t>> bad;
    for (uint32_t i = 0; i < std::min(count, dev::kBadLog); ++i)
      bad.push_back({bad_log_h_[2 * i], int32_t(bad_log_h_[2 * i + 1])});
    ck(cudaMemset(ctl_ + 6, 0, 8), "cudaMemset (landing check)");
    store_release(bad_flag_h_, 0);
    check_failed_ += count;
    if (touts || count > dev::kBadLog) {
      poisoned_ = true;
      fail(SS_E_BACKEND, touts ? "device-gated: a staging copy of the landing check did not complete in 2 s"
                               : "device-gated: " + std::to_string(count) +
                                     " landed units differ from their descriptor hashes, more than the check logs");
    }
    std::sort(bad.begin(), bad.end());
    bad.erase(std::unique(bad.begin(), bad.end(), [](auto& a, auto& b) { return a.first == b.first; }), bad.end());
    std::string names;
    for (const auto& [key, slot] : bad) {
      const uint32_t g = core_->gated_of(key);
      const int layer = x_.gated[g], unit = int(key - x_.unit_base[g]);
      names += (names.empty() ? "(" : ", (") + std::to_string(layer) + ", " + std::to_string(unit) + ")";
      repair(key);
    }
    fail(SS_E_HASH, "device-gated: landed bytes of unit(s) " + names +
                        " differ from their descriptor hashes (read again from their files; the outputs of this token and "
                        "the two before it must be discarded)");
  }

  // A unit whose landed bytes were wrong: every copy this context keeps of it (its slot, its pinned block) read again
  // from its file, checked against its descriptor hash on the host. Between tokens; the service is idle and every
  // landing check has finished.
  void repair(uint32_t key) {
    const uint32_t g = core_->gated_of(key);
    const int layer = x_.gated[g], unit = int(key - x_.unit_base[g]);
    const bool owned = peer_ && peer_->owned(key);
    const int32_t slot = core_->slot_of(key), block = core_->block_of(key);
    const bool in_slot = slot >= 0 && core_->home(key) != SlotCache::Home::Host && core_->home(key) != SlotCache::Home::File;
    if (!in_slot && (block < 0 || owned)) return;
    std::vector<char> bytes(size_t(x_.unit_bytes));
    read_checked(layer, unit, bytes.data(), readers_.get());
    if (in_slot)
      for (size_t p = 0; p < x_.part_bytes.size(); ++p)
        ck(cudaMemcpy(unit_part_dst(slot, uint32_t(p)), bytes.data() + x_.part_offset[p], size_t(x_.part_bytes[p]),
                      cudaMemcpyHostToDevice),
           "cudaMemcpy (repair)");
    if (block >= 0 && !owned) std::memcpy(bufs_.blocks[size_t(block)], bytes.data(), bytes.size());
    ++check_repaired_;
  }

  void seed(int layer, const int32_t* units, int n) override {
    require(!in_token_, SS_E_INVALID, "ss_seed: between tokens in device-gated mode");
    const int g = gated_index(layer);
    require(g >= 0, SS_E_INVALID, "ss_seed: layer " + std::to_string(layer) + " is not gated");
    core_->seed(keys_of(g, units, n, "ss_seed", "unit"));
  }

  void check_unit(int layer, int unit) override {
    require(!in_token_, SS_E_INVALID, "ss_check_unit: between tokens in device-gated mode");
    const int g = gated_index(layer);
    require(g >= 0, SS_E_INVALID, "ss_check_unit: layer " + std::to_string(layer) + " is not gated");
    require(unit >= 0 && uint32_t(unit) < core_->units(uint32_t(g)), SS_E_INVALID, "ss_check_unit: unit out of range");
    core_->drain();
    const uint32_t k = core_->key(uint32_t(g), uint32_t(unit));
    std::vector<char> held;
    if (live_copy(k, held)) {  // (a unit whose only copy is its file has nothing to compare)
      std::vector<char> source(held.size());
      read_unit(layer, unit, source.data());
      require(held == source, SS_E_HASH,
              "check_unit: the bytes of (" + std::to_string(layer) + ", " + std::to_string(unit) +
                  ") differ from the source");
    }
    core_->check();
  }

  // The bytes of key k's live copy into `out`: its slot while on the device (or being evicted from it), else its
  // peer store or its pinned block; false when its only copy is its file.
  bool live_copy(uint32_t k, std::vector<char>& out) {
    const SlotCache::Home home = core_->home(k);
    if (home == SlotCache::Home::File || home == SlotCache::Home::Landing || home == SlotCache::Home::Landed)
      return false;  // (only its file is a unit's own copy)
    out.resize(size_t(x_.unit_bytes));
    const int32_t slot = core_->slot_of(k);
    if (slot >= 0 && (home == SlotCache::Home::Device || home == SlotCache::Home::Evicting)) {
      for (size_t part = 0; part < x_.part_bytes.size(); ++part) {
        const char* src = bufs_.arena[part] + uint64_t(slot) * x_.part_bytes[part];
        ck(cudaMemcpy(out.data() + x_.part_offset[part], src, size_t(x_.part_bytes[part]), cudaMemcpyDeviceToHost),
           "cudaMemcpy (check)");
      }
    } else if (peer_ && peer_->owned(k)) {
      peer_->pieces(k, x_.unit_bytes, [&](const char* src, uint64_t off, uint64_t n, int32_t) {
        ck(cudaMemcpy(out.data() + off, src, size_t(n), cudaMemcpyDefault), "cudaMemcpy (check)");
      });
    } else {
      std::memcpy(out.data(), bufs_.blocks[size_t(core_->block_of(k))], out.size());
    }
    return true;
  }

  void device_view(ss_dg_device_view* v) const override {
    std::memset(v, 0, sizeof *v);
    v->struct_size = uint32_t(sizeof *v);
    v->protocol = SS_DG_PROTOCOL;
    v->n_gated = uint32_t(x_.gated.size());
    v->n_parts = uint32_t(x_.part_bytes.size());
    v->guard_slot = x_.guard_slot;
    v->slots = x_.slots;
    v->slot_of = bufs_.slot_of;
    v->unit_base = dev_.unit_base;
    v->abort = dev_.abort;
    for (size_t p = 0; p < x_.part_bytes.size(); ++p) v->parts[p] = {bufs_.arena[p], x_.part_bytes[p], x_.part_bytes[p]};
    v->absent_err = dev_.absent_err;
  }

  void enqueue_begin(void* s) override {
    require(s != nullptr, SS_E_INVALID, "ss_dg_enqueue_begin: null stream");
    ck_launch(dev::launch_dg_begin(dev_, s), "begin kernel");
  }
  void enqueue_export(int g, const int32_t* ids, int n, int n_pred, void* s) override {
    require(s && ids, SS_E_INVALID, "ss_dg_enqueue_export: null argument");
    check_g(g, "ss_dg_enqueue_export");
    require(n >= 1 && uint32_t(n) <= x_.B, SS_E_INVALID,
            "ss_dg_enqueue_export: n must be 1..dg_max_ids (" + std::to_string(x_.B) + ")");
    require(n_pred >= 0 && n_pred <= int(dev::kMaxIds), SS_E_INVALID, "ss_dg_enqueue_export: n_pred must be 0..64");
    require(n_pred == 0 || uint32_t(g) + 1 < x_.gated.size(), SS_E_INVALID,
            "ss_dg_enqueue_export: the last gated layer cannot promise a prediction");
    ck_launch(dev::launch_dg_export(dev_, uint32_t(g), ids, uint32_t(n), uint32_t(n_pred), s), "export kernel");
  }
  void enqueue_predict(int g, const int32_t* ids, int n, void* s) override {
    require(s && ids, SS_E_INVALID, "ss_dg_enqueue_predict: null argument");
    check_g(g, "ss_dg_enqueue_predict");
    require(uint32_t(g) + 1 < x_.gated.size(), SS_E_INVALID, "ss_dg_enqueue_predict: the last gated layer has no next");
    require(n >= 1 && n <= int(dev::kMaxIds), SS_E_INVALID, "ss_dg_enqueue_predict: n must be 1..64");
    ck_launch(dev::launch_dg_predict(dev_, uint32_t(g), ids, uint32_t(n), s), "predict kernel");
  }
  void enqueue_wait(int g, void* s) override {
    require(s != nullptr, SS_E_INVALID, "ss_dg_enqueue_wait: null stream");
    check_g(g, "ss_dg_enqueue_wait");
    ck_launch(dev::launch_dg_wait(dev_, uint32_t(g), s), "wait kernel");
  }
  void enqueue_end(void* s) override {
    require(s != nullptr, SS_E_INVALID, "ss_dg_enqueue_end: null stream");
    ck_launch(dev::launch_dg_end(dev_, s), "end kernel");
  }

  void keep(int g, const int32_t* ids, int n) override {
    require(!in_token_, SS_E_INVALID, "ss_dg_keep: between tokens only");
    check_g(g, "ss_dg_keep");
    keep_[size_t(g)] = keys_of(g, ids, n, "ss_dg_keep", "unit");
    held_[size_t(g)] = 0;  // a plain keep: g is exported again
    held_changed();
  }
  // ss_dg_make_resident: the units of gated layer g all on the device and kept there; g is not exported while held (the
  // engine reads its units through the table without an export); n = 0 releases it.
  void make_resident(int g, const int32_t* ids, int n) override {
    require(!in_token_, SS_E_INVALID, "ss_dg_make_resident: between tokens only");
    check_g(g, "ss_dg_make_resident");
    std::vector<uint32_t> keys = keys_of(g, ids, n, "ss_dg_make_resident", "id");
    if (keys.empty()) {  // a release
      keep_[size_t(g)].clear();
      held_[size_t(g)] = 0;
      held_changed();
      return;
    }
    std::vector<uint32_t> units(ids, ids + n);  // (checked: 0 <= id < units of g)
    core_->make_resident(uint32_t(g), units, keep_all());  // a refusal changes nothing (g keeps its former keep)
    keep_[size_t(g)] = std::move(keys);
    held_[size_t(g)] = 1;
    held_changed();
  }
  uint32_t residency(ss_dg_unit* out, uint32_t cap) override {
    require(!in_token_, SS_E_INVALID, "ss_dg_residency: between tokens only");
    const std::vector<uint32_t> keys = core_->residency();  // most recent first
    auto as_unit = [this](uint32_t k) {
      const uint32_t g = core_->gated_of(k);
      return ss_dg_unit{int32_t(g), int32_t(k - core_->key(g, 0))};
    };
    std::transform(keys.begin(), keys.begin() + std::min<size_t>(keys.size(), cap), out, as_unit);
    return uint32_t(keys.size());
  }
  void set_peer(const PeerTier& t) override {
    require(!in_token_, SS_E_INVALID, "tsb_dg_peer_retier: between tokens only");
    require(peer_ != nullptr, SS_E_INVALID,
            "tsb_dg_peer_retier: the context was opened without the peer tier (tsb_open_peer)");
    require(t.world == peer_->world && t.rank == peer_->rank, SS_E_INVALID,
            "tsb_dg_peer_retier: world and rank must stay those of the open");
    require(t.layout == peer_->layout, SS_E_INVALID, "tsb_dg_peer_retier: the store layout must stay that of the open");
    require(t.owner.size() == peer_->owner.size(), SS_E_INVALID, "tsb_dg_peer_retier: the owner map covers other keys");
    for (size_t k = 0; k < t.owner.size(); ++k)
      require((t.owner[k] >= 0) == (peer_->owner[k] >= 0), SS_E_INVALID,
              "tsb_dg_peer_retier: key " + std::to_string(k) + " would join or leave the tier (only owners change: a "
              "unit's block holds no bytes while it is owned)");
    // every copy issued so far has landed (the streams synced; the cache's own state is left as it is, so its
    // decisions stay those of an uninterrupted run): no copy reads an old store after this
    for (Mover::Stream st : {Mover::kDem, Mover::kPf, Mover::kD2h}) mover_->sync(st);
    const uint64_t stripe = peer_->stripe;  // (the same world and units: the same stripes)
    *peer_ = t;
    peer_->stripe = stripe;
  }
  void set_sched(uint32_t wb_defer, uint32_t flush_ready) override {
    require(!in_token_, SS_E_INVALID, "ss_dg_set_sched: between tokens only");
    require(wb_defer <= 1 && flush_ready <= 1, SS_E_INVALID, "ss_dg_set_sched: 0 or 1 each");
    core_->set_wb_defer(wb_defer != 0);
  }
  void set_budgets(uint32_t spare_target, uint32_t per_layer, uint32_t per_token) override {
    require(!in_token_, SS_E_INVALID, "ss_dg_set_budgets: between tokens only");
    require(spare_target <= x_.D, SS_E_INVALID,
            "ss_dg_set_budgets: spare_target above the billed spares (" + std::to_string(x_.D) + ")");
    core_->set_spare_target(spare_target);
    core_->set_prefetch_budget(per_layer, per_token);
  }
  void timeline(int g, ss_dg_layer_timeline* out) const override {
    require(!in_token_, SS_E_INVALID, "ss_dg_timeline: between tokens only");
    require(o_.dg_diag != 0, SS_E_INVALID, "ss_dg_timeline: the context was opened without dg_diag");
    check_g(g, "ss_dg_timeline");
    ss_dg_layer_timeline t{};
    t.struct_size = uint32_t(sizeof t);
    t.layer = uint32_t(x_.gated[size_t(g)]);
    t.dma_ms = t.gpu_wait_us = t.gpu_export_ready_us = t.wb_left_ms = t.dma_first_ms = -1;
    const std::vector<LayerTimes>& tt = svc_->times();
    if (timeline_valid_ && size_t(g) < tt.size()) {
      const LayerTimes& l = tt[size_t(g)];
      t.seen_us = l.seen_us;
      t.demand_us = l.demand_us;
      t.pred_wait_us = l.pred_wait_us;
      t.prefetch_us = l.prefetch_us;
      t.serve_us = l.serve_us;
      t.ids = l.ids;
      t.misses = l.misses;
      t.covered = l.covered;
      t.fetched = l.fetched;
      t.prefetched = l.prefetched;
      t.predicted_true = l.predicted_true;
      t.covered_waits = l.covered_waits;
      t.gpu_wait_us = gpu_wait_us_[size_t(g)];
      t.gpu_export_ready_us = gpu_ready_us_[size_t(g)];
      t.dma_ms = mover_->dma_ms(uint32_t(g));
    }
    std::memcpy(out, &t, sizeof t);
  }
  void boundary_timeline(ss_dg_boundary_timeline* out) const override {
    ss_dg_boundary_timeline b = boundary_;
    b.struct_size = uint32_t(sizeof b);
    std::memcpy(out, &b, sizeof b);
  }
  void stats(ss_dg_stats* out) const override {
    ss_dg_stats s{};
    s.struct_size = uint32_t(sizeof s);
    const CacheStats& c = core_->stats();
    auto d = [&](uint64_t now, uint64_t base) { return now - base; };
    s.tokens = d(c.tokens, base_.tokens);
    s.lookups = d(c.lookups, base_.lookups);
    s.misses = d(c.misses, base_.misses);
    s.covered = d(c.covered, base_.covered);
    s.fetched = d(c.fetched, base_.fetched);
    s.prefetched = d(c.prefetched, base_.prefetched);
    s.prefetch_used = d(c.prefetch_used, base_.prefetch_used);
    s.pred_invalid = d(c.pred_invalid, base_.pred_invalid);
    s.resurrected = d(c.resurrected, base_.resurrected);
    s.bank_serves = d(c.bank_serves, base_.bank_serves);
    s.collected_mid = d(c.collected_mid, base_.collected_mid);
    s.evicted = d(c.evicted, base_.evicted);
    s.evict_short = d(c.evict_short, base_.evict_short);
    s.writebacks_done = d(c.writebacks_done, base_.writebacks_done);
    s.stalled = d(c.stalled, base_.stalled);
    s.free_slots = core_->free_slots();
    s.blocks = x_.blocks;
    s.slots = x_.slots;
    s.predicted = d(c.predicted, base_.predicted);
    s.predicted_true = d(c.predicted_true, base_.predicted_true);
    s.miss_layers = d(c.miss_layers, base_.miss_layers);
    s.device_timeouts = *m_.err_count;
    s.covered_waits = d(c.covered_waits, base_.covered_waits);
    s.wb_deferred = d(c.wb_deferred, base_.wb_deferred);
    s.wb_cancelled = d(c.wb_cancelled, base_.wb_cancelled);
    s.wb_forced = d(c.wb_forced, base_.wb_forced);
    s.wb_boundary_flushed = d(c.wb_boundary_flushed, base_.wb_boundary_flushed);
    s.wb_issued_bytes = d(c.wb_issued_bytes, base_.wb_issued_bytes);
    s.wb_completed_bytes = d(c.wb_completed_bytes, base_.wb_completed_bytes);
    s.wb_cancelled_bytes = d(c.wb_cancelled_bytes, base_.wb_cancelled_bytes);
    s.wb_boundary_flushed_bytes = d(c.wb_boundary_flushed_bytes, base_.wb_boundary_flushed_bytes);
    s.wb_outstanding_bytes = core_->wb_outstanding_bytes();
    s.wb_forced_wait_ns = d(c.wb_forced_wait_ns, base_.wb_forced_wait_ns);
    s.cuda_module_loading = module_loading_;
    s.inclusive_kept = d(c.inclusive_kept, base_.inclusive_kept);
    s.inclusive_drops = d(c.inclusive_drops, base_.inclusive_drops);
    s.backed_units = core_->backed_units();
    s.disk_reads = d(c.disk_reads, base_.disk_reads);
    s.disk_read_bytes = d(c.disk_read_bytes, base_.disk_read_bytes);
    s.disk_read_ns = d(c.disk_read_ns, base_.disk_read_ns);
    s.disk_wait_ns = d(c.disk_wait_ns, base_.disk_wait_ns);
    s.disk_stage_waits = d(c.disk_stage_waits, base_.disk_stage_waits);
    s.disk_drops = d(c.disk_drops, base_.disk_drops);
    s.disk_discards = d(c.disk_discards, base_.disk_discards);
    s.disk_units = core_->file_units();
    s.disk_max_in_flight = c.disk_max_in_flight;  // (a gauge since open)
    s.disk_overlapped = d(c.disk_overlapped, base_.disk_overlapped);
    s.disk_carried = d(c.disk_carried, base_.disk_carried);
    s.disk_carried_bytes = d(c.disk_carried_bytes, base_.disk_carried_bytes);
    s.score_fallbacks = d(c.score_fallbacks, base_.score_fallbacks);
    s.scored_victims = d(c.scored_victims, base_.scored_victims);
    s.score_layers = d(c.score_layers, base_.score_layers);
    s.score_candidates = d(c.score_candidates, base_.score_candidates);
    s.score_saturated = d(c.score_saturated, base_.score_saturated);
    s.score_ns = d(c.score_ns, base_.score_ns);
    s.round_count = d(c.round_count, base_.round_count);
    s.round_units = d(c.round_units, base_.round_units);
    s.round_bytes = d(c.round_bytes, base_.round_bytes);
    s.round_ns = d(c.round_ns, base_.round_ns);
    s.round_cancelled = d(c.round_cancelled, base_.round_cancelled);
    s.resident_units = d(c.resident_units, base_.resident_units);
    s.resident_evicted = d(c.resident_evicted, base_.resident_evicted);
    s.resident_bytes = d(c.resident_bytes, base_.resident_bytes);
    s.resident_ns = d(c.resident_ns, base_.resident_ns);
    s.mkres_file_reads = d(c.mkres_file_reads, base_.mkres_file_reads);
    s.mkres_file_bytes = d(c.mkres_file_bytes, base_.mkres_file_bytes);
    s.mkres_read_ns = d(c.mkres_read_ns, base_.mkres_read_ns);
    s.mkres_h2d_bytes = d(c.mkres_h2d_bytes, base_.mkres_h2d_bytes);
    s.mkres_wb_bytes = d(c.mkres_wb_bytes, base_.mkres_wb_bytes);
    s.clean_drops = d(c.clean_drops, base_.clean_drops);
    s.clean_drop_bytes = d(c.clean_drop_bytes, base_.clean_drop_bytes);
    s.pf_reverted = d(c.pf_reverted, base_.pf_reverted);
    s.pf_revert_bytes = d(c.pf_revert_bytes, base_.pf_revert_bytes);
    s.pf_strict_refused = d(c.pf_strict_refused, base_.pf_strict_refused);
    s.bank_kept = d(c.bank_kept, base_.bank_kept);
    s.landing_issued = d(c.landing_issued, base_.landing_issued);
    s.landing_promoted = d(c.landing_promoted, base_.landing_promoted);
    s.landing_late = d(c.landing_late, base_.landing_late);
    s.landing_wait_ns = d(c.landing_wait_ns, base_.landing_wait_ns);
    s.landing_expired = d(c.landing_expired, base_.landing_expired);
    s.landing_dropped_full = d(c.landing_dropped_full, base_.landing_dropped_full);
    s.landing_read_bytes = d(c.landing_read_bytes, base_.landing_read_bytes);
    s.landing_cancelled = d(c.landing_cancelled, base_.landing_cancelled);
    s.landing_expired_layer = d(c.landing_expired_layer, base_.landing_expired_layer);
    s.landing_skipped_passed = d(c.landing_skipped_passed, base_.landing_skipped_passed);
    s.landing_yields = d(c.landing_yields, base_.landing_yields);
    s.landing_aborted_bytes = d(c.landing_aborted_bytes, base_.landing_aborted_bytes);
    s.disk_queue_resolved = x_.disk_queue;
    s.disk_depth_adapt = adapt_;  // (properties of the open's controller since open / reset_open)
    s.disk_depth_active = x_.disk_tier ? x_.disk_queue : 0;
    if (adapt_ == 1)
      async_->with_depth([&](const ReadDepth& c) {
        s.disk_depth_active = c.depth();
        s.disk_depth_changes = c.changes;
        s.disk_depth_calibrations = c.calibrations;
      });
    s.disk_locations = x_.disk_tier && o_.dg_disk_queue == 0xFFFFFFFFu ? 1u : 0u;
    std::memcpy(out, &s, sizeof s);
  }
  void layer_stats(int layer, ss_layer_stats* out) const override {
    require(layer >= 0 && size_t(layer) < d_.layers.size(), SS_E_INVALID, "ss_stats_layer: layer out of range");
    *out = ss_layer_stats{};
    const int g = gated_index(layer);
    if (g < 0) return;
    const LayerCounts& c = core_->layer_counts()[size_t(g)];
    const LayerCounts& b = lbase_[size_t(g)];
    out->routed = c.lookups - b.lookups;
    out->hits = (c.lookups - b.lookups) - (c.misses - b.misses);
    out->admitted = c.fetched - b.fetched - (c.bank_serves - b.bank_serves);
    out->transient = c.bank_serves - b.bank_serves;
    out->evicted = c.evicted - b.evicted;
    out->prefetched = c.prefetch_used - b.prefetch_used;
    out->spec_issued = c.prefetched - b.prefetched;
    out->spec_used = c.prefetch_used - b.prefetch_used;
    out->bytes_pinned = (c.fetched - b.fetched + c.prefetched - b.prefetched) * x_.unit_bytes;
  }
  void total_stats(ss_layer_stats* out) const override {
    *out = ss_layer_stats{};
    for (size_t L = 0; L < d_.layers.size(); ++L) {
      ss_layer_stats s;
      layer_stats(int(L), &s);
      out->routed += s.routed;
      out->hits += s.hits;
      out->admitted += s.admitted;
      out->transient += s.transient;
      out->evicted += s.evicted;
      out->prefetched += s.prefetched;
      out->spec_issued += s.spec_issued;
      out->spec_used += s.spec_used;
      out->bytes_pinned += s.bytes_pinned;
    }
  }
  void reset_stats() override {
    base_ = core_->stats();
    lbase_ = core_->layer_counts();
  }
  void exclusive_stats(ss_exclusive_stats* out) const override {
    ss_exclusive_stats s{};
    s.struct_size = uint32_t(sizeof s);
    const CacheStats& c = core_->stats();
    s.writebacks = c.evicted - c.wb_cancelled - c.inclusive_drops - c.disk_discards;
    s.writeback_bytes = c.wb_issued_bytes;
    s.free_blocks = core_->free_blocks();
    s.min_free_blocks = core_->free_blocks();
    std::memcpy(out, &s, sizeof s);
  }
  std::string stats_json() const override {
    ss_dg_stats s;
    stats(&s);
    char buf[8192];
    const int len = std::snprintf(buf, sizeof buf,
                  "{\"schema\":\"strix-stream/stats-v1\",\"mode\":\"device-gated\",\"copy\":\"%s\","
                  "\"dg\":{\"tokens\":%llu,\"lookups\":%llu,\"misses\":%llu,\"covered\":%llu,\"fetched\":%llu,"
                  "\"prefetched\":%llu,\"bank_serves\":%llu,\"evicted\":%llu,\"resurrected\":%llu,"
                  "\"writebacks_done\":%llu,\"wb_issued_bytes\":%llu,\"free_slots\":%llu,\"land_launches\":%llu,"
                  "\"dma_ms_total\":%.6f,\"open_seconds\":%.3f,\"disk_reads\":%llu,\"disk_read_bytes\":%llu,"
                  "\"disk_read_ns\":%llu,\"disk_drops\":%llu,\"disk_discards\":%llu,\"disk_units\":%llu,"
                  "\"bank_keep\":%u,\"bank_kept\":%llu,\"bank_keep_drops\":%llu,\"bank_keep_rereads\":%llu},"
                  "\"peer\":{\"world\":%u,\"rank\":%d,"
                  "\"all_owned\":%d,\"copy\":\"%s\",\"layout\":\"%s\",\"peer_units\":%llu,\"self_units\":%llu,"
                  "\"peer_bytes\":%llu,\"self_bytes\":%llu},"
                  "\"open\":{\"alloc_s\":%.3f,\"alloc_arena_s\":%.3f,\"alloc_pinned_s\":%.3f,\"place_s\":%.3f,"
                  "\"fill_s\":%.3f,\"fill_pinned_s\":%.3f,\"fill_residents_s\":%.3f,\"verify_s\":%.3f,"
                  "\"load\":\"%s\",\"load_readers\":%u,\"load_buffers\":%u,\"load_buffer_bytes\":%llu,"
                  "\"load_batches\":%llu,\"load_slot_units\":%llu,\"load_pinned_units\":%llu,"
                  "\"load_reader_waits\":%llu,\"load_recycles\":%llu,\"load_residents_submitted_s\":%.3f},"
                  "\"check\":{\"on\":%d,\"units\":%llu,\"bytes\":%llu,\"launches\":%llu,\"merged\":%llu,\"hold_waits\":%llu,"
                  "\"mismatches\":%llu,\"repaired\":%llu,\"end_wait_s\":%.6f}}",
                  mover_->kernel_copies() ? "land-kernel" : "copy-engine", (unsigned long long)s.tokens,
                  (unsigned long long)s.lookups, (unsigned long long)s.misses, (unsigned long long)s.covered,
                  (unsigned long long)s.fetched, (unsigned long long)s.prefetched, (unsigned long long)s.bank_serves,
                  (unsigned long long)s.evicted, (unsigned long long)s.resurrected,
                  (unsigned long long)s.writebacks_done, (unsigned long long)s.wb_issued_bytes,
                  (unsigned long long)s.free_slots, (unsigned long long)mover_->kernel_launches(),
                  mover_->dma_total_ms(), open_seconds_, (unsigned long long)s.disk_reads,
                  (unsigned long long)s.disk_read_bytes, (unsigned long long)s.disk_read_ns,
                  (unsigned long long)s.disk_drops, (unsigned long long)s.disk_discards,
                  (unsigned long long)s.disk_units, o_.dg_bank_keep, (unsigned long long)s.bank_kept,
                  (unsigned long long)(core_->stats().bank_keep_drops - base_.bank_keep_drops),
                  (unsigned long long)(core_->stats().bank_keep_rereads - base_.bank_keep_rereads),
                  peer_ ? peer_->world : 0u, peer_ ? peer_->rank : -1,
                  peer_ && peer_->all_owned ? 1 : 0, peer_ && peer_->copy == 1 ? "copy-engine" : "land-kernel",
                  peer_ && peer_->layout == kStriped ? "striped" : "whole-units",
                  (unsigned long long)mover_->peer_units(), (unsigned long long)mover_->self_units(),
                  (unsigned long long)mover_->peer_bytes(), (unsigned long long)mover_->self_bytes(), open_alloc_s_,
                  open_arena_s_, open_pinned_s_, open_cache_s_, open_fill_s_, open_fill_pinned_s_, open_fill_res_s_,
                  open_verify_s_, load_serial_ ? "serial" : "pipeline", load_readers_, load_buffers_,
                  (unsigned long long)load_buffer_bytes_, (unsigned long long)load_.batches,
                  (unsigned long long)load_.slot_units, (unsigned long long)load_.host_units,
                  (unsigned long long)load_.reader_waits, (unsigned long long)load_.recycles, load_.slot_seconds,
                  mover_->check_on() ? 1 : 0, (unsigned long long)mover_->check_stats().units,
                  (unsigned long long)mover_->check_stats().bytes, (unsigned long long)mover_->check_stats().launches,
                  (unsigned long long)mover_->check_stats().merged,
                  (unsigned long long)mover_->check_stats().hold_waits, (unsigned long long)check_failed_,
                  (unsigned long long)check_repaired_, check_wait_s_);
    require(len > 0 && size_t(len) < sizeof buf, SS_E_BACKEND, "device-gated: the stats text does not fit its buffer");
    std::string out(buf);
    out.pop_back();  // the closing brace: the read depth's and the landings' sections follow
    out += adapt_json();
    if (x_.L) {
      char b[768];
      std::snprintf(b, sizeof b,
                    ",\"landing\":{\"blocks\":%u,\"ttl\":%u,\"max_queued\":%u,\"chunk\":%u,\"issued\":%llu,"
                    "\"promoted\":%llu,\"late\":%llu,\"wait_ns\":%llu,\"expired\":%llu,\"dropped_full\":%llu,"
                    "\"read_bytes\":%llu,\"failed\":%llu,\"cancelled\":%llu,\"expired_layer\":%llu,"
                    "\"skipped_passed\":%llu,\"units\":%u}",
                    x_.L, x_.landing_ttl, x_.landing_queued, x_.landing_chunk, (unsigned long long)s.landing_issued,
                    (unsigned long long)s.landing_promoted, (unsigned long long)s.landing_late,
                    (unsigned long long)s.landing_wait_ns, (unsigned long long)s.landing_expired,
                    (unsigned long long)s.landing_dropped_full, (unsigned long long)s.landing_read_bytes,
                    (unsigned long long)(core_->stats().landing_failed - base_.landing_failed),
                    (unsigned long long)s.landing_cancelled, (unsigned long long)s.landing_expired_layer,
                    (unsigned long long)s.landing_skipped_passed, core_->landing_units());
      out += b;
    }
    out += '}';
    return out;
  }
  // ,"disk_queue_adapt":"on"|"off"|"declined: <why>" and, adapting, the controller's state and its verdict ring
  std::string adapt_json() const {
    std::string out = std::string(",\"disk_queue_adapt\":\"") +
                      (adapt_ == 1 ? "on" : adapt_ == 2 ? std::string("declined: ") + adapt_why_ : "off") + "\"";
    if (adapt_ != 1) return out;
    async_->with_depth([&](const ReadDepth& c) {
      char b[640];
      std::snprintf(b, sizeof b,
                    ",\"disk_depth\":{\"depth\":%u,\"bound\":%u,\"calibrating\":%d,\"changes\":%llu,"
                    "\"calibrations\":%llu,\"windows\":%llu,\"decisions\":%llu,\"reads_1\":%llu,\"bytes_1\":%llu,"
                    "\"busy_ns_1\":%llu,\"reads_u\":%llu,\"bytes_u\":%llu,\"busy_ns_u\":%llu,\"ring\":[",
                    c.depth(), c.bound(), c.calibrating() ? 1 : 0, (unsigned long long)c.changes,
                    (unsigned long long)c.calibrations, (unsigned long long)c.windows, (unsigned long long)c.verdicts(),
                    (unsigned long long)c.reads_1, (unsigned long long)c.bytes_1, (unsigned long long)c.ns_1,
                    (unsigned long long)c.reads_u, (unsigned long long)c.bytes_u, (unsigned long long)c.ns_u);
      out += b;
      static const char* const kWhy[] = {"start", "keep_u", "keep_1", "split", "recheck", "drift"};
      const char* sep = "";
      for (const ReadDepth::Verdict& v : c.recent()) {  // (rates in bytes / ns = GB/s)
        std::snprintf(b, sizeof b,
                      "%s{\"seq\":%llu,\"reads\":%llu,\"from\":%u,\"to\":%u,\"gbps_u\":%.6g,\"gbps_1\":%.6g,"
                      "\"reason\":\"%s\"}",
                      sep, (unsigned long long)v.seq, (unsigned long long)v.reads, v.from, v.to, v.rate_u, v.rate_1,
                      kWhy[v.why]);
        out += b;
        sep = ",";
      }
      out += "]}";
    });
    return out;
  }
  void arm_adapt() {
    if (adapt_ == 1) async_->set_depth(std::make_unique<ReadDepth>(x_.disk_queue), x_.unit_bytes);
  }
  void reset_open() override {
    require(!in_token_, SS_E_INVALID, "ss_dg_reset_open: between tokens only");
    try {
      core_->reset_open();
      for (auto& k : keep_) k.clear();
      std::fill(held_.begin(), held_.end(), uint8_t(0));
      held_changed();
      arm_adapt();  // (a fresh calibration: every read has ended)
    } catch (...) {
      poisoned_ = true;
      throw;
    }
    base_ = core_->stats();
    lbase_ = core_->layer_counts();
    timeline_valid_ = false;
  }

  void round(const RoundIn& in) override {
    require(!in_token_, SS_E_INVALID, "ss_dg_round: between tokens only");
    core_->round(in, keep_all());  // (a device failure poisons the context through the ABI's guard)
  }
  const RoundOut& last_round() const override { return core_->last_round(); }
  void round_cancel() override { core_->cancel_round(); }
  void set_clean_evict(uint32_t on) override {
    require(!in_token_, SS_E_INVALID, "ss_dg_set_clean_evict: between tokens only");
    require(on <= 1, SS_E_INVALID, "ss_dg_set_clean_evict: 0 or 1");
    core_->set_clean_evict(on != 0);
  }
  void set_pf_revert_unused(uint32_t on) override {
    require(!in_token_, SS_E_INVALID, "ss_dg_set_pf_revert_unused: between tokens only");
    require(on <= 1, SS_E_INVALID, "ss_dg_set_pf_revert_unused: 0 or 1");
    core_->set_pf_revert(on != 0);
  }
  void round_seed_counts(const ss_dg_unit* units, const float* counts, uint32_t n) override {
    require(!in_token_, SS_E_INVALID, "ss_dg_round_seed_counts: between tokens only");
    std::vector<uint32_t> keys;
    std::vector<float> v;
    for (uint32_t i = 0; i < n; ++i) {
      const int g = units[i].gated;
      require(g >= 0 && uint32_t(g) < core_->gated() && units[i].unit >= 0 &&
                  uint32_t(units[i].unit) < core_->units(uint32_t(g)),
              SS_E_INVALID, "ss_dg_round_seed_counts: unit " + std::to_string(i) + " is out of range");
      keys.push_back(core_->key(uint32_t(g), uint32_t(units[i].unit)));
      v.push_back(counts[i]);
    }
    core_->seed_round_counts(keys, v);
  }

  void set_policy(uint32_t policy) override {
    require(!in_token_, SS_E_INVALID, "ss_dg_set_policy: between tokens only");
    require(policy <= 2, SS_E_INVALID, "ss_dg_set_policy: policy must be LRU, SCORED or SCORED_AUTO");
    require(!policy || core_->scoring_ready(), SS_E_INVALID,
            "ss_dg_set_policy: scored eviction must be set up at ss_open (policy SCORED or SCORED_AUTO)");
    core_->set_policy(policy);
  }

  void test_mutate(int m) override {
    hooks("ss_test_dg_mutate");
    require(m >= 0 && m <= 2, SS_E_UNSUPPORTED, "ss_test_dg_mutate: mutation " + std::to_string(m) + " not in this build");
    core_->set_mutation(m);
  }
  void test_pressure(uint32_t f, uint32_t r) override {
    hooks("ss_test_dg_pressure");
    core_->set_pressure(f, r);
  }
  void test_check() override {
    hooks("ss_test_dg_check");
    core_->check();
  }
  void test_gate(int stream, void* event) override {
    hooks("ss_test_dg_gate");
    require(stream == 0 || stream == 1, SS_E_INVALID, "ss_test_dg_gate: stream 0 or 1");
    mover_->gate(stream == 0 ? Mover::kDem : Mover::kPf, static_cast<cudaEvent_t>(event));
  }
  void test_flags(uint32_t flags) override {
    hooks("ss_test_dg_flags");
    dev_.test_flags = flags & dev::kSkipWait;
    skip_edge_ = (flags & 2u) != 0;
  }
  uint32_t test_coming() override {
    hooks("ss_test_dg_coming");
    return core_->coming();
  }
  void test_stop_service() override {
    hooks("ss_test_dg_stop_service");
    svc_->stop_join();
  }
  void test_corrupt(int layer, int unit, uint64_t offset) override {
    hooks("tsb_test_dg_corrupt");
    require(!in_token_, SS_E_INVALID, "tsb_test_dg_corrupt: between tokens only");
    const int g = gated_index(layer);
    require(g >= 0 && unit >= 0 && uint32_t(unit) < core_->units(uint32_t(g)), SS_E_INVALID,
            "tsb_test_dg_corrupt: not a gated unit");
    const uint32_t k = core_->key(uint32_t(g), uint32_t(unit));
    require(core_->home(k) == SlotCache::Home::Host && core_->block_of(k) >= 0 && !(peer_ && peer_->owned(k)),
            SS_E_INVALID, "tsb_test_dg_corrupt: the unit is not in a pinned block");
    require(offset < x_.unit_bytes, SS_E_INVALID, "tsb_test_dg_corrupt: offset beyond the unit");
    bufs_.blocks[size_t(core_->block_of(k))][offset] ^= char(0x5a);
  }
  uint32_t test_table(int32_t* out, uint32_t cap) override {
    hooks("tsb_test_dg_table");
    require(!in_token_, SS_E_INVALID, "tsb_test_dg_table: between tokens only");
    require(out && cap >= x_.keys, SS_E_INVALID, "tsb_test_dg_table: the output holds fewer entries than the keys");
    ck(cudaMemcpy(out, bufs_.slot_of, size_t(x_.keys) * 4, cudaMemcpyDeviceToHost), "cudaMemcpy (table)");
    return x_.keys;
  }

 private:
  void hooks(const char* fn) const {
    require(o_.dg_test_hooks != 0, SS_E_INVALID, std::string(fn) + ": the context was opened without dg_test_hooks");
  }
  void check_g(int g, const char* fn) const {
    require(g >= 0 && size_t(g) < x_.gated.size(), SS_E_INVALID, std::string(fn) + ": gated layer out of range");
  }
  // A layer held or released: table uploads write only changed entries while any layer is held.
  void held_changed() {
    core_->set_range_uploads(std::any_of(held_.begin(), held_.end(), [](uint8_t h) { return h != 0; }));
  }
  // The keys of units `ids[0..n)` of gated layer g, each checked (`fn`: the entry point; `what`: "unit" or "id").
  std::vector<uint32_t> keys_of(int g, const int32_t* ids, int n, const char* fn, const char* what) const {
    require(n >= 0 && (n == 0 || ids), SS_E_INVALID, std::string(fn) + ": bad arguments");
    const uint32_t limit = core_->units(uint32_t(g));
    std::vector<uint32_t> keys(static_cast<size_t>(n));
    for (int i = 0; i < n; ++i) {
      require(ids[i] >= 0 && uint32_t(ids[i]) < limit, SS_E_INVALID, std::string(fn) + ": " + what + " out of range");
      keys[size_t(i)] = core_->key(uint32_t(g), uint32_t(ids[i]));
    }
    return keys;
  }
  std::vector<uint32_t> keep_all() const {
    std::vector<uint32_t> all;
    for (const auto& k : keep_) all.insert(all.end(), k.begin(), k.end());
    return all;
  }
  std::string device_error() const {
    static const char* names[] = {"", "a wait timed out", "an exported id is out of range", "the host aborted the token",
                                  "sequence desync (a step the host did not open)", "a lookup met an absent entry"};
    const uint32_t code = load_acquire(m_.err_code), aux = load_acquire(m_.err_aux);
    if (!code) return "";
    return std::string("device: ") + (code < 6 ? names[code] : "unknown error") + " (gated layer / seq " +
           std::to_string(aux) + ")";
  }
  std::string token_failure(const std::string& dev, const std::string& host) const {
    std::string s = "device-gated: token " + std::to_string(seq_) + " failed: ";
    if (!dev.empty()) s += dev + (host.empty() ? "" : "; ");
    return s + host + " (the token's outputs must be discarded; the context is poisoned)";
  }
  void collect_diag() {
    mover_->diag_collect();
    const uint32_t G = uint32_t(x_.gated.size());
    for (uint32_t g = 0; g < G; ++g) {
      const volatile unsigned long long* t = stamps_h_ + 4u * g;
      const unsigned long long ex = t[0], in = t[1], rd = t[2];
      const bool ok = ex && in && rd && rd >= in && rd >= ex;
      gpu_wait_us_[g] = ok ? double(rd - in) / 1000.0 : -1;
      gpu_ready_us_[g] = ok ? double(rd - ex) / 1000.0 : -1;
    }
  }
  char* unit_part_dst(int32_t slot, uint32_t p) const { return bufs_.arena[p] + uint64_t(slot) * x_.part_bytes[p]; }
  // A gated unit's engine bytes from its source file into dst (parts back to back).
  void read_unit(int layer, int unit, char* dst) const {
    const Layer& l = d_.layers[size_t(layer)];
    uint64_t off = 0;
    for (const Part& p : l.parts) {
      files_[size_t(p.source)]->read(dst + off, p.offset + uint64_t(unit) * p.stride, p.bytes);
      off += p.bytes;
    }
  }
  // A file-tier read: the unit's parts in pieces of at most 8 MiB, read by the reader pool at once (the reference
  // reads a unit in one pass on one reader); with verify_hash and descriptor hashes, the bytes are checked on the host
  // before any copy reads them (the reference's read_checked, dg_ctx.cpp:1625-1633).
  void read_checked(int layer, int unit, char* dst, ReadPool* pool) const {
    const Layer& l = d_.layers[size_t(layer)];
    struct Piece {
      const SourceFile* f;
      uint64_t off, bytes;
      char* dst;
    };
    std::vector<Piece> pieces;
    uint64_t at = 0;
    for (const Part& p : l.parts) {
      const uint64_t base = p.offset + uint64_t(unit) * p.stride;
      for (uint64_t o = 0; o < p.bytes; o += kReadPiece)
        pieces.push_back({files_[size_t(p.source)].get(), base + o, std::min(kReadPiece, p.bytes - o), dst + at + o});
      at += p.bytes;
    }
    const bool check = o_.verify_hash && !l.hash.empty();
    Xxh64State h(0);
    size_t hashed = 0;  // pieces fed to the hash, in unit order
    if (pool) {
      // the hash runs while later pieces are still being read: a reader that finishes a piece advances it over the
      // finished prefix unless another reader is already doing so; what is left is fed below
      std::unique_ptr<std::atomic<uint8_t>[]> done(new std::atomic<uint8_t>[pieces.size()]());
      std::mutex hashing;
      pool->run(pieces.size(), [&](size_t i) {
        pieces[i].f->read(pieces[i].dst, pieces[i].off, pieces[i].bytes);
        done[i].store(1, std::memory_order_release);
        if (!check) return;
        std::unique_lock<std::mutex> lk(hashing, std::try_to_lock);
        if (!lk.owns_lock()) return;
        while (hashed < pieces.size() && done[hashed].load(std::memory_order_acquire)) {
          h.feed(pieces[hashed].dst, size_t(pieces[hashed].bytes));
          ++hashed;
        }
      });
    } else {
      for (const Piece& q : pieces) q.f->read(q.dst, q.off, q.bytes);
    }
    if (!check) return;
    for (; hashed < pieces.size(); ++hashed) h.feed(pieces[hashed].dst, size_t(pieces[hashed].bytes));
    require(h.digest() == l.hash[size_t(unit)], SS_E_HASH,
            "device-gated: unit (" + std::to_string(layer) + ", " + std::to_string(unit) +
                ") bytes differ from the descriptor hash");
  }

  void init() {
    auto t_start = Clock::now();
    device_ = o_.device;
    ck(cudaSetDevice(device_), "cudaSetDevice");
    ck_launch(dev::preload(), "loading the kernels");
    CUmoduleLoadingMode mode{};
    if (driver().loading_mode && driver().loading_mode(&mode) == CUDA_SUCCESS)
      module_loading_ = mode == CU_MODULE_EAGER_LOADING ? 1u : mode == CU_MODULE_LAZY_LOADING ? 2u : 0u;
    for (const Source& s : d_.sources) files_.push_back(std::make_unique<SourceFile>(s.path, s.align, o_.direct_io != 0));
    const uint32_t G = uint32_t(x_.gated.size());
    // HBM: the arena (guard slot zeroed), the table, the control words
    for (uint64_t pb : x_.part_bytes) {
      void* a = nullptr;
      ck(cudaMalloc(&a, size_t(uint64_t(x_.slots) * pb)), "cudaMalloc (arena)");
      bufs_.arena.push_back(static_cast<char*>(a));
      ck(cudaMemset(static_cast<char*>(a) + uint64_t(x_.guard_slot) * pb, 0, size_t(pb)), "cudaMemset (guard slot)");
    }
    const auto t_arena = Clock::now();
    ck(cudaMalloc(reinterpret_cast<void**>(&bufs_.slot_of), size_t(x_.keys) * 4), "cudaMalloc (slot table)");
    const size_t ctl_words = 8 + 2 * size_t(G) + (G + 1) + 4;
    ck(cudaMalloc(reinterpret_cast<void**>(&ctl_), ctl_words * 4), "cudaMalloc (controls)");
    ck(cudaMemset(ctl_, 0, ctl_words * 4), "cudaMemset (controls)");
    dev_ = dev::DgDev{};
    dev_.seq = ctl_;
    dev_.abort = ctl_ + 1;
    dev_.err_count = ctl_ + 2;
    dev_.err_code = ctl_ + 3;
    dev_.err_aux = ctl_ + 4;
    dev_.absent_err = ctl_ + 5;
    bufs_.counters = ctl_ + 8;  // 3 words (one per copy stream)
    dev_.any_miss = ctl_ + 12;
    dev_.ready = ctl_ + 12 + G;
    bufs_.ready = dev_.ready;
    uint32_t* ub = ctl_ + 12 + 2 * G;
    ck(cudaMemcpy(ub, x_.unit_base.data(), size_t(G + 1) * 4, cudaMemcpyHostToDevice), "cudaMemcpy (unit_base)");
    dev_.unit_base = ub;
    dev_.slot_of = bufs_.slot_of;
    dev_.timeout_ns = uint64_t(o_.dg_wait_timeout_ms) * 1000000ull;
    // the mapped control area, 64-byte aligned pieces
    const size_t rec_b = size_t(G) * sizeof(dev::DgRecord), prec_b = size_t(G) * sizeof(dev::DgPredRecord);
    auto r64 = [](size_t n) { return (n + 63) / 64 * 64; };
    // the landing check's flag, log and launch done words
    const size_t check_b = (1 + 2 * size_t(dev::kBadLog) + CudaMover::kCheckRing) * 4;
    const size_t mapped_bytes = r64(rec_b) + r64(prec_b) + 2 * r64(size_t(G) * 4) + 64 + r64(check_b);
    ck(cudaHostAlloc(&mapped_h_, mapped_bytes, cudaHostAllocMapped | cudaHostAllocPortable), "cudaHostAlloc (mapped)");
    std::memset(mapped_h_, 0, mapped_bytes);
    void* md = nullptr;
    ck(cudaHostGetDevicePointer(&md, mapped_h_, 0), "cudaHostGetDevicePointer");
    size_t off = 0;
    auto carve = [&](size_t bytes, auto** host, auto** devp) {
      using T = std::remove_pointer_t<std::remove_reference_t<decltype(*host)>>;
      *host = reinterpret_cast<T*>(static_cast<char*>(mapped_h_) + off);
      *devp = reinterpret_cast<T*>(static_cast<char*>(md) + off);
      off += r64(bytes);
    };
    carve(rec_b, &m_.rec, &dev_.rec);
    carve(prec_b, &m_.prec, &dev_.prec);
    carve(size_t(G) * 4, &m_.flag, &dev_.flag);
    carve(size_t(G) * 4, &m_.pflag, &dev_.pflag);
    {  // single control words, each seen by the host (m_) and the device (dev_) at its two addresses
      uint32_t** host_side[] = {&m_.done, &m_.err_code, &m_.err_aux, &m_.host_abort, &m_.host_seq, &m_.began,
                                &m_.err_count};
      uint32_t** device_side[] = {&dev_.done, &dev_.m_err_code, &dev_.m_err_aux, &dev_.host_abort, &dev_.host_seq,
                                  &dev_.began, &dev_.m_err_count};
      constexpr size_t kWords = sizeof host_side / sizeof host_side[0];
      static_assert(kWords == sizeof device_side / sizeof device_side[0], "one device address per host word");
      uint32_t *words_h = nullptr, *words_d = nullptr;
      carve(kWords * 4, &words_h, &words_d);
      for (size_t w = 0; w < kWords; ++w) {
        *host_side[w] = words_h + w;
        *device_side[w] = words_d + w;
      }
    }
    uint32_t *chk_h = nullptr, *chk_d = nullptr;
    carve(check_b, &chk_h, &chk_d);
    bad_flag_h_ = chk_h;
    bad_log_h_ = chk_h + 1;
    if (o_.dg_diag) {
      void* h = nullptr;
      ck(cudaHostAlloc(&h, size_t(G) * 32, cudaHostAllocMapped | cudaHostAllocPortable), "cudaHostAlloc (stamps)");
      std::memset(h, 0, size_t(G) * 32);
      stamps_h_ = static_cast<unsigned long long*>(h);
      void* dd = nullptr;
      ck(cudaHostGetDevicePointer(&dd, h, 0), "cudaHostGetDevicePointer (stamps)");
      dev_.stamps = static_cast<unsigned long long*>(dd);
    }
    gpu_wait_us_.assign(G, -1);
    gpu_ready_us_.assign(G, -1);
    // pinned blocks (mapped: the land kernel reads them) in <= 1 GiB chunks (pinned.cu: mapped, populated by a pool of
    // threads with huge pages, registered), the file tier's staging buffers after them (block indices blocks ..);
    // the reset staging unit
    const uint64_t hs = x_.host_stride;
    const uint64_t per_chunk = std::max<uint64_t>(1, (uint64_t(1) << 30) / hs);
    std::vector<uint64_t> chunk_units;
    std::vector<size_t> chunk_bytes;
    for (uint64_t left = peer_ && peer_->all_owned ? 0 : uint64_t(x_.blocks) + x_.S + x_.L; left > 0;) {
      chunk_units.push_back(std::min(per_chunk, left));
      chunk_bytes.push_back(size_t(chunk_units.back() * hs));
      left -= chunk_units.back();
    }
    const auto t_pinned0 = Clock::now();
    pinned_ = alloc_pinned(chunk_bytes, device_);
    open_pinned_s_ = std::chrono::duration<double>(Clock::now() - t_pinned0).count();
    open_arena_s_ = std::chrono::duration<double>(t_arena - t_start).count();
    for (const PinnedChunk& c : pinned_) chunks_.push_back(c.ptr);
    for (size_t c = 0; c < chunks_.size(); ++c) {
      void* pd = nullptr;
      ck(cudaHostGetDevicePointer(&pd, chunks_[c], 0), "cudaHostGetDevicePointer (blocks)");
      for (uint64_t i = 0; i < chunk_units[c]; ++i) {
        bufs_.blocks.push_back(static_cast<char*>(chunks_[c]) + i * hs);
        bufs_.blocks_d.push_back(static_cast<char*>(pd) + i * hs);
      }
    }
    ck(cudaHostAlloc(reinterpret_cast<void**>(&bufs_.staging), size_t(hs), cudaHostAllocMapped | cudaHostAllocPortable),
       "cudaHostAlloc (staging)");
    void* sd = nullptr;
    ck(cudaHostGetDevicePointer(&sd, bufs_.staging, 0), "cudaHostGetDevicePointer (staging)");
    bufs_.staging_d = static_cast<char*>(sd);
    // the cache: residents in slots 0.., every other unit in a block
    mover_ = std::make_unique<CudaMover>(x_, bufs_, peer_.get());
    if (o_.dg_diag) mover_->enable_diag(G);
    // the landing check: with verify_hash and a hash for every gated unit, every unit landed in a slot is hashed on the
    // device and compared with its descriptor hash (ss_end reports a mismatch)
    bool hashed = o_.verify_hash != 0;
    for (int L : x_.gated) hashed = hashed && !d_.layers[size_t(L)].hash.empty();
    if (hashed) {
      std::vector<uint64_t> expect;
      expect.reserve(x_.keys);
      for (int L : x_.gated)
        expect.insert(expect.end(), d_.layers[size_t(L)].hash.begin(), d_.layers[size_t(L)].hash.end());
      ck(cudaMalloc(reinterpret_cast<void**>(&expect_dev_), expect.size() * 8), "cudaMalloc (descriptor hashes)");
      ck(cudaMemcpy(expect_dev_, expect.data(), expect.size() * 8, cudaMemcpyHostToDevice),
         "cudaMemcpy (descriptor hashes)");
      ck(cudaMalloc(reinterpret_cast<void**>(&done_cnt_), CudaMover::kCheckRing * 4), "cudaMalloc (landing check)");
      ck(cudaMemset(done_cnt_, 0, CudaMover::kCheckRing * 4), "cudaMemset (landing check)");
      CudaMover::CheckWords w{};
      w.expect = expect_dev_;
      w.bad_count = ctl_ + 6;
      w.timeouts = ctl_ + 7;
      w.bad_flag = chk_d;
      w.bad_log = chk_d + 1;
      w.done_cnt = done_cnt_;
      w.done_dev = chk_d + 1 + 2 * dev::kBadLog;
      w.done_host = bad_flag_h_ + 1 + 2 * dev::kBadLog;
      mover_->enable_check(w);
    }
    CacheConfig c;
    for (int L : x_.gated) c.n_units.push_back(uint32_t(d_.layers[size_t(L)].n_units));
    c.persistent_slots = x_.persistent_slots;
    c.bank_slots = x_.B;
    c.blocks = x_.blocks;
    const uint32_t T = o_.dg_spare_target == 0xFFFFFFFFu ? x_.D : o_.dg_spare_target;
    require(T <= x_.D, SS_E_INVALID,
            "device-gated: dg_spare_target " + std::to_string(T) + " above the billed spares (" + std::to_string(x_.D) + ")");
    c.spare_target = T;
    c.prefetch_reserve_auto = o_.dg_prefetch_reserve == 0xFFFFFFFFu;
    c.prefetch_reserve = c.prefetch_reserve_auto ? std::min<uint32_t>(24, T / 4) : o_.dg_prefetch_reserve;
    c.prefetch_per_layer = o_.dg_prefetch_per_layer;
    c.prefetch_per_token = o_.dg_prefetch_per_token;
    c.wb_defer = o_.dg_wb_defer != 0;
    c.wb_on_d2h = o_.dg_wb_stream == 1;
    c.wb_layer_bytes = o_.dg_wb_layer_bytes;
    c.wb_max_outstanding = o_.dg_wb_max_outstanding;
    c.inclusive = x_.I;
    c.disk_tier = x_.disk_tier;
    c.disk_prefetch = x_.disk_prefetch;
    c.home_blocks = x_.disk_tier ? x_.P : 0;  // the plan's pinned units get the blocks; the rest are spares
    c.disk_staging = x_.S;
    c.disk_queue = std::max<uint32_t>(1, x_.disk_queue);
    c.scored = x_.scored;
    c.scored_auto = x_.scored_auto;
    c.w_trans = x_.w_trans;
    c.w_freq = x_.w_freq;
    c.w_rec = x_.w_rec;
    c.max_ids = x_.B;
    c.no_admit = o_.dg_no_admit != 0;  // (the banks hold dg_max_ids each: the layout checked the ring)
    c.clean_evict = o_.dg_clean_evict != 0;  // (no effect without the file tier)
    c.pf_revert = o_.dg_pf_revert_unused != 0;
    c.pf_strict = o_.dg_pf_strict_admit != 0;
    c.bank_keep = o_.dg_bank_keep;  // (0..2; no effect without the file tier or with dg_no_admit)
    c.landing_blocks = x_.L;        // (after the staging buffers: block indices blocks + S ..)
    c.landing_ttl = x_.landing_ttl;
    if (x_.disk_tier) {  // a file miss: the unit's parts from their files, checked against the descriptor's hash
      unsigned n = 8;
      if (const char* e = std::getenv("TSB_FILE_READERS")) n = unsigned(std::max(1L, std::min(64L, std::atol(e))));
      readers_ = std::make_unique<ReadPool>(n);
      mover_->set_reader([this](uint32_t key, char* dst) {
        const uint32_t g = uint32_t(std::upper_bound(x_.unit_base.begin(), x_.unit_base.end(), key) -
                                    x_.unit_base.begin()) - 1;
        read_checked(x_.gated[g], int(key - x_.unit_base[g]), dst, readers_.get());
      });
      if (x_.disk_queue > 1) {  // reads in flight: one reader thread per read the queue holds, each read's pieces
        // spread over a pool of that thread's own (a miss read in flight is as fast as a synchronous one)
        for (uint32_t i = 0; i < x_.disk_queue; ++i) flight_pools_.push_back(std::make_unique<ReadPool>(n));
        async_ = std::make_unique<AsyncReads>(x_.disk_queue, [this](uint32_t key, char* dst, unsigned worker) {
          const uint32_t g = uint32_t(std::upper_bound(x_.unit_base.begin(), x_.unit_base.end(), key) -
                                      x_.unit_base.begin()) - 1;
          read_checked(x_.gated[g], int(key - x_.unit_base[g]), dst, flight_pools_[worker].get());
        });
        mover_->set_async(async_.get());
        async_->set_landing(x_.landing_queued, x_.landing_chunk != 0);
      }
      // dg_disk_queue_adapt: the pool's demand reads at a measured depth (1 or the resolved queue); declined where
      // the pool is not demand-only over several readers
      if (o_.dg_disk_queue_adapt) {
        adapt_ = 2;
        if (!async_) adapt_why_ = "one reader";
        else if (x_.L) adapt_why_ = "landing blocks";
        else if (o_.dg_disk_prefetch) adapt_why_ = "file prefetches";
        else adapt_ = 1;
      }
      arm_adapt();
    }
    core_ = std::make_unique<SlotCache>(c, mover_.get());
    std::vector<uint32_t> order;
    if (o_.dg_seed_n) {
      require(o_.dg_seed != nullptr, SS_E_INVALID, "device-gated: dg_seed_n > 0 with a null dg_seed");
      for (uint32_t i = 0; i < o_.dg_seed_n; ++i) {
        const ss_dg_unit& e = o_.dg_seed[i];
        require(e.gated >= 0 && uint32_t(e.gated) < G && e.unit >= 0 && uint32_t(e.unit) < core_->units(uint32_t(e.gated)),
                SS_E_INVALID, "device-gated: dg_seed entry " + std::to_string(i) + " is out of range");
        order.push_back(core_->key(uint32_t(e.gated), uint32_t(e.unit)));
      }
    }
    o_.dg_seed = nullptr;
    o_.dg_seed_n = 0;
    order.insert(order.end(), x_.residents.begin(), x_.residents.end());
    for (uint32_t k = 0; k < x_.keys; ++k) order.push_back(k);
    const auto t_place = Clock::now();
    core_->place(order, x_.disk_tier ? &x_.disk : nullptr);
    if (!x_.profile.empty()) core_->load_counts(x_.profile);
    open_alloc_s_ = std::chrono::duration<double>(Clock::now() - t_start).count();
    open_cache_s_ = std::chrono::duration<double>(Clock::now() - t_place).count();
    fill();
    mover_->upload_table(core_->table().data(), x_.keys);
    core_->check();
    keep_.assign(G, {});
    held_.assign(G, 0);
    run_.assign(G, 1);
    lbase_.assign(G, LayerCounts{});
    svc_ = std::make_unique<Service>(core_.get(), m_, x_.B, o_.dg_wait_timeout_ms, device_, mover_->deterministic(),
                                     o_.dg_diag != 0);
    svc_->start();
    open_seconds_ = std::chrono::duration<double>(Clock::now() - t_start).count();
  }

  // The open's fill: every unit's bytes from its file into its slot or block; with verify_hash and descriptor hashes,
  // pinned units are hashed on the host as they are read and residents on the device (one K3 launch over every
  // resident slot) before the first token. By default a pipeline (loader.hpp): reader threads read the residents into
  // a ring of pinned buffers, whose copies this thread enqueues as each buffer is full, and the pinned units in place
  // in between, so the reads, the host link and the pinned units' reads overlap (the reference's startup loader,
  // src/dg_ctx.cpp:1953-2016). TSB_LOAD_SERIAL=1 selects the phased order instead (pinned units, then residents in
  // rounds of reads and copies; the reference's DG_LOAD_SERIAL); TSB_LOAD_READERS (1-32, default 8), TSB_LOAD_BUFFERS
  // (1-16, default 4) and TSB_LOAD_BUFFER_MIB (1-1024, default 64, at least one unit) size the pipeline.
  void fill() {
    const auto t_fill = Clock::now();
    const uint32_t G = uint32_t(x_.gated.size());
    std::vector<std::pair<uint32_t, uint32_t>> res, pin, from_store;  // (g, unit)
    std::vector<LoadUnit> units;  // every resident and pinned unit read from its file, in key order
    for (uint32_t g = 0; g < G; ++g)
      for (uint32_t u = 0; u < core_->units(g); ++u) {
        const uint32_t k = core_->key(g, u);
        const bool owned = peer_ && peer_->owned(k);  // an owned unit's block is never read: not filled
        if (core_->slot_of(k) >= 0) {
          (owned ? from_store : res).push_back({g, u});
          if (!owned) units.push_back(LoadUnit{x_.gated[g], int(u), core_->slot_of(k), nullptr});
        } else if (!owned && core_->block_of(k) >= 0) {  // (a file home stays in its file)
          pin.push_back({g, u});
          units.push_back(LoadUnit{x_.gated[g], int(u), -1, bufs_.blocks[size_t(core_->block_of(k))]});
        }
      }
    const bool serial = std::getenv("TSB_LOAD_SERIAL") && std::atoi(std::getenv("TSB_LOAD_SERIAL")) != 0;
    if (serial) fill_serial(res, pin);
    else fill_pipeline(units, res.size());
    load_serial_ = serial;
    cudaStream_t fs = mover_->stream(Mover::kDem);
    // owned residents from their stores (the stores were checked against the hashes when they were filled)
    for (const auto& [g, u] : from_store) {
      const uint32_t k = core_->key(g, u);
      peer_->pieces(k, x_.unit_bytes, [&](const char* src, uint64_t off, uint64_t n, int32_t) {
        for (size_t p = 0; p < x_.part_bytes.size(); ++p) {
          const uint64_t a = std::max(off, x_.part_offset[p]);
          const uint64_t b = std::min(off + n, x_.part_offset[p] + x_.part_bytes[p]);
          if (a < b)
            ck(cudaMemcpyAsync(unit_part_dst(core_->slot_of(k), uint32_t(p)) + (a - x_.part_offset[p]), src + (a - off),
                               size_t(b - a), cudaMemcpyDefault, fs),
               "cudaMemcpyAsync (fill from store)");
        }
      });
    }
    ck(cudaStreamSynchronize(fs), "cudaStreamSynchronize (fill from store)");
    res.insert(res.end(), from_store.begin(), from_store.end());
    const auto t_res = Clock::now();
    if (o_.verify_hash && !res.empty() && !d_.layers[size_t(x_.gated[0])].hash.empty()) verify_residents(res);
    open_fill_s_ = std::chrono::duration<double>(t_res - t_fill).count();
    open_verify_s_ = std::chrono::duration<double>(Clock::now() - t_res).count();
  }

  // One environment count in [lo, hi], else the default (a value out of range is refused).
  static unsigned env_count(const char* name, unsigned def, unsigned lo, unsigned hi) {
    const char* e = std::getenv(name);
    if (!e || !*e) return def;
    char* end = nullptr;
    const long v = std::strtol(e, &end, 10);
    require(end && *end == 0 && v >= long(lo) && v <= long(hi), SS_E_INVALID,
            std::string("device-gated: invalid ") + name + " (" + std::to_string(lo) + "-" + std::to_string(hi) + ")");
    return unsigned(v);
  }

  void fill_pipeline(const std::vector<LoadUnit>& units, size_t n_res) {
    const uint64_t hs = x_.host_stride;
    const unsigned readers = env_count("TSB_LOAD_READERS", 8, 1, 32);
    unsigned nbuf = env_count("TSB_LOAD_BUFFERS", 4, 1, 16);
    const uint64_t target = uint64_t(env_count("TSB_LOAD_BUFFER_MIB", 64, 1, 1024)) << 20;
    // a buffer holds whole units (at least one), never more than the residents need
    const uint64_t per = std::max<uint64_t>(1, std::min<uint64_t>(target / hs, std::max<size_t>(n_res, 1)));
    const uint64_t batches = (uint64_t(n_res) + per - 1) / per;
    nbuf = unsigned(std::min<uint64_t>(nbuf, batches));
    struct Ring {
      std::vector<char*> buf;
      std::vector<cudaEvent_t> ev;
      cudaStream_t s = nullptr;
      ~Ring() {
        if (s) (void)cudaStreamSynchronize(s);  // (an error path: no copy may read a buffer being freed)
        for (char* b : buf) (void)cudaFreeHost(b);
        for (cudaEvent_t e : ev) (void)cudaEventDestroy(e);
      }
    } ring;
    ring.s = mover_->stream(Mover::kDem);
    for (unsigned b = 0; b < nbuf; ++b) {
      char* p = nullptr;
      ck(cudaHostAlloc(reinterpret_cast<void**>(&p), size_t(per * hs), cudaHostAllocPortable), "cudaHostAlloc (load ring)");
      ring.buf.push_back(p);
      cudaEvent_t e = nullptr;
      ck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate (load ring)");
      ring.ev.push_back(e);
    }
    const bool verify = o_.verify_hash != 0;
    const LoadStats st = run_load(
        units, ring.buf, per * hs, hs, readers,
        [&](const LoadUnit& lu, char* dst) {  // a reader thread: file reads and hashes only
          read_unit(lu.layer, lu.unit, dst);
          const Layer& l = d_.layers[size_t(lu.layer)];
          if (lu.slot < 0 && verify && !l.hash.empty())
            require(xxh64(dst, size_t(x_.unit_bytes)) == l.hash[size_t(lu.unit)], SS_E_HASH,
                    "device-gated: unit (" + std::to_string(lu.layer) + ", " + std::to_string(lu.unit) +
                        ") differs from its descriptor hash");
        },
        [&](size_t b, const std::vector<LoadCopy>& copies) {  // this thread: the batch's copies, then its event
          for (const LoadCopy& c : copies)
            for (size_t p = 0; p < x_.part_bytes.size(); ++p)
              ck(cudaMemcpyAsync(unit_part_dst(c.slot, uint32_t(p)), c.data + x_.part_offset[p],
                                 size_t(x_.part_bytes[p]), cudaMemcpyHostToDevice, ring.s),
                 "cudaMemcpyAsync (load)");
          ck(cudaEventRecord(ring.ev[b], ring.s), "cudaEventRecord (load ring)");
        },
        [&](size_t b) { ck(cudaEventSynchronize(ring.ev[b]), "cudaEventSynchronize (load ring)"); });
    ck(cudaStreamSynchronize(ring.s), "cudaStreamSynchronize (load)");
    load_ = st;
    load_readers_ = readers;
    load_buffers_ = nbuf;
    load_buffer_bytes_ = per * hs;
  }

  // The phased fill: the pinned units by a pool of reader threads, then the residents through a ring of pinned staging
  // units, read a ringful at a time and copied before the next round of reads.
  void fill_serial(const std::vector<std::pair<uint32_t, uint32_t>>& res,
                   const std::vector<std::pair<uint32_t, uint32_t>>& pin) {
    const auto t_fill = Clock::now();
    const bool verify = o_.verify_hash != 0;
    unsigned nthreads = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    std::atomic<size_t> next{0};
    std::mutex err_mu;
    std::exception_ptr err;  // the first failure, with its status (SS_E_IO, SS_E_HASH)
    auto worker = [&](auto&& job, size_t n) {
      for (;;) {
        const size_t i = next.fetch_add(1);
        if (i >= n) return;
        try {
          job(i);
        } catch (...) {
          std::lock_guard<std::mutex> lk(err_mu);
          if (!err) err = std::current_exception();
        }
      }
    };
    auto run_pool = [&](auto&& job, size_t n) {
      next = 0;
      std::vector<std::thread> th;
      for (unsigned t = 0; t < nthreads; ++t) th.emplace_back([&] { worker(job, n); });
      for (auto& t : th) t.join();
      if (err) std::rethrow_exception(err);
    };
    auto hash_of = [&](uint32_t g, uint32_t u) -> const uint64_t* {
      const Layer& l = d_.layers[size_t(x_.gated[g])];
      return l.hash.empty() ? nullptr : &l.hash[u];
    };
    run_pool(
        [&](size_t i) {
          const auto [g, u] = pin[i];
          char* dst = bufs_.blocks[size_t(core_->block_of(core_->key(g, u)))];
          read_unit(x_.gated[g], int(u), dst);
          if (verify)
            if (const uint64_t* h = hash_of(g, u))
              require(xxh64(dst, size_t(x_.unit_bytes)) == *h, SS_E_HASH,
                      "device-gated: unit (" + std::to_string(x_.gated[g]) + ", " + std::to_string(u) +
                          ") differs from its descriptor hash");
        },
        pin.size());
    const auto t_pinned = Clock::now();
    // residents: through a ring of pinned staging units, nthreads at a time
    const size_t ring = std::min<size_t>(std::max<size_t>(res.size(), 1), nthreads);
    std::vector<char*> stage(ring, nullptr);
    for (auto& s : stage)
      ck(cudaHostAlloc(reinterpret_cast<void**>(&s), size_t(x_.host_stride), cudaHostAllocPortable), "cudaHostAlloc (fill)");
    cudaStream_t fs = mover_->stream(Mover::kDem);
    try {
      for (size_t first = 0; first < res.size(); first += ring) {
        const size_t n = std::min(ring, res.size() - first);
        run_pool([&](size_t i) { read_unit(x_.gated[res[first + i].first], int(res[first + i].second), stage[i]); }, n);
        for (size_t i = 0; i < n; ++i) {
          const int32_t slot = core_->slot_of(core_->key(res[first + i].first, res[first + i].second));
          for (size_t p = 0; p < x_.part_bytes.size(); ++p)
            ck(cudaMemcpyAsync(unit_part_dst(slot, uint32_t(p)), stage[i] + x_.part_offset[p], size_t(x_.part_bytes[p]),
                               cudaMemcpyHostToDevice, fs),
               "cudaMemcpyAsync (fill)");
        }
        ck(cudaStreamSynchronize(fs), "cudaStreamSynchronize (fill)");
      }
    } catch (...) {
      for (char* s : stage) cudaFreeHost(s);
      throw;
    }
    for (char* s : stage) cudaFreeHost(s);
    open_fill_pinned_s_ = std::chrono::duration<double>(t_pinned - t_fill).count();
    open_fill_res_s_ = std::chrono::duration<double>(Clock::now() - t_pinned).count();
  }

  // K3 over every resident slot at once: the arena's bytes against the descriptor's hashes.
  void verify_residents(const std::vector<std::pair<uint32_t, uint32_t>>& res) {
    const size_t n = res.size();
    std::vector<dev::HashUnit> units(n);
    std::vector<uint64_t> expect(n);
    for (size_t i = 0; i < n; ++i) {
      const int32_t slot = core_->slot_of(core_->key(res[i].first, res[i].second));
      dev::HashUnit& h = units[i];
      h = dev::HashUnit{};
      h.n_spans = uint32_t(x_.part_bytes.size());
      for (uint32_t p = 0; p < h.n_spans; ++p) {
        h.span[p] = reinterpret_cast<const uint8_t*>(unit_part_dst(slot, p));
        h.bytes[p] = x_.part_bytes[p];
      }
      expect[i] = d_.layers[size_t(x_.gated[res[i].first])].hash[res[i].second];
    }
    void* buf = nullptr;
    const size_t bytes = n * (sizeof(dev::HashUnit) + 16) + 16;
    ck(cudaMalloc(&buf, bytes), "cudaMalloc (verify)");
    auto* du = static_cast<dev::HashUnit*>(buf);
    auto* de = reinterpret_cast<uint64_t*>(du + n);
    auto* dout = de + n;
    auto* dmis = reinterpret_cast<uint32_t*>(dout + n);  // [0] mismatches, [1] this call's staging timeouts
    cudaStream_t s = mover_->stream(Mover::kDem);
    uint32_t words[2] = {0, 0};
    try {
      ck(cudaMemcpyAsync(du, units.data(), n * sizeof(dev::HashUnit), cudaMemcpyHostToDevice, s), "verify upload");
      ck(cudaMemcpyAsync(de, expect.data(), n * 8, cudaMemcpyHostToDevice, s), "verify upload");
      ck(cudaMemsetAsync(dmis, 0, 8, s), "verify clear");
      ck_launch(dev::launch_xxh64(du, uint32_t(n), de, dout, nullptr, dmis, s, dmis + 1), "xxh64 kernel");
      ck(cudaMemcpyAsync(words, dmis, 8, cudaMemcpyDeviceToHost, s), "verify result");
      ck(cudaStreamSynchronize(s), "verify sync");
      require(!words[1], SS_E_BACKEND, "device-gated: a staging copy of the xxh64 kernel did not complete");
    } catch (...) {
      cudaFree(buf);
      throw;
    }
    cudaFree(buf);
    const uint32_t mism = words[0];
    require(mism == 0, SS_E_HASH,
            "device-gated: " + std::to_string(mism) + " resident unit(s) differ from their descriptor hashes");
  }

  void close() noexcept {
    if (closed_) return;
    closed_ = true;
    if (m_.host_abort) store_release(m_.host_abort, 1);
    if (svc_) svc_->stop_join();
    if (mover_) mover_->drain_all();
    cudaDeviceSynchronize();
    svc_.reset();
    core_.reset();
    mover_.reset();
    async_.reset();
    flight_pools_.clear();
    readers_.reset();
    for (char* a : bufs_.arena) cudaFree(a);
    if (bufs_.slot_of) cudaFree(bufs_.slot_of);
    if (expect_dev_) cudaFree(expect_dev_);
    if (done_cnt_) cudaFree(done_cnt_);
    if (ctl_) cudaFree(ctl_);
    if (mapped_h_) cudaFreeHost(mapped_h_);
    if (stamps_h_) cudaFreeHost(stamps_h_);
    free_pinned(pinned_);
    chunks_.clear();
    if (bufs_.staging) cudaFreeHost(bufs_.staging);
  }

  Desc d_;
  ss_options o_;
  std::unique_ptr<PeerTier> peer_;  // the peer tier's owners and store addresses (null: pinned RAM only)
  Layout x_;
  int device_ = 0;
  std::vector<std::unique_ptr<SourceFile>> files_;
  static constexpr uint64_t kReadPiece = uint64_t(8) << 20;  // file tier: the reader pool's piece
  std::unique_ptr<ReadPool> readers_;                        // file tier: the reads of one miss at once
  std::vector<std::unique_ptr<ReadPool>> flight_pools_;      // file tier: one per reader thread of async_
  std::unique_ptr<AsyncReads> async_;                        // file tier: reads in flight (dg_disk_queue > 1)
  uint32_t adapt_ = 0;            // dg_disk_queue_adapt: 0 off, 1 adapting (async_'s controller), 2 declined
  const char* adapt_why_ = "";    // (declined: why)
  CudaMover::Buffers bufs_;
  uint32_t* ctl_ = nullptr;
  uint64_t* expect_dev_ = nullptr;  // the landing check: descriptor hashes in key order
  uint32_t* done_cnt_ = nullptr;    // the landing check: CTAs finished per launch ring entry
  uint32_t* bad_flag_h_ = nullptr;  // mapped: set by a mismatch
  uint32_t* bad_log_h_ = nullptr;   // mapped: (key, slot) of the first mismatches
  uint64_t check_marks_[2] = {0, 0};  // the last check launch of the two previous tokens
  uint64_t check_failed_ = 0, check_repaired_ = 0;
  double check_wait_s_ = 0;
  void* mapped_h_ = nullptr;
  unsigned long long* stamps_h_ = nullptr;
  std::vector<void*> chunks_;       // the block chunks' host addresses
  std::vector<PinnedChunk> pinned_;  // their allocation
  dev::DgDev dev_{};
  Mapped m_;
  std::unique_ptr<CudaMover> mover_;
  std::unique_ptr<SlotCache> core_;
  std::unique_ptr<Service> svc_;
  std::vector<uint8_t> held_;  // gated layers holding a ss_dg_make_resident set (not exported)
  std::vector<std::vector<uint32_t>> keep_;
  std::vector<uint8_t> run_;
  uint32_t seq_ = 0;
  bool in_token_ = false, poisoned_ = false, closed_ = false, skip_edge_ = false, timeline_valid_ = false;
  uint32_t module_loading_ = 0;
  CacheStats base_;
  std::vector<LayerCounts> lbase_;
  uint64_t evicted_before_ = 0;
  ss_dg_boundary_timeline boundary_{};
  std::vector<double> gpu_wait_us_, gpu_ready_us_;
  double open_seconds_ = 0, open_alloc_s_ = 0, open_fill_pinned_s_ = 0, open_fill_res_s_ = 0, open_verify_s_ = 0;
  double open_fill_s_ = 0, open_arena_s_ = 0, open_pinned_s_ = 0, open_cache_s_ = 0;
  bool load_serial_ = false;
  LoadStats load_;
  unsigned load_readers_ = 0, load_buffers_ = 0;
  uint64_t load_buffer_bytes_ = 0;
};

}  // namespace

DeviceScope::DeviceScope(int device) {
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess) {
    (void)cudaGetLastError();
    cur = -1;
  }
  if (cur != device && cudaSetDevice(device) == cudaSuccess) prev_ = cur;
  else (void)cudaGetLastError();
}
DeviceScope::~DeviceScope() {
  if (prev_ >= 0) cudaSetDevice(prev_);
}

// The device-gated layout of an open as numbers (the layout test hook): keys, R, D, B, P, Q, I, F, S, disk_queue,
// blocks, persistent_slots, slots, guard_slot, unit_bytes, host_stride, disk_tier, disk_prefetch, scored, w_trans,
// w_freq, w_rec, the resident count; then the residents' keys.
std::vector<uint64_t> dg_layout_summary(const Desc& d, const Plan& p, const ss_options& o,
                                        std::vector<uint32_t>* residents) {
  const Layout x = make_layout(d, p, o, nullptr);
  if (residents) *residents = x.residents;
  return {x.keys, x.R, x.D, x.B, x.P, x.Q, x.I, x.F, x.S, x.disk_queue, x.blocks, x.persistent_slots, x.slots,
          x.guard_slot, x.unit_bytes, x.host_stride, x.disk_tier, x.disk_prefetch, x.scored, x.w_trans, x.w_freq,
          x.w_rec, x.residents.size(), x.L, x.landing_queued, x.landing_ttl, x.landing_chunk};
}

std::unique_ptr<DgContext> open_dg_context(const Desc& d, const Plan& p, const ss_options& o, const PeerTier* peer) {
  require(o.backend == SS_BACKEND_CUDA, SS_E_UNSUPPORTED,
          "device-gated: this build has the CUDA backend only (ss_options.backend = SS_BACKEND_CUDA)");
  return std::make_unique<CudaDgContext>(d, p, o, peer);
}

}  // namespace tsb
