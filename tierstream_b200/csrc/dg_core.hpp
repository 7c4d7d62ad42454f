// Device-gated decode: the slot cache's state machine, with no device API in it. A Mover performs the copies, the
// table publications and the events on three streams; the CUDA mover lives in dg_ctx.cu (copy engines or this
// library's gather kernels), a host mover in dg_host_mover.cpp (the CPU tests and the deterministic replay).
//
// Every gated unit (key = unit_base[g] + unit) has one home: a slot of the arena shared by all gated layers
// (Device; Coming while its copy is in flight; Bank for a demand served through a per-layer bank slot; Evicting while
// its write-back runs), a pinned block (Host), or, with the file tier, only its file (File). Inside a token entries
// only go from -1 to a slot, published on the stream that copied the bytes; evictions happen at the boundary
// (end_token), whose write-backs are either enqueued there or deferred part by part into the next token's served
// layers.
//
// The decisions are those of the reference's DgCore (dg_core.cpp) for its LRU configuration with two tiers, or three
// with synchronous file reads, so the slot table after every token matches it on the same trace when the schedule is
// deterministic:
//   - open placement: residents by priority into slots 0.., every other key a block in key order
//     (dg_core.cpp:769-858); free slots and blocks are LIFO stacks whose next is the lowest index;
//   - a demand miss takes the last free slot, else (write-backs deferred) waits for one, else its layer's bank slot
//     (bank g & 1, reused two layers later) (dg_core.cpp:1146-1368, 1059-1097);
//   - a prefetch keeps prefetch_reserve slots free and stays under the per-layer and per-token budgets;
//   - the boundary admits the token's arrivals, returns bank units to their blocks, collects finished write-backs,
//     then evicts from the recency tail until free + pending write-backs reaches the spare target, one free block per
//     victim (dg_core.cpp:1636-1927); deferred write-backs are carried and flushed by the same counts;
//   - file tier (the reference's dg_disk_tier with synchronous reads, dg_disk_queue 0 / 1): the open gives blocks to
//     home_blocks non-resident units (the plan's pinned units first, then by priority) and leaves the rest in their
//     files; a file miss reads the unit into the next of disk_staging staging buffers (round robin, after that
//     buffer's last copy landed) and copies it from there; pinned homes keep a recency order of their own, and a
//     victim with no free block frees one by dropping the least recently homed pinned unit to its file, or goes to
//     its own file when no pinned unit is left (dg_core.cpp:113-238, 769-858, 1146-1368, 1783);
//   - scored eviction (the reference's SS_POLICY_SCORED / SCORED_AUTO with its boundary selection): per gated layer a
//     transition count table between successive tokens' unions of routed ids, a frequency ring of the last 16 unions
//     and each unit's last routed token; the boundary takes, among the same eligible units, the lowest integer scores
//     w_t P + w_f F + w_r Rec first (ties: the older use, then the less recent unit) instead of the recency tail
//     (dg_core.cpp:1933-2130, 1811-1826);
//   - placement rounds (between tokens): a decayed count per unit of the tokens that routed it; a round promotes the
//     hottest pinned units to the device (into free slots while the device holds less than its share, else in place of
//     the coldest device unit when hotter by the hysteresis factor) and, with the file tier, the hottest file units into
//     the blocks of the coldest pinned ones (dg_core.cpp:2592-2897).
#pragma once

#include <atomic>
#include <cstdint>
#include <deque>
#include <functional>
#include <string>
#include <utility>
#include <vector>

namespace tsb {

class Mover {
 public:
  enum Stream { kDem = 0, kPf = 1, kD2h = 2 };
  virtual ~Mover() = default;
  virtual uint32_t parts() const = 0;
  virtual uint64_t part_bytes(uint32_t p) const = 0;
  // Every part of unit `key`, held by `block`, into `slot` (block -1 = the one-unit reset staging buffer).
  virtual void h2d(Stream s, int32_t slot, int32_t block, uint32_t key) = 0;
  // Part p (p < 0: every part) of unit `key`, held by `slot`, into `block`.
  virtual void d2h(Stream s, int32_t slot, int32_t block, int32_t p, uint32_t key) = 0;
  // Reset: slot-to-slot moves (src, dst). Moves of one wave touch disjoint slots and run together; waves run in
  // ascending order. Complete when the call returns.
  virtual void d2d_moves(const std::vector<std::pair<int32_t, int32_t>>& moves, const std::vector<uint32_t>& wave) = 0;
  virtual void h2h(int32_t src_block, int32_t dst_block, uint32_t key) = 0;
  // File tier: every part of unit `key` from its file into `block` (blocks [blocks, blocks + disk_staging) are the
  // staging buffers, -1 the reset staging buffer), synchronously; no copy reads the block meanwhile.
  virtual void read_unit(uint32_t key, int32_t block);
  // The same read in flight (disk_queue > 1): begin starts it and returns a handle; end waits for it, rethrows its
  // failure and returns its own read time in ns (0: begin was the read); done answers without waiting. Every begun
  // read is ended once. Default: begin is the synchronous read.
  virtual void* read_begin(uint32_t key, int32_t block) {
    read_unit(key, block);
    return nullptr;
  }
  virtual uint64_t read_end(void* handle) {
    (void)handle;
    return 0;
  }
  virtual bool read_done(void* handle) {
    (void)handle;
    return true;
  }
  // Landings (landing_blocks): the same checked read into landing block `block` (blocks + disk_staging + l), behind
  // every demand read not started yet, ended and queried like read_begin's handles (ending one still queued starts
  // it first). A landing read not running can be cancelled (true: nothing more is written to its block and the handle
  // is gone; false: it runs or ran, end it as usual) and a running one asked to stop early (it is still ended). How
  // one ended: aborted (stopped before its end: its block holds part of the unit), the bytes it did not read, the
  // times it gave its reader to a demand read. Defaults: the plain read, never cancelled or stopped.
  struct LandingEnd {
    uint64_t aborted_bytes = 0;
    uint32_t yields = 0;
    bool aborted = false;
  };
  virtual void* read_landing_begin(uint32_t key, int32_t block) { return read_begin(key, block); }
  virtual uint64_t read_landing_end(void* handle, LandingEnd* end) {
    *end = LandingEnd{};
    return read_end(handle);
  }
  virtual bool read_landing_cancel(void* handle, LandingEnd* end) noexcept {
    (void)handle;
    *end = LandingEnd{};
    return false;
  }
  virtual void read_landing_abort(void* handle) noexcept { (void)handle; }
  // slot_of[key] = v after everything enqueued on s so far (a release at system scope).
  virtual void publish(Stream s, uint32_t key, int32_t v) = 0;
  // ready[g] = seq on kDem after everything enqueued there.
  virtual void ready(uint32_t g, uint32_t seq) = 0;
  virtual void* event_create() = 0;
  virtual void event_destroy(void* ev) = 0;
  virtual void record(void* ev, Stream s) = 0;
  virtual void wait(Stream s, void* ev) = 0;  // device side
  virtual bool done(void* ev) = 0;            // host query
  virtual void event_sync(void* ev) = 0;
  virtual void sync(Stream s) = 0;
  virtual void upload_table(const int32_t* table, uint32_t n) = 0;  // the whole table on kDem, then sync
  // Only entries [ranges[2 i], ranges[2 i] + ranges[2 i + 1]) for i < n, on kDem, then sync (also with n = 0): the
  // device table's other entries are not written.
  virtual void upload_table_ranges(const int32_t* table, const uint32_t* ranges, uint32_t n) = 0;
  // Timing marks on kDem for a layer with a miss: which = 0 before its first demand copy, 1 after its ready.
  virtual void diag_mark(uint32_t g, int which) {
    (void)g;
    (void)which;
  }
};

struct CacheConfig {
  std::vector<uint32_t> n_units;  // per gated layer
  uint32_t persistent_slots = 0;  // residents + spare slots: [0, persistent_slots)
  uint32_t bank_slots = 0;        // per bank: [persistent_slots, persistent_slots + 2 * bank_slots)
  uint32_t blocks = 0;
  uint32_t spare_target = 0;
  uint32_t prefetch_reserve = 0;
  bool prefetch_reserve_auto = false;  // follows the spare target: min(24, spare_target / 4)
  uint32_t prefetch_per_layer = 4, prefetch_per_token = 48;
  bool wb_defer = false, wb_on_d2h = false;
  uint64_t wb_layer_bytes = 0, wb_max_outstanding = 0;
  // Inclusive share (dg_inclusive_blocks): at most this many device units keep the pinned block they were promoted
  // from as a clean copy, so their eviction is a drop with no write-back (0 = exclusive).
  uint32_t inclusive = 0;
  // File tier (dg_disk_tier): see the file comment. disk_prefetch: predictions may read file-homed units too.
  bool disk_tier = false, disk_prefetch = false;
  uint32_t home_blocks = 0, disk_staging = 0;
  // file reads in flight at once (1 = each read inside its fetch): a read's copy and entry follow when it ends, at the
  // first drain point that needs it (its key touched again, its layer's ready, its staging buffer reused, a full queue,
  // the boundary); a prefetch's read may stay in flight across the service's calls
  uint32_t disk_queue = 1;
  // Scored eviction: the history is kept from the open when `scored` (the tables exist only then); scored_auto takes
  // scored victims only after a boundary of more than one row. Weights out of 1000 (sum 1000); max_ids = the most ids
  // one export holds (a union's bound).
  bool scored = false, scored_auto = false;
  uint32_t w_trans = 700, w_freq = 200, w_rec = 100;
  uint32_t max_ids = 64;
  // The reference's opt-in policies: no_admit = every demand miss served through its layer's bank slot and released at
  // the boundary (homes never change; no prefetch, no boundary eviction); clean_evict (file tier) = a victim that
  // would need a block while none is free goes to its file with no copy, no pinned unit dropped for it; pf_revert = an
  // unused prefetch goes back at the boundary (to its block at the pinned recency tail, or its file), not admitted;
  // pf_strict = a prefetch also leaves the spare target's slots free.
  bool no_admit = false, clean_evict = false, pf_revert = false, pf_strict = false;
  // bank_keep (file tier; no effect with no_admit): a demand file miss served through a bank slot is read into a
  // pinned block (a free one, else the least recently homed pinned unit's, that unit going to its file) instead of a
  // staging buffer, and that block is its pinned home once the bank lets it go: at the front of the pinned recency
  // list (1), or after its front half (2), so that a unit read once does not push out the most recently homed ones
  // (dg_core.cpp:237-250, 1286-1303, 142-160, 200-213).
  uint32_t bank_keep = 0;
  // landing_blocks (file tier, reads in flight): a prediction of a file-homed unit reads it into one of this many
  // pinned landing blocks instead of a slot (no slot taken, nothing evicted, outside the prefetch budgets; no free
  // landing block: the advice is dropped); a demand then copies it from there (a read still running ends first, never
  // a second read). landing_ttl 0: a landing its layer did not route goes back to its file right after that layer's
  // demand, and a prediction for a layer already served this token is not issued; N >= 1: a landing not demanded
  // for N boundaries goes back to its file. Every read in flight ends at the boundary (dg_core.cpp:440-612,
  // 1146-1162, 1216-1222, 1309-1324, 1439-1460, 1633, 1648-1662, 2499-2511, 2910-2919, 2997-2999).
  uint32_t landing_blocks = 0, landing_ttl = 0;
};

struct CacheStats {
  uint64_t tokens = 0, lookups = 0, misses = 0, covered = 0, fetched = 0, prefetched = 0, prefetch_used = 0;
  uint64_t resurrected = 0, bank_serves = 0, collected_mid = 0, evicted = 0, evict_short = 0, writebacks_done = 0;
  uint64_t stalled = 0, pred_invalid = 0, covered_waits = 0, predicted = 0, predicted_true = 0, miss_layers = 0;
  uint64_t wb_deferred = 0, wb_cancelled = 0, wb_forced = 0, wb_boundary_flushed = 0;
  uint64_t wb_issued_bytes = 0, wb_completed_bytes = 0, wb_cancelled_bytes = 0, wb_boundary_flushed_bytes = 0;
  uint64_t wb_forced_wait_ns = 0;
  uint64_t reset_moves = 0, reset_bytes = 0;
  uint64_t inclusive_kept = 0, inclusive_drops = 0;
  // file tier: reads of file-homed units and their bytes and summed time; reads that waited for their staging
  // buffer's last copy; pinned units dropped to their file to free a block; victims dropped to their file
  uint64_t disk_reads = 0, disk_read_bytes = 0, disk_read_ns = 0, disk_stage_waits = 0, disk_drops = 0;
  uint64_t disk_discards = 0;
  // reads begun while another was in flight, the most in flight at once, reads ended in a later public call than
  // their fetch's and their bytes, the wall time spent waiting for reads to end
  uint64_t disk_overlapped = 0, disk_max_in_flight = 0, disk_carried = 0, disk_carried_bytes = 0, disk_wait_ns = 0;
  // scored eviction: boundaries that fell back to the recency order (a layer without this token's ranking), victims
  // taken by score, layers scored and the candidates they ranked, saturated transition increments, selection time
  uint64_t score_fallbacks = 0, scored_victims = 0, score_layers = 0, score_candidates = 0, score_saturated = 0;
  uint64_t score_ns = 0;
  // placement rounds: rounds run, units whose home they changed, bytes moved, host time, rounds cancelled
  uint64_t round_count = 0, round_units = 0, round_bytes = 0, round_ns = 0, round_cancelled = 0;
  // opt-in policies: victims dropped to their file by clean_evict and their bytes; unused prefetches reverted and
  // their bytes; prefetches pf_strict refused
  uint64_t clean_drops = 0, clean_drop_bytes = 0, pf_reverted = 0, pf_revert_bytes = 0, pf_strict_refused = 0;
  // bank_keep: file reads kept in a pinned block; pinned units dropped to their file for one; of those, the ones read
  // back from their file within 8 tokens
  uint64_t bank_kept = 0, bank_keep_drops = 0, bank_keep_rereads = 0;
  // landings: reads begun; demands served from a landing block (late ones included) and of those the ones whose read
  // was still running, with the host's wait for them; landings back to their file unused (TTL); advice dropped with no
  // free landing block; bytes landed; reads that failed; reads cancelled before running; (TTL 0) landings their layer
  // did not route and predictions for a layer already served; a chunked read's yields and the bytes it did not read
  uint64_t landing_issued = 0, landing_promoted = 0, landing_late = 0, landing_wait_ns = 0, landing_expired = 0;
  uint64_t landing_dropped_full = 0, landing_read_bytes = 0, landing_failed = 0, landing_cancelled = 0;
  uint64_t landing_expired_layer = 0, landing_skipped_passed = 0, landing_yields = 0, landing_aborted_bytes = 0;
  // make_resident: units copied in and evicted, bytes copied in, host time; its file reads, their bytes and time,
  // its write-back bytes
  uint64_t resident_units = 0, resident_evicted = 0, resident_bytes = 0, resident_ns = 0;
  uint64_t mkres_file_reads = 0, mkres_file_bytes = 0, mkres_read_ns = 0, mkres_h2d_bytes = 0, mkres_wb_bytes = 0;
};

// A placement round's limits and what it did (ss_dg_round_params / ss_dg_round_result without the struct sizes).
struct RoundIn {
  uint64_t budget_bytes = 0;  // file reads + host-to-device copies + write-backs (0 = no limit)
  uint32_t max_units = 96;    // promotions at most
  double hysteresis = 1.25;   // a unit replaces another only when its count is above this x the other's
  double decay = 0.85;        // s = decay x s + hits since the last round
  uint32_t flags = 0;
};
struct RoundOut {
  uint32_t promoted_to_device = 0, promoted_to_pinned = 0, demoted_from_device = 0, dropped_to_file = 0;
  uint32_t cancelled = 0;
  uint64_t bytes_read = 0, bytes_h2d = 0, bytes_written_back = 0, ns = 0;
};

struct LayerCounts {
  uint64_t lookups = 0, misses = 0, fetched = 0, bank_serves = 0, prefetched = 0, prefetch_used = 0, evicted = 0;
};

class SlotCache {
 public:
  // Landing / Landed (landing_blocks): a file home whose landing read is running / done, holding a landing block
  enum class Home : uint8_t { Host, Device, Coming, Bank, Evicting, File, Landing, Landed };
  enum Mutation { kNone0 = 0, kEntryBeforeCopy = 1, kNoCover = 2 };

  SlotCache(const CacheConfig& cfg, Mover* m);
  ~SlotCache();
  SlotCache(const SlotCache&) = delete;
  SlotCache& operator=(const SlotCache&) = delete;

  // Open: `order` names keys by priority (duplicates ignored); the first persistent_slots - spare_target distinct
  // ones take slots 0.., in that recency order; every other key takes a block, numbered in key order. File tier:
  // `disk` flags the plan's disk units; only min(home_blocks, blocks) non-resident keys take a block (unflagged ones
  // first, each group by priority; the first most recently homed), the others are file-homed.
  void place(const std::vector<uint32_t>& order, const std::vector<uint8_t>* disk = nullptr);

  uint32_t keys() const { return keys_; }
  uint32_t gated() const { return uint32_t(base_.size() - 1); }
  uint32_t key(uint32_t g, uint32_t u) const { return base_[g] + u; }
  uint32_t units(uint32_t g) const { return base_[g + 1] - base_[g]; }
  uint32_t gated_of(uint32_t k) const;
  const std::vector<uint32_t>& unit_base() const { return base_; }
  const std::vector<int32_t>& table() const { return table_; }
  int32_t slot_of(uint32_t k) const { return e_[k].slot; }
  int32_t block_of(uint32_t k) const { return e_[k].block; }
  Home home(uint32_t k) const { return e_[k].home; }
  uint32_t on_device() const { return on_device_; }
  uint32_t free_slots() const { return uint32_t(free_slots_.size()); }
  uint32_t free_blocks() const { return uint32_t(free_blocks_.size()); }
  uint32_t deferred() const { return uint32_t(deferred_.size()); }
  uint32_t backed_units() const { return backed_; }
  uint32_t file_units() const { return on_file_ + on_land_; }  // (landings' homes are their files)
  uint32_t landing_units() const { return on_land_; }
  // Pinned homes, most recently homed first (file tier only).
  std::vector<uint32_t> host_order() const;
  uint64_t wb_outstanding_bytes() const { return outstanding_; }
  const CacheStats& stats() const { return st_; }
  const std::vector<LayerCounts>& layer_counts() const { return lc_; }
  const CacheConfig& config() const { return c_; }
  uint32_t coming() const;
  // Most recently used first, device homes only.
  std::vector<uint32_t> residency() const;

  // ---- inside a token (the service thread) ----
  // run (optional, one flag per gated layer): the layers this token exports (scored eviction ranks the others at the
  // boundary from their unchanged history).
  void begin_token(uint32_t seq, const std::vector<uint8_t>* run = nullptr);
  void serve_demand(uint32_t g, const uint32_t* ids, uint32_t n, uint64_t mask);
  void serve_use(uint32_t g, const uint32_t* ids, uint32_t n, uint64_t mask);
  void serve_prediction(uint32_t g_next, const uint32_t* pred, uint32_t n, bool ahead);
  // Deferred write-back parts after layer g was served (its ready already enqueued); ahead() is asked before every
  // part: a later layer already exported, so no more parts now.
  void issue_writebacks(uint32_t g, const std::function<bool()>& ahead);

  // ---- between tokens (the engine thread) ----
  // rows: the token's rows (scored_auto takes scored victims only above 1).
  void end_token(const std::vector<uint32_t>& keep, uint32_t rows = 1);
  // Scored eviction: gated layer g is closed for this token (its union, epochs and stamps are final); the service
  // calls it after each served layer.
  void score_layer(uint32_t g);
  // Between tokens: LRU (0), SCORED (1) or SCORED_AUTO (2); the history restarts and the recency stamps follow the
  // current recency order. Scoring must have been set up at the open (scored).
  void set_policy(uint32_t policy);
  bool scored() const { return c_.scored; }
  bool scoring_ready() const { return !sc_.empty(); }
  // A score profile's transition counts (units(g)^2 per gated layer, row-major [previous unit][unit]) as the open
  // state of the tables (scored only; kept for reset_open).
  void load_counts(const std::vector<std::vector<uint32_t>>& cells);
  // Between tokens: gated layer g's units `units` (distinct ids) all on the device (ss_dg_make_resident), the call's
  // other protected keys `other_kept` never evicted. Every refusal comes before any action; then every copy landed
  // and the table is uploaded when it returns. Victims in the policy's order (the recency tail, or scores) with the
  // boundary's lower-tier rules; copies in from the pinned block or, through the staging buffers, the file; the units
  // copied in become the most recent (dg_core.cpp:2248-2590).
  struct ResidentResult {
    uint32_t copied = 0, evicted = 0;
  };
  ResidentResult make_resident(uint32_t g, const std::vector<uint32_t>& units, const std::vector<uint32_t>& other_kept);
  // Between tokens: one placement round (kept: keys that never move). Every copy landed and the table is uploaded when
  // it returns.
  RoundOut round(const RoundIn& in, const std::vector<uint32_t>& kept);
  // Any thread: a running round stops at its next unit boundary (no effect when none runs).
  void cancel_round() {
    int running = kRoundRunning;
    round_state_.compare_exchange_strong(running, kRoundCancel, std::memory_order_acq_rel);
  }
  void seed_round_counts(const std::vector<uint32_t>& keys, const std::vector<float>& counts);
  // The last round's result (also after a failure once it began; zeros before the first).
  const RoundOut& last_round() const { return last_round_; }
  double round_count(uint32_t k) const { return rs_[k]; }
  uint32_t seed(const std::vector<uint32_t>& keys);
  void drain();
  // Restores the open placement, moving only misplaced units; `plan` receives the slot-to-slot moves in execution
  // order when given (the mover performs them as they come).
  void reset_open();
  void set_wb_defer(bool on);
  void set_spare_target(uint32_t n);
  void set_prefetch_budget(uint32_t per_layer, uint32_t per_token);
  void set_pressure(uint32_t free_per_token, uint32_t evict_recent);
  void set_clean_evict(bool on);
  void set_pf_revert(bool on);
  // While some layer is held (ss_dg_make_resident): uploads write only the entries changed since the last upload,
  // so an engine kernel reading a held layer's entries never meets a write; off: the whole table in one copy.
  void set_range_uploads(bool on);
  void set_mutation(int m) { mut_ = m; }
  // Every ownership rule (throws SS_E_BACKEND naming the first broken one).
  void check() const;

 private:
  static constexpr uint32_t kNil = 0xffffffffu;
  // An intrusive doubly linked list of keys (front: the most recent); the links live in the list, one pair per key.
  class KeyList {
   public:
    void reset(uint32_t keys) {
      link_.assign(keys, Link{});
      front_ = back_ = kNil;
    }
    bool has(uint32_t k) const { return link_[k].in; }
    uint32_t front() const { return front_; }
    uint32_t back() const { return back_; }
    uint32_t older(uint32_t k) const { return link_[k].next; }  // toward the back
    uint32_t newer(uint32_t k) const { return link_[k].prev; }  // toward the front
    void push_front(uint32_t k) { insert(k, kNil, front_); }
    void push_back(uint32_t k) { insert(k, back_, kNil); }
    void insert_behind(uint32_t at, uint32_t k) { insert(k, at, link_[at].next); }  // just older than `at`
    void erase(uint32_t k) {
      Link& l = link_[k];
      (l.prev == kNil ? front_ : link_[l.prev].next) = l.next;
      (l.next == kNil ? back_ : link_[l.next].prev) = l.prev;
      l = Link{};
    }

   private:
    struct Link {
      uint32_t prev = kNil, next = kNil;
      bool in = false;
    };
    void insert(uint32_t k, uint32_t before, uint32_t after) {
      link_[k] = Link{before, after, true};
      (before == kNil ? front_ : link_[before].next) = k;
      (after == kNil ? back_ : link_[after].prev) = k;
    }
    std::vector<Link> link_;
    uint32_t front_ = kNil, back_ = kNil;
  };
  // The pinned homes, front = most recently homed, with a cursor on the oldest unit of the front half (its size / 2
  // newest units) kept through every change, so a unit can enter right behind that half in O(1) (bank_keep 2).
  class HomeList {
   public:
    void reset(uint32_t keys) {
      list_.reset(keys);
      in_front_.assign(keys, 0);
      edge_ = kNil;
      size_ = front_n_ = 0;
    }
    bool has(uint32_t k) const { return list_.has(k); }
    uint32_t front() const { return list_.front(); }
    uint32_t back() const { return list_.back(); }
    uint32_t older(uint32_t k) const { return list_.older(k); }
    uint32_t newer(uint32_t k) const { return list_.newer(k); }
    void push_front(uint32_t k) {
      list_.push_front(k);
      in_front_[k] = 1;
      ++front_n_;
      if (edge_ == kNil) edge_ = k;
      grew();
    }
    void push_back(uint32_t k) {
      list_.push_back(k);
      grew();
    }
    void push_behind_front_half(uint32_t k) {
      if (edge_ == kNil) list_.push_front(k);
      else list_.insert_behind(edge_, k);
      grew();
    }
    void erase(uint32_t k) {
      if (in_front_[k]) {
        in_front_[k] = 0;
        --front_n_;
        if (edge_ == k) edge_ = list_.newer(k);
      }
      list_.erase(k);
      --size_;
      settle();
    }
    // The cursor's invariant, walked: the first size / 2 units are marked as the front half, none after them, and the
    // cursor is the last marked one (none when the half is empty).
    bool consistent() const {
      uint32_t at = 0, last_front = kNil;
      for (uint32_t k = list_.front(); k != kNil; k = list_.older(k), ++at) {
        if (at > size_) return false;  // (a cycle)
        if (bool(in_front_[k]) != (at < size_ / 2)) return false;
        if (in_front_[k]) last_front = k;
      }
      return at == size_ && front_n_ == size_ / 2 && last_front == edge_;
    }

   private:
    void grew() {
      ++size_;
      settle();
    }
    // the front half back to size / 2 units: one step per change at most
    void settle() {
      for (; front_n_ > size_ / 2; --front_n_) {
        in_front_[edge_] = 0;
        edge_ = list_.newer(edge_);
      }
      for (; front_n_ < size_ / 2; ++front_n_) {
        edge_ = edge_ == kNil ? list_.front() : list_.older(edge_);
        in_front_[edge_] = 1;
      }
    }
    KeyList list_;
    std::vector<uint8_t> in_front_;
    uint32_t edge_ = kNil, size_ = 0, front_n_ = 0;
  };
  // Free slots or blocks: a stack whose next is the one returned last (at open, the lowest index).
  class LifoPool {
   public:
    void clear() { v_.clear(); }
    void fill_down(int32_t hi, int32_t lo) {  // hi - 1 .. lo pushed in that order: lo is taken first
      v_.clear();
      for (int32_t i = hi; i-- > lo;) v_.push_back(i);
    }
    void give(int32_t i) { v_.push_back(i); }
    int32_t take() {
      const int32_t i = v_.back();
      v_.pop_back();
      return i;
    }
    bool empty() const { return v_.empty(); }
    size_t size() const { return v_.size(); }
    const std::vector<int32_t>& items() const { return v_; }

   private:
    std::vector<int32_t> v_;
  };
  struct Entry {
    Home home = Home::Host;
    int32_t slot = -1, block = -1;
    bool wb_pending = false, via_pf = false, used = false;
    bool backed = false;  // a device unit whose block still holds its bytes (inclusive share)
    bool keep_mid = false;  // bank_keep 2: a kept read, homed behind the pinned list's front half when released
    int32_t land = -1;      // Landing / Landed: its landing block
    uint32_t land_age = 0;  // Landed: boundaries passed since
    uint64_t keep_drop = 0;  // bank_keep: tokens + 1 when dropped to its file for a kept read (0: not)
    uint64_t demand_epoch = 0, lru_stamp = 0;  // scored: the last token that routed it; its recency list position
    void* pf_done = nullptr;
  };
  struct Writeback {
    uint32_t key;
    int32_t slot, block;
    void* done;
    bool discard;
    uint64_t bytes;
  };
  struct Deferred {
    uint32_t key;
    int32_t slot, block;
    uint32_t parts_done;
    uint64_t bytes;
  };
  // The state reset_open restores.
  struct OpenState {
    CacheConfig cfg;
    std::vector<Entry> ent;
    std::vector<int32_t> table;
    LifoPool slots, blocks;
    KeyList recent;
    HomeList homes;
    LifoPool lands;
    uint32_t on_device = 0, on_file = 0;
    uint64_t stamp = 0;
  };

  // ---- the recency list and the pinned homes' list ----
  void touch(uint32_t k);          // to the recency front (a fresh stamp when scored)
  void leave_device(uint32_t k);   // out of the recency list, entry withdrawn
  // file tier: a pinned home, most (cold: least) recently homed, or (mid) behind the front half of the list
  void home_push(uint32_t k, bool cold = false, bool mid = false);
  void home_erase(uint32_t k);
  void recycle(void*& ev);         // an event back to the pool
  void count_fetch(uint32_t g, bool prefetch, int delta = 1);
  void count_evicted(uint32_t k);
  // one event of gated layer g: the context's total and the layer's own count
  void bump(uint32_t g, uint64_t CacheStats::*total, uint64_t LayerCounts::*layer) {
    ++(st_.*total);
    ++(lc_[g].*layer);
  }
  // ---- file reads in flight ----
  struct Pending {
    uint32_t key;
    int32_t slot, stage;
    Mover::Stream s;
    bool prefetch, bank, free_counted;  // free_counted: a demand that took a free slot (demand_free_used_)
    void* handle;
    uint64_t entry;  // the public call that began it
  };
  void enter();  // a public entry point: the demand reads end
  void end_reads(const std::function<bool(const Pending&)>& pick);
  void drain_pending(size_t n = SIZE_MAX);
  void drain_demand();
  void drain_key(uint32_t k);
  void drain_layer(uint32_t g, const uint32_t* ids, uint32_t n);
  void finish_pending(const Pending& p);
  void undo_pending(const Pending& p);
  void make_room_for_read();
  // ---- scored eviction ----
  struct ScoreCand {
    uint64_t s, epoch, stamp;
    uint32_t key;
  };
  struct LayerScore {
    std::vector<uint32_t> T, open_T;  // transition counts [r][e]; open_T: a profile's (empty = zeros)
    std::vector<uint64_t> rowsum;
    std::vector<uint16_t> cnt;        // unions of the window holding each unit
    std::vector<uint32_t> ring;       // kWindow unions of at most max_ids ids
    std::vector<uint8_t> ring_len;
    uint32_t ring_head = 0, ring_n = 0;
    std::vector<uint32_t> prev, cur;  // the previous and this token's sorted unions
    uint64_t served = 0, list_epoch = 0;
  };
  static constexpr uint32_t kWindow = 16;
  static constexpr uint64_t kStampLimit = UINT64_MAX - (uint64_t(1) << 40);
  static bool cand_less(const ScoreCand& a, const ScoreCand& b) {
    if (a.s != b.s) return a.s < b.s;
    if (a.epoch != b.epoch) return a.epoch < b.epoch;
    return a.stamp < b.stamp;
  }
  void score_history(uint32_t g);
  ScoreCand score_candidate(uint32_t g, uint32_t u, uint64_t denominator, const ScoreCand* cutoff) const;
  void select_scored(size_t need, const std::function<bool(uint32_t)>& eligible, bool count = true);
  void reset_score();
  void stamp_room(const char* what) const;
  void* event();
  uint32_t collect();
  void submit_part(Deferred& d);
  void* record_front(bool discard);
  void* finish_front();
  void force_free_slot();
  void settle_writebacks(const char* what);
  int32_t bank_slot(uint32_t g);
  bool resurrect(uint32_t k);
  void to_lower(uint32_t k, bool cold = false);
  bool clean_now() const { return c_.clean_evict && c_.disk_tier && free_blocks_.empty(); }
  void count_clean() {
    ++st_.clean_drops;
    st_.clean_drop_bytes += unit_bytes_;
  }
  // the least recently homed pinned unit not in `skip` to its file; count: a disk drop of the boundary
  bool drop_host_lru(const std::vector<uint8_t>* skip = nullptr, bool count = true);
  int32_t keep_block();  // bank_keep: the block a bank-served file read goes to, or -1 (a staging buffer)
  // ---- landings ----
  struct LandRead {
    uint32_t key;
    int32_t land;
    void* handle;
    bool doomed;  // (TTL 0) its layer passed while it ran: back to its file when it ends
  };
  struct LandBusy {  // a landing block a promotion's copy still reads, free once the event completed
    int32_t land;
    void* ev;
  };
  static bool file_homed(Home h) { return h == Home::File || h == Home::Landing || h == Home::Landed; }
  int32_t land_block(int32_t l) const { return int32_t(c_.blocks + c_.disk_staging) + l; }
  bool advise_land(uint32_t g, uint32_t unit);  // true: the landing path took the advice
  bool land(uint32_t k);
  bool end_landing(size_t i);                   // false: failed or doomed (the key back to its file)
  void end_landings();                          // every read in flight, oldest first
  void poll_landings(size_t max = SIZE_MAX);    // the completed ones among the max oldest
  bool cancel_landing(size_t i);
  void cancel_landings();                       // the ones not running
  void expire_layer_landings(uint32_t g, const uint32_t* ids, uint32_t n);
  void unland(uint32_t k);                      // back to its file, its landing block free
  void reclaim_lands(bool synced);              // landing blocks whose promotion copy landed back to the free list
  int32_t take_stage();
  void publish(Mover::Stream s, uint32_t k, int32_t v);
  bool fetch(uint32_t g, uint32_t unit, bool prefetch);
  void cover(uint32_t g, uint32_t unit);
  void use(uint32_t g, uint32_t unit, bool was_miss);
  void apply_wb_defer();
  [[noreturn]] void broken(const std::string& what) const;

  CacheConfig c_;
  Mover* m_;
  std::vector<uint32_t> base_;
  uint32_t keys_ = 0, slots_ = 0, bank_first_ = 0;
  std::vector<Entry> e_;
  std::vector<int32_t> table_;
  // Changed entries since the last upload: per gated layer the range [dirty_lo_, dirty_hi_] of keys written (empty
  // while lo > hi). device_table_: the device's table as of the last range upload (while device_table_known_), which
  // check() compares with the marks.
  std::vector<uint32_t> dirty_lo_, dirty_hi_, ranges_;
  std::vector<int32_t> device_table_;
  bool ranged_ = false, device_table_known_ = false;
  void set_entry(uint32_t k, int32_t v);
  void clear_dirty();
  void upload();
  LifoPool free_slots_, free_blocks_;
  KeyList recent_;
  HomeList homes_;  // the file tier's pinned homes, front = most recently homed
  uint32_t on_device_ = 0, backed_ = 0, on_file_ = 0;
  OpenState open_;
  uint32_t stage_next_ = 0;
  std::vector<void*> stage_ev_;  // per staging buffer: its last copy's event
  std::vector<Pending> pending_;  // file reads in flight, oldest first
  LifoPool free_lands_;
  std::vector<uint32_t> land_owner_;  // per landing block: its Landing / Landed key (kNil: none)
  std::vector<LandRead> landing_;     // landing reads in flight, oldest first
  std::vector<LandBusy> land_busy_;
  std::vector<uint8_t> served_;       // (TTL 0) the layers whose demand this token served
  std::vector<uint32_t> late_;        // a layer's misses whose landing read still runs (fetched after the others)
  uint32_t on_land_ = 0;
  uint64_t entries_ = 0;          // public calls so far (a read ended in a later one was carried)
  std::vector<LayerScore> sc_;
  std::vector<uint8_t> run_;
  uint64_t epoch_ = 0, stamp_ = 0;
  std::vector<ScoreCand> select_heap_;
  std::vector<double> rs_;         // placement rounds: the decayed counts
  std::vector<uint32_t> rhits_;    // the tokens that routed each unit since the last round
  static constexpr int kRoundIdle = 0, kRoundRunning = 1, kRoundCancel = 2;
  std::atomic<int> round_state_{kRoundIdle};
  RoundOut last_round_;
  std::deque<Writeback> wbs_;
  std::deque<Deferred> deferred_;
  Mover::Stream wb_stream_ = Mover::kDem;
  uint64_t unit_bytes_ = 0, layer_bytes_ = 0, max_outstanding_ = 0, outstanding_ = 0;
  int64_t credit_ = 0;
  size_t prev_evict_ = 0;
  void* post_ready_ev_ = nullptr;
  std::vector<void*> pool_, all_events_;
  std::vector<uint32_t> bank_key_;
  uint32_t bank_seq_[2] = {0, 0}, bank_layer_[2] = {kNil, kNil}, bank_next_[2] = {0, 0};
  std::vector<uint32_t> pf_layer_;
  uint32_t pf_token_ = 0;
  bool pressure_ = false;
  uint32_t pressure_free_ = 0, pressure_recent_ = 0, demand_free_used_ = 0;
  std::vector<uint32_t> coming_, banked_, pred_, uniq_, victims_;
  uint32_t pred_layer_ = kNil;
  std::vector<uint8_t> layer_missed_;
  uint32_t seq_ = 0;
  CacheStats st_;
  std::vector<LayerCounts> lc_;
  int mut_ = 0;
};

}  // namespace tsb
