// The device-gated slot cache (dg_core.hpp states its rules). The state: one Entry per gated key (its home, slot,
// block and flags), the recency list and the pinned homes' list (KeyList: links kept per list), the free slots and
// free blocks (LifoPool), the write-backs in flight (wbs_) and deferred (deferred_), the file reads in flight
// (pending_), and the scored eviction's per-layer history (sc_).
#include "dg_core.hpp"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <numeric>

#include "errors.hpp"

namespace tsb {

namespace {
using Clock = std::chrono::steady_clock;
uint64_t ns_since(Clock::time_point t0) {
  return uint64_t(std::chrono::duration_cast<std::chrono::nanoseconds>(Clock::now() - t0).count());
}
}  // namespace

SlotCache::SlotCache(const CacheConfig& cfg, Mover* m) : c_(cfg), m_(m) {
  base_ = {0};
  for (uint32_t n : c_.n_units) {
    require(n >= 1, SS_E_INVALID, "device-gated: a gated layer without units");
    base_.push_back(base_.back() + n);
  }
  keys_ = base_.back();
  require(c_.persistent_slots >= 1 && c_.spare_target <= c_.persistent_slots, SS_E_INVALID,
          "device-gated: spare target above the persistent slots");
  const uint64_t all_slots = uint64_t(c_.persistent_slots) + 2ull * c_.bank_slots;
  require(all_slots < 0x7fffffffull, SS_E_INVALID, "device-gated: more than 2^31 - 1 slots");
  slots_ = uint32_t(all_slots);
  bank_first_ = c_.persistent_slots;
  require(!c_.inclusive || c_.inclusive < c_.blocks, SS_E_INVALID,
          "device-gated: the inclusive share must leave a block for write-backs");
  require(!c_.disk_tier || c_.disk_staging >= 1, SS_E_INVALID, "device-gated: the file tier needs staging buffers");
  require(c_.disk_tier || (!c_.disk_prefetch && !c_.disk_staging && !c_.home_blocks), SS_E_INVALID,
          "device-gated: file tier options without the file tier");
  require(uint64_t(c_.blocks) + c_.disk_staging < 0x7fffffffull, SS_E_INVALID, "device-gated: too many host blocks");
  require(!c_.no_admit || c_.bank_slots >= c_.max_ids, SS_E_CAPACITY,
          "device-gated: dg_no_admit serves every miss through a bank slot: it needs " + std::to_string(c_.max_ids) +
              " bank slots per bank (dg_max_ids), " + std::to_string(c_.bank_slots) + " configured");
  require(!c_.landing_blocks || c_.disk_tier, SS_E_INVALID, "device-gated: landing blocks without the file tier");
  require(uint64_t(c_.blocks) + c_.disk_staging + c_.landing_blocks < 0x7fffffffull, SS_E_INVALID,
          "device-gated: too many landing blocks");
  stage_ev_.assign(c_.disk_staging, nullptr);
  free_lands_.fill_down(int32_t(c_.landing_blocks), 0);  // (landing block 0 taken first)
  land_owner_.assign(c_.landing_blocks, kNil);
  served_.assign(c_.n_units.size(), 0);
  late_.reserve(c_.max_ids);
  run_.assign(c_.n_units.size(), 1);
  dirty_lo_.assign(c_.n_units.size(), kNil);
  dirty_hi_.assign(c_.n_units.size(), 0);
  rs_.assign(keys_, 0.0);
  rhits_.assign(keys_, 0);
  if (c_.scored) {  // the history's tables exist from the open (the service thread never allocates)
    require(c_.w_trans <= 1000 && c_.w_freq <= 1000 && c_.w_rec <= 1000 && c_.w_trans + c_.w_freq + c_.w_rec == 1000,
            SS_E_INVALID, "device-gated: score weights must each be 0..1000 and sum to 1000");
    require(c_.max_ids >= 1 && c_.max_ids <= 64, SS_E_INVALID, "device-gated: score unions need max ids 1..64");
    sc_.resize(c_.n_units.size());
    for (size_t g = 0; g < sc_.size(); ++g) {
      const size_t n = c_.n_units[g];
      require(n <= 65536, SS_E_INVALID,
              "device-gated: scored eviction needs at most 65536 units per gated layer (gated layer " +
                  std::to_string(g) + " has " + std::to_string(n) + ")");
      LayerScore& h = sc_[g];
      h.T.assign(n * n, 0);
      h.rowsum.assign(n, 0);
      h.cnt.assign(n, 0);
      h.ring.assign(size_t(kWindow) * c_.max_ids, 0);
      h.ring_len.assign(kWindow, 0);
      h.prev.reserve(c_.max_ids);
      h.cur.reserve(c_.max_ids);
    }
    select_heap_.reserve(c_.persistent_slots);
  }
  e_.assign(keys_, Entry{});
  table_.assign(keys_, -1);
  recent_.reset(keys_);
  homes_.reset(keys_);
  bank_key_.assign(2u * size_t(c_.bank_slots), kNil);
  pf_layer_.assign(gated(), 0);
  layer_missed_.assign(gated(), 0);
  lc_.assign(gated(), LayerCounts{});
  if (c_.prefetch_reserve_auto) c_.prefetch_reserve = std::min<uint32_t>(24, c_.spare_target / 4);
  require(m_->parts() >= 1, SS_E_INVALID, "device-gated: a unit without parts");
  for (uint32_t p = 0; p < m_->parts(); ++p) unit_bytes_ += m_->part_bytes(p);
  apply_wb_defer();
  victims_.reserve(c_.persistent_slots);
}

SlotCache::~SlotCache() {
  for (const Pending& p : pending_) {  // a read in flight ends before the buffer it writes can be freed
    try {
      m_->read_end(p.handle);
    } catch (...) {
    }
  }
  for (const LandRead& r : landing_) {  // (a landing read: dropped if it has not started, else waited for)
    Mover::LandingEnd end;
    if (m_->read_landing_cancel(r.handle, &end)) continue;
    try {
      m_->read_landing_end(r.handle, &end);
    } catch (...) {
    }
  }
  for (void* ev : all_events_) m_->event_destroy(ev);
}

void Mover::read_unit(uint32_t, int32_t) {
  fail(SS_E_UNSUPPORTED, "device-gated: this mover cannot read a unit from its file");
}

[[noreturn]] void SlotCache::broken(const std::string& what) const {
  fail(SS_E_BACKEND, "device-gated: cache invariant broken: " + what);
}

uint32_t SlotCache::gated_of(uint32_t k) const {
  return uint32_t(std::upper_bound(base_.begin(), base_.end(), k) - base_.begin()) - 1;
}

uint32_t SlotCache::coming() const {
  return uint32_t(std::count_if(coming_.begin(), coming_.end(), [&](uint32_t k) { return e_[k].home == Home::Coming; }));
}

void SlotCache::apply_wb_defer() {
  layer_bytes_ = max_outstanding_ = 0;
  wb_stream_ = Mover::kDem;
  if (!c_.wb_defer) return;
  if (c_.wb_on_d2h) wb_stream_ = Mover::kD2h;
  layer_bytes_ = c_.wb_layer_bytes ? c_.wb_layer_bytes : m_->part_bytes(0);
  max_outstanding_ = c_.wb_max_outstanding ? c_.wb_max_outstanding : 2 * unit_bytes_;
  require(layer_bytes_ <= uint64_t(INT64_MAX) / 4, SS_E_INVALID, "device-gated: dg_wb_layer_bytes too large");
  if (c_.wb_on_d2h && !post_ready_ev_) post_ready_ev_ = event();
}

// ---- small steps shared by the decisions ----
void SlotCache::touch(uint32_t k) {
  if (recent_.has(k)) recent_.erase(k);
  recent_.push_front(k);
  if (c_.scored) {  // unique stamps, larger nearer the front (stamp_room keeps the counter far from wrapping)
    if (stamp_ == UINT64_MAX) broken("the recency stamp counter wrapped");
    e_[k].lru_stamp = ++stamp_;
  }
}

void SlotCache::leave_device(uint32_t k) {
  if (recent_.has(k)) recent_.erase(k);
  --on_device_;
  set_entry(k, -1);
}

void SlotCache::home_push(uint32_t k, bool cold, bool mid) {
  if (!c_.disk_tier) return;
  if (cold) homes_.push_back(k);  // the least recently homed: the first to drop to its file
  else if (mid) homes_.push_behind_front_half(k);
  else homes_.push_front(k);
}

void SlotCache::home_erase(uint32_t k) {
  if (!c_.disk_tier) return;
  if (!homes_.has(k)) broken("a pinned home outside the pinned recency list");
  homes_.erase(k);
}

void SlotCache::recycle(void*& ev) {
  if (!ev) return;
  pool_.push_back(ev);
  ev = nullptr;
}

void SlotCache::count_fetch(uint32_t g, bool prefetch, int delta) {
  uint64_t& total = prefetch ? st_.prefetched : st_.fetched;
  uint64_t& layer = prefetch ? lc_[g].prefetched : lc_[g].fetched;
  total += uint64_t(int64_t(delta));
  layer += uint64_t(int64_t(delta));
}

void SlotCache::count_evicted(uint32_t k) { bump(gated_of(k), &CacheStats::evicted, &LayerCounts::evicted); }

void SlotCache::stamp_room(const char* what) const {
  if (c_.scored && stamp_ > kStampLimit)
    fail(SS_E_BACKEND, std::string("device-gated: ") + what +
                           ": the scored eviction's recency stamp counter is exhausted (reopen the context)");
}

void* SlotCache::event() {
  if (pool_.empty()) {
    all_events_.push_back(m_->event_create());
    return all_events_.back();
  }
  void* ev = pool_.back();
  pool_.pop_back();
  return ev;
}

void SlotCache::set_entry(uint32_t k, int32_t v) {
  table_[k] = v;
  const uint32_t g = gated_of(k);
  dirty_lo_[g] = std::min(dirty_lo_[g], k);
  dirty_hi_[g] = std::max(dirty_hi_[g], k);
}

void SlotCache::clear_dirty() {
  std::fill(dirty_lo_.begin(), dirty_lo_.end(), kNil);
  std::fill(dirty_hi_.begin(), dirty_hi_.end(), 0u);
}

// The mirror to the device: whole, or (held layers) only each layer's changed range; the marks are cleared once the
// mover took the upload (a failed one keeps them for the next).
void SlotCache::upload() {
  if (!ranged_) {
    m_->upload_table(table_.data(), keys_);
    clear_dirty();
    device_table_known_ = false;
    return;
  }
  ranges_.clear();
  for (size_t g = 0; g < dirty_lo_.size(); ++g)
    if (dirty_lo_[g] <= dirty_hi_[g]) {
      ranges_.push_back(dirty_lo_[g]);
      ranges_.push_back(dirty_hi_[g] - dirty_lo_[g] + 1);
    }
  m_->upload_table_ranges(table_.data(), ranges_.data(), uint32_t(ranges_.size() / 2));
  if (!device_table_known_) {  // every change since the last whole upload was marked: the device now equals the mirror
    device_table_ = table_;
    device_table_known_ = true;
  } else {
    for (size_t r = 0; r < ranges_.size(); r += 2)
      std::copy_n(table_.begin() + ranges_[r], ranges_[r + 1], device_table_.begin() + ranges_[r]);
  }
  clear_dirty();
}

void SlotCache::set_range_uploads(bool on) {
  ranged_ = on;
  if (!on) device_table_known_ = false;
}

void SlotCache::publish(Mover::Stream s, uint32_t k, int32_t v) {
  set_entry(k, v);
  m_->publish(s, k, v);
}

std::vector<uint32_t> SlotCache::host_order() const {
  std::vector<uint32_t> out;
  for (uint32_t k = homes_.front(); k != kNil; k = homes_.older(k)) out.push_back(k);
  return out;
}

// ---- the open placement ----
void SlotCache::place(const std::vector<uint32_t>& order, const std::vector<uint8_t>* disk) {
  drain_pending();
  // residents: the first distinct keys of `order`, as many as leave the spare target free
  const uint32_t room = c_.persistent_slots - c_.spare_target;
  std::vector<uint8_t> resident(keys_, 0);
  std::vector<uint32_t> dev;
  for (uint32_t k : order) {
    require(k < keys_, SS_E_INVALID, "device-gated: resident key out of range");
    if (resident[k] || dev.size() >= room) continue;
    resident[k] = 1;
    dev.push_back(k);
  }
  // pinned homes: every other key, or with the file tier min(home_blocks, blocks) of them (the plan's pinned units
  // before its disk units, each group by priority: `order` first, then key order); `ranked` is their recency order
  std::vector<uint8_t> gets_block(keys_, 0);
  std::vector<uint32_t> ranked;
  if (c_.disk_tier) {
    require(!disk || disk->size() == keys_, SS_E_INVALID, "device-gated: the disk flags do not cover the keys");
    std::vector<uint32_t> by_priority;
    std::vector<uint8_t> listed(keys_, 0);
    auto list = [&](uint32_t k) {
      if (!listed[k]) by_priority.push_back(k);
      listed[k] = 1;
    };
    for (uint32_t k : order) list(k);
    for (uint32_t k = 0; k < keys_; ++k) list(k);
    const size_t cap = std::min(c_.home_blocks, c_.blocks);
    for (uint8_t want_disk : {uint8_t(0), uint8_t(1)})
      for (uint32_t k : by_priority) {
        const uint8_t is_disk = disk ? (*disk)[k] : uint8_t(0);
        if (ranked.size() >= cap) break;
        if (resident[k] || is_disk != want_disk) continue;
        gets_block[k] = 1;
        ranked.push_back(k);
      }
  } else {
    require(uint64_t(keys_) - dev.size() <= c_.blocks, SS_E_CAPACITY,
            "device-gated: fewer host blocks than non-resident units");
  }
  int32_t blocks_used = 0;
  on_file_ = 0;
  homes_.reset(keys_);
  recent_.reset(keys_);
  for (uint32_t k = 0; k < keys_; ++k) {
    Entry& x = e_[k] = Entry{};
    set_entry(k, -1);
    if (resident[k]) continue;
    if (c_.disk_tier && !gets_block[k]) {
      x.home = Home::File;
      ++on_file_;
    } else {
      x.block = blocks_used++;  // a pinned home; blocks in key order
    }
  }
  for (auto it = ranked.rbegin(); it != ranked.rend(); ++it) home_push(*it);  // ranked[0] most recently homed
  for (uint32_t i = 0; i < dev.size(); ++i) {
    e_[dev[i]].home = Home::Device;
    e_[dev[i]].slot = int32_t(i);
    table_[dev[i]] = int32_t(i);
  }
  for (auto it = dev.rbegin(); it != dev.rend(); ++it) touch(*it);  // dev[0] most recent
  on_device_ = uint32_t(dev.size());
  free_slots_.fill_down(int32_t(c_.persistent_slots), int32_t(on_device_));
  free_blocks_.fill_down(int32_t(c_.blocks), blocks_used);
  free_lands_.fill_down(int32_t(c_.landing_blocks), 0);
  land_owner_.assign(c_.landing_blocks, kNil);
  on_land_ = 0;
  open_ = OpenState{c_, e_, table_, free_slots_, free_blocks_, recent_, homes_, free_lands_, on_device_, on_file_,
                    stamp_};
}

// ---- file tier ----
// A unit that leaves the device or a bank slot without a write-back: its block (a clean copy, or the block it was
// served from) is its home again, else (file tier) its file.
void SlotCache::to_lower(uint32_t k, bool cold) {
  Entry& x = e_[k];
  x.slot = -1;
  if (x.backed) --backed_;
  x.backed = false;
  if (x.block < 0) {
    if (!c_.disk_tier) broken("a unit without a block left the device without a write-back");
    x.home = Home::File;
    ++on_file_;
    return;
  }
  x.home = Home::Host;
  home_push(k, cold, x.keep_mid);
  x.keep_mid = false;
}

// The least recently homed pinned unit (not skipped) goes to its file (no copy: the file holds its bytes); its block
// is free.
bool SlotCache::drop_host_lru(const std::vector<uint8_t>* skip, bool count) {
  if (!c_.disk_tier) return false;
  uint32_t k = homes_.back();
  for (; k != kNil && skip && (*skip)[k]; k = homes_.newer(k)) {
  }
  if (k == kNil) return false;
  Entry& x = e_[k];
  home_erase(k);
  free_blocks_.give(x.block);
  x.block = -1;
  x.home = Home::File;
  ++on_file_;
  st_.disk_drops += count ? 1 : 0;
  return true;
}

int32_t SlotCache::keep_block() {
  if (!c_.bank_keep || !c_.disk_tier || c_.no_admit) return -1;
  if (free_blocks_.empty()) {
    const uint32_t oldest = homes_.back();
    if (!drop_host_lru()) return -1;
    e_[oldest].keep_drop = st_.tokens + 1;
    ++st_.bank_keep_drops;
  }
  return free_blocks_.take();
}

// ---- landings (landing_blocks): the file tier's two-stage prefetch ----
// A landing holds exactly its key (Landing while its read runs, Landed after; its home is still its file: no slot,
// block or entry) and one landing block. A failed landing read only frees its block (advice: a demand reads the unit
// as any file miss).
bool SlotCache::advise_land(uint32_t g, uint32_t unit) {
  if (!c_.landing_blocks) return false;
  const uint32_t k = key(g, unit);
  const Home h = e_[k].home;
  if (h == Home::Landing || h == Home::Landed) return true;
  if (h != Home::File) return false;
  if (c_.landing_ttl == 0 && served_[g]) {  // its layer's demand already passed this token: it could not be used
    ++st_.landing_skipped_passed;
    return true;
  }
  land(k);
  return true;
}

bool SlotCache::land(uint32_t k) {
  reclaim_lands(false);
  if (free_lands_.empty()) {  // never displaces another landing
    ++st_.landing_dropped_full;
    return false;
  }
  const int32_t l = free_lands_.items().back();
  void* handle = nullptr;
  try {
    handle = m_->read_landing_begin(k, land_block(l));
  } catch (...) {  // nothing begun: the block stays free, the key in its file
    ++st_.landing_failed;
    return false;
  }
  free_lands_.take();
  landing_.push_back(LandRead{k, l, handle, false});
  land_owner_[size_t(l)] = k;
  Entry& x = e_[k];
  x.home = Home::Landing;
  x.land = l;
  x.land_age = 0;
  --on_file_;
  ++on_land_;
  ++st_.landing_issued;
  return true;
}

bool SlotCache::end_landing(size_t i) {
  const LandRead r = landing_[i];
  landing_.erase(landing_.begin() + std::ptrdiff_t(i));
  Mover::LandingEnd end;
  bool ok = true;
  try {
    m_->read_landing_end(r.handle, &end);
  } catch (...) {  // advice: its error is dropped (a demand's own read reports one)
    ok = false;
  }
  st_.landing_yields += end.yields;
  if (!ok) {
    ++st_.landing_failed;
    unland(r.key);
    return false;
  }
  st_.landing_read_bytes += unit_bytes_ - end.aborted_bytes;
  st_.landing_aborted_bytes += end.aborted_bytes;
  if (r.doomed || end.aborted) {  // its layer passed undemanded: never promoted, its block free
    unland(r.key);
    ++st_.landing_expired_layer;
    return false;
  }
  e_[r.key].home = Home::Landed;
  return true;
}

void SlotCache::end_landings() {
  while (!landing_.empty()) end_landing(0);
}

void SlotCache::poll_landings(size_t max) {
  for (size_t i = 0, seen = 0; i < landing_.size() && seen < max; ++seen) {
    if (m_->read_done(landing_[i].handle)) end_landing(i);
    else ++i;
  }
}

bool SlotCache::cancel_landing(size_t i) {
  Mover::LandingEnd end;
  if (!m_->read_landing_cancel(landing_[i].handle, &end)) return false;
  const uint32_t k = landing_[i].key;
  landing_.erase(landing_.begin() + std::ptrdiff_t(i));
  unland(k);
  ++st_.landing_cancelled;
  st_.landing_yields += end.yields;
  st_.landing_aborted_bytes += end.aborted_bytes;
  if (end.aborted_bytes) st_.landing_read_bytes += unit_bytes_ - end.aborted_bytes;  // (yielded part-way)
  return true;
}

void SlotCache::cancel_landings() {
  for (size_t i = 0; i < landing_.size();)
    if (!cancel_landing(i)) ++i;
}

// landing_ttl 0, layer g's demand served: a landing of layer g that it did not route cannot be used this token. A
// landed one goes back to its file now; one not running is cancelled; a running one is asked to stop and goes back
// to its file when it ends.
void SlotCache::expire_layer_landings(uint32_t g, const uint32_t* ids, uint32_t n) {
  const uint32_t first = base_[g], last = base_[g + 1];
  for (uint32_t l = 0; l < c_.landing_blocks; ++l) {
    const uint32_t k = land_owner_[l];
    if (k == kNil || k < first || k >= last || std::find(ids, ids + n, k - first) != ids + n) continue;
    if (e_[k].home == Home::Landed) {
      unland(k);
      ++st_.landing_expired_layer;
      continue;
    }
    size_t i = 0;
    while (landing_[i].key != k) ++i;
    if (!cancel_landing(i)) {
      landing_[i].doomed = true;
      m_->read_landing_abort(landing_[i].handle);
    }
  }
}

void SlotCache::unland(uint32_t k) {
  Entry& x = e_[k];
  free_lands_.give(x.land);
  land_owner_[size_t(x.land)] = kNil;
  x.land = -1;
  x.land_age = 0;
  x.home = Home::File;
  --on_land_;
  ++on_file_;
}

void SlotCache::reclaim_lands(bool synced) {
  size_t kept = 0;
  for (const LandBusy& b : land_busy_) {
    if (synced || m_->done(b.ev)) {
      free_lands_.give(b.land);
      pool_.push_back(b.ev);
    } else {
      land_busy_[kept++] = b;
    }
  }
  land_busy_.resize(kept);
}

// The next staging buffer in rotation, once a read still holding it ended and its last copy landed.
int32_t SlotCache::take_stage() {
  const uint32_t i = stage_next_;
  stage_next_ = (stage_next_ + 1) % c_.disk_staging;
  const int32_t stage = int32_t(c_.blocks + i);
  end_reads([stage](const Pending& p) { return p.stage == stage; });
  if (stage_ev_[i] != nullptr && !m_->done(stage_ev_[i])) {
    m_->event_sync(stage_ev_[i]);
    ++st_.disk_stage_waits;
  }
  return stage;
}

// ---- file reads in flight (disk_queue > 1) ----
// A file miss's fetch takes its slot and staging buffer and changes every host record at once (homes, the table
// mirror, lists, counters); only the device work that needs the bytes waits for the read's end: its copy, its entry,
// the staging buffer's event and a prefetch's event. Reads end at drain points: the demand reads at every public entry
// point, a key's read when the key is touched again, the reads a layer routes before its ready, a staging buffer's read
// before its reuse, the oldest when the queue is full, every read at the boundary and at any setting.
void SlotCache::enter() {
  ++entries_;
  drain_demand();
}

void SlotCache::drain_pending(size_t n) {
  size_t left = n;
  end_reads([&left](const Pending&) { return left != 0 && left-- != 0; });
}

void SlotCache::drain_demand() {
  end_reads([](const Pending& p) { return !p.prefetch; });
}

void SlotCache::drain_key(uint32_t k) {
  end_reads([k](const Pending& p) { return p.key == k; });
}

// The demand reads, and the prefetch reads of units layer g routes (a wrong prediction's read keeps running).
void SlotCache::drain_layer(uint32_t g, const uint32_t* ids, uint32_t n) {
  const uint32_t first = key(g, 0);
  end_reads([&](const Pending& p) {
    if (!p.prefetch) return true;
    return gated_of(p.key) == g && std::find(ids, ids + n, p.key - first) != ids + n;
  });
}

// The picked records leave pending_ (the others keep their order) and end oldest first. A read that failed is undone
// (its key back in its file, its slot back); after a failed copy every record left is undone and nothing more is
// enqueued. The first failure is rethrown.
void SlotCache::end_reads(const std::function<bool(const Pending&)>& pick) {
  if (pending_.empty()) return;
  std::vector<Pending> ending, staying;
  for (const Pending& p : pending_) (pick(p) ? ending : staying).push_back(p);
  pending_.swap(staying);
  std::exception_ptr failure;
  bool device_down = false;
  for (size_t i = 0; i < ending.size(); ++i) {
    const Pending p = ending[i];
    if (p.entry != entries_) {  // it ran on while its fetch's caller went on
      ++st_.disk_carried;
      st_.disk_carried_bytes += unit_bytes_;
    }
    const auto t0 = Clock::now();
    bool landed = true;
    try {
      st_.disk_read_ns += m_->read_end(p.handle);
    } catch (...) {
      landed = false;
      if (!failure) failure = std::current_exception();
    }
    st_.disk_wait_ns += ns_since(t0);
    if (!landed || device_down) {
      undo_pending(p);
      continue;
    }
    ++st_.disk_reads;
    st_.disk_read_bytes += unit_bytes_;
    try {
      finish_pending(p);
    } catch (...) {
      if (!failure) failure = std::current_exception();
      device_down = true;  // (this record stays fetched, as a synchronous fetch whose copy failed)
      ending.insert(ending.end(), pending_.begin(), pending_.end());
      pending_.clear();
    }
  }
  if (failure) std::rethrow_exception(failure);
}

// An ended read's device work: the copy from its staging buffer and the entry, the buffer's event, a prefetch's event.
void SlotCache::finish_pending(const Pending& p) {
  if (mut_ == kEntryBeforeCopy) publish(p.s, p.key, p.slot);  // test-only fault: the entry before its bytes
  m_->h2d(p.s, p.slot, p.stage, p.key);
  if (mut_ != kEntryBeforeCopy) publish(p.s, p.key, p.slot);
  if (uint32_t(p.stage) >= c_.blocks) {  // (a kept read's block is its key's own, not a staging buffer)
    void*& stage_ev = stage_ev_[uint32_t(p.stage) - c_.blocks];  // the buffer is reusable once this copy landed
    if (stage_ev == nullptr) stage_ev = event();
    m_->record(stage_ev, p.s);
  }
  if (!p.prefetch) return;
  Entry& x = e_[p.key];
  x.pf_done = event();
  m_->record(x.pf_done, p.s);
}

// A read that failed: the key goes back to its file, its slot to where it came from (a bank slot stays used for the
// layer, unpublished); nothing was enqueued for it.
void SlotCache::undo_pending(const Pending& p) {
  Entry& x = e_[p.key];
  const uint32_t g = gated_of(p.key);
  if (p.bank) {
    set_entry(p.key, -1);
    bank_key_[size_t(p.slot) - bank_first_] = kNil;
    banked_.erase(std::find(banked_.begin(), banked_.end(), p.key));
    --st_.bank_serves;
    --lc_[g].bank_serves;
    if (x.block >= 0) {  // a kept read's block: never a home, free again
      free_blocks_.give(x.block);
      x.block = -1;
      x.keep_mid = false;
      --st_.bank_kept;
    }
  } else {
    leave_device(p.key);
    coming_.erase(std::find(coming_.begin(), coming_.end(), p.key));
    free_slots_.give(p.slot);
    demand_free_used_ -= p.free_counted ? 1 : 0;
  }
  x.home = Home::File;
  x.slot = -1;
  x.via_pf = x.used = false;
  ++on_file_;
  count_fetch(g, p.prefetch, -1);
}

// A file miss with the queue full: the completed reads end, then the oldest demand reads, then the oldest.
void SlotCache::make_room_for_read() {
  const size_t depth = std::max<uint32_t>(c_.disk_queue, 1);
  if (pending_.size() < depth) return;
  end_reads([this](const Pending& p) { return m_->read_done(p.handle); });
  if (pending_.size() >= depth) {
    size_t over = pending_.size() + 1 - depth;
    end_reads([&over](const Pending& p) { return !p.prefetch && over != 0 && over-- != 0; });
  }
  if (pending_.size() >= depth) drain_pending(pending_.size() + 1 - depth);
}

// ---- write-backs ----
// Finished write-backs in submission order: the unit's home becomes its block and its slot is free; a discarded one
// (the unit was resurrected) only returns its block.
uint32_t SlotCache::collect() {
  uint32_t done = 0;
  for (; !wbs_.empty() && m_->done(wbs_.front().done); ++done) {
    Writeback w = wbs_.front();
    wbs_.pop_front();
    Entry& x = e_[w.key];
    x.wb_pending = false;
    if (w.discard) {
      free_blocks_.give(w.block);
    } else {
      x.home = Home::Host;
      x.block = w.block;
      x.slot = -1;
      home_push(w.key);
      free_slots_.give(w.slot);
    }
    outstanding_ -= w.bytes;
    st_.wb_completed_bytes += w.bytes;
    recycle(w.done);
  }
  st_.writebacks_done += done;
  return done;
}

void SlotCache::submit_part(Deferred& d) {
  const uint32_t p = d.parts_done;
  m_->d2h(wb_stream_, d.slot, d.block, int32_t(p), d.key);
  d.parts_done = p + 1;
  const uint64_t n = m_->part_bytes(p);
  d.bytes += n;
  outstanding_ += n;
  st_.wb_issued_bytes += n;
}

// The deferred front, as far as it was submitted, becomes a write-back in flight (its completion event recorded).
void* SlotCache::record_front(bool discard) {
  const Deferred& d = deferred_.front();
  void* ev = event();
  m_->record(ev, wb_stream_);
  wbs_.push_back(Writeback{d.key, d.slot, d.block, ev, discard, d.bytes});
  deferred_.pop_front();
  return ev;
}

void* SlotCache::finish_front() {
  for (Deferred& d = deferred_.front(); d.parts_done < m_->parts();) submit_part(d);
  return record_front(false);
}

// After layer g was served: the deferred write-backs' parts, within the layer's byte credit and the outstanding cap,
// unless a later layer was already exported (ahead), never behind the last layer (the boundary's sync would wait).
void SlotCache::issue_writebacks(uint32_t g, const std::function<bool()>& ahead) {
  enter();
  if (deferred_.empty()) {
    credit_ = 0;
    return;
  }
  if (g + 1 >= gated()) return;
  const int64_t grant = int64_t(layer_bytes_);
  credit_ = std::min(credit_ + grant, grant);  // a debt carries over, unused credit does not
  st_.collected_mid += collect();
  bool fenced = false;  // the write-back stream waits for this layer's ready (once)
  while (credit_ > 0 && !deferred_.empty() && outstanding_ < max_outstanding_) {
    if (ahead && ahead()) break;
    if (wb_stream_ == Mover::kD2h && !fenced) {
      m_->record(post_ready_ev_, Mover::kDem);
      m_->wait(Mover::kD2h, post_ready_ev_);
      fenced = true;
    }
    Deferred& d = deferred_.front();
    credit_ -= int64_t(m_->part_bytes(d.parts_done));
    if (d.parts_done + 1 < m_->parts()) submit_part(d);
    else finish_front();
  }
}

// A demand with no free slot while write-backs are deferred: wait for the oldest live write-back in flight (or finish
// the deferred front and wait for it) until a slot is free.
void SlotCache::force_free_slot() {
  while (free_slots_.empty() && !deferred_.empty()) {
    const auto live = std::find_if(wbs_.begin(), wbs_.end(), [](const Writeback& w) { return !w.discard; });
    void* ev = live != wbs_.end() ? live->done : finish_front();
    ++st_.wb_forced;
    const auto t0 = Clock::now();
    m_->event_sync(ev);
    st_.wb_forced_wait_ns += ns_since(t0);
    st_.collected_mid += collect();
  }
}

// Between tokens: every copy settled and every write-back collected (the round, make-resident and reset need it).
void SlotCache::settle_writebacks(const char* what) {
  drain();
  for (const Writeback& w : wbs_) m_->event_sync(w.done);
  collect();
  if (!wbs_.empty()) broken(std::string(what) + ": write-backs not collected");
}

// ---- banks ----
// Bank g & 1 of the demand bank slots; a bank is reused two gated layers later, when the device has finished the
// layer that used it before. The slot's previous unit goes back to its block and its entry is withdrawn first.
int32_t SlotCache::bank_slot(uint32_t g) {
  const uint32_t b = g & 1u;
  if (bank_seq_[b] != seq_ || bank_layer_[b] != g) {  // the bank's first use by this layer this token
    bank_seq_[b] = seq_;
    bank_layer_[b] = g;
    bank_next_[b] = 0;
  }
  if (bank_next_[b] >= c_.bank_slots) return -1;
  const uint32_t at = b * c_.bank_slots + bank_next_[b]++;
  const int32_t slot = int32_t(bank_first_ + at);
  const uint32_t prior = bank_key_[at];
  if (prior != kNil && e_[prior].home == Home::Bank && e_[prior].slot == slot) {
    drain_key(prior);  // (its read, were it still in flight, ends before the alias goes)
    to_lower(prior);   // its block, or (read from it) its file
    publish(Mover::kDem, prior, -1);
  }
  bank_key_[at] = kNil;
  return slot;
}

// ---- a token ----
void SlotCache::begin_token(uint32_t seq, const std::vector<uint8_t>* run) {
  require(!run || run->size() == gated(), SS_E_INVALID, "device-gated: the exported layers do not cover the gated layers");
  enter();
  if (run) run_ = *run;
  else std::fill(run_.begin(), run_.end(), uint8_t(1));
  if (c_.scored) {  // the token's epoch (the first is 1); one token cannot push more than 2^40 stamps
    stamp_room("begin_token");
    require(epoch_ < (uint64_t(1) << 63), SS_E_BACKEND, "device-gated: the scored eviction's epoch counter is exhausted");
    ++epoch_;
  }
  seq_ = seq;
  pf_token_ = demand_free_used_ = 0;
  std::fill(pf_layer_.begin(), pf_layer_.end(), 0u);
  std::fill(layer_missed_.begin(), layer_missed_.end(), uint8_t(0));
  std::fill(served_.begin(), served_.end(), uint8_t(0));
  pred_.clear();
  pred_layer_ = kNil;
}

// An Evicting unit routed again: its slot still holds the bytes (a write-back only reads them). A deferred write-back
// not yet begun is cancelled (its block free again); one partly submitted (only the front can be) or in flight is
// kept as a discard. The unit is a device home again.
bool SlotCache::resurrect(uint32_t k) {
  Entry& x = e_[k];
  const auto d = std::find_if(deferred_.begin(), deferred_.end(), [k](const Deferred& v) { return v.key == k; });
  if (d != deferred_.end() && d->parts_done == 0) {
    free_blocks_.give(d->block);
    deferred_.erase(d);
    x.wb_pending = false;
    ++st_.wb_cancelled;
    st_.wb_cancelled_bytes += unit_bytes_;
  } else if (d != deferred_.end()) {
    if (d != deferred_.begin()) broken("parts submitted behind the deferred front");
    st_.wb_cancelled_bytes += unit_bytes_ - d->bytes;
    record_front(true);
  } else {
    const auto w = std::find_if(wbs_.begin(), wbs_.end(), [k](const Writeback& v) { return v.key == k && !v.discard; });
    if (w != wbs_.end()) w->discard = true;
  }
  x.home = Home::Device;
  x.block = -1;
  publish(Mover::kDem, k, x.slot);
  touch(k);
  ++on_device_;
  ++st_.resurrected;
  return true;
}

bool SlotCache::fetch(uint32_t g, uint32_t unit, bool prefetch) {
  const uint32_t k = key(g, unit);
  Entry& x = e_[k];
  if (x.home == Home::Landing || x.home == Home::Landed) {
    if (prefetch) return false;  // a landing is promoted by a demand only
    if (x.home == Home::Landing) {  // its read ends now, out of order (failed: a file miss below, as any)
      size_t i = 0;
      while (landing_[i].key != k) ++i;
      const bool late = !m_->read_done(landing_[i].handle);
      const auto t0 = Clock::now();
      const bool ok = end_landing(i);
      if (late) {
        st_.landing_wait_ns += ns_since(t0);
        st_.landing_late += ok ? 1 : 0;
      }
    }
  }
  if (prefetch && (c_.no_admit || pf_layer_[g] >= c_.prefetch_per_layer || pf_token_ >= c_.prefetch_per_token))
    return false;
  if (x.home == Home::Coming) {
    drain_key(k);  // (its own prefetch read in flight: ended)
    return false;
  }
  if (x.home == Home::Device || x.home == Home::Bank) return false;
  if (x.home == Home::Evicting) return resurrect(k);
  if (x.home == Home::File && prefetch && !c_.disk_prefetch) return false;  // a file prefetch only with disk_prefetch
  // where the unit goes: a free slot (a prefetch leaves the reserve free, pf_strict the spare target's slots too), else
  // for a demand its layer's bank slot (no_admit: always)
  const size_t reserve =
      !prefetch ? 0u : c_.pf_strict ? std::max<size_t>(c_.prefetch_reserve, c_.spare_target) : c_.prefetch_reserve;
  int32_t slot = -1;
  bool bank = false, free_counted = false;
  if (c_.no_admit) {  // a demand: its layer's bank slot, released at the boundary, its home unchanged
    slot = bank_slot(g);
    if (slot < 0)
      fail(SS_E_BACKEND, "device-gated: dg_no_admit: no bank slot for a miss of gated layer " + std::to_string(g) +
                             " (more distinct misses than dg_max_ids)");
    bank = true;
  } else if (free_slots_.size() <= reserve || (pressure_ && !prefetch)) {
    st_.collected_mid += collect();
  }
  const bool capped = !prefetch && pressure_ && demand_free_used_ >= pressure_free_;
  if (!bank && !prefetch && !capped && free_slots_.empty()) force_free_slot();
  if (!bank) {
    if (!capped && free_slots_.size() > reserve) {
      free_counted = !prefetch;
      demand_free_used_ += free_counted ? 1 : 0;
      slot = free_slots_.take();
    } else if (prefetch) {
      if (c_.pf_strict && free_slots_.size() > c_.prefetch_reserve) ++st_.pf_strict_refused;
      return false;
    } else if ((slot = bank_slot(g)) >= 0) {
      bank = true;
    } else {  // more distinct misses than a bank holds: only an internal error gets here
      drain_pending();
      force_free_slot();
      for (; free_slots_.empty() && !wbs_.empty(); ++st_.stalled) {
        m_->event_sync(wbs_.front().done);
        collect();
      }
      if (free_slots_.empty()) fail(SS_E_BACKEND, "device-gated: no free slot, no bank slot, no write-back to wait for");
      slot = free_slots_.take();
    }
  }
  const Mover::Stream s = prefetch ? Mover::kPf : Mover::kDem;
  const bool from_file = x.home == Home::File;
  if (from_file) {  // its bytes from the file into a staging buffer, then the same copy once the read ended
    int32_t stage = -1;
    try {
      make_room_for_read();
      stage = bank ? keep_block() : -1;  // bank_keep: into the pinned block that becomes its home
      if (stage < 0) stage = take_stage();
      const auto t0 = Clock::now();
      void* handle = m_->read_begin(k, stage);
      st_.disk_read_ns += ns_since(t0);
      st_.disk_overlapped += pending_.empty() ? 0 : 1;
      pending_.push_back(Pending{k, slot, stage, s, prefetch, bank, free_counted, handle, entries_});
      st_.disk_max_in_flight = std::max<uint64_t>(st_.disk_max_in_flight, pending_.size());
    } catch (...) {  // nothing begun for this key: its slot goes back (a bank slot stays used, unpublished)
      if (!bank) {
        free_slots_.give(slot);
        demand_free_used_ -= free_counted ? 1 : 0;
      }
      if (stage >= 0 && uint32_t(stage) < c_.blocks) free_blocks_.give(stage);  // (a kept read's block)
      throw;
    }
    if (uint32_t(stage) < c_.blocks) {  // kept: the block is the unit's own, its home once the bank lets it go
      x.block = stage;
      x.keep_mid = c_.bank_keep == 2;
      ++st_.bank_kept;
    }
    set_entry(k, slot);  // the mirror now; the device's entry with the copy
    --on_file_;
    if (x.keep_drop) {  // dropped to its file for a kept read: read back within 8 tokens counts as churn
      st_.bank_keep_rereads += st_.tokens + 1 - x.keep_drop <= 8 ? 1 : 0;
      x.keep_drop = 0;
    }
  } else if (x.home == Home::Landed) {  // from its landing block, free again once this copy's event completed
    if (mut_ == kEntryBeforeCopy) publish(s, k, slot);
    m_->h2d(s, slot, land_block(x.land), k);
    if (mut_ != kEntryBeforeCopy) publish(s, k, slot);
    void* ev = event();
    m_->record(ev, s);
    land_busy_.push_back(LandBusy{x.land, ev});
    land_owner_[size_t(x.land)] = kNil;
    x.land = -1;
    x.land_age = 0;
    --on_land_;
    ++st_.landing_promoted;
  } else {
    if (mut_ == kEntryBeforeCopy) publish(s, k, slot);  // test-only fault: the entry before its bytes
    m_->h2d(s, slot, x.block, k);
    if (mut_ != kEntryBeforeCopy) publish(s, k, slot);
    home_erase(k);  // (a Host unit: out of the pinned recency list)
  }
  x.slot = slot;
  x.via_pf = prefetch;
  x.used = false;
  if (prefetch && !from_file) {  // (a file read's event comes with its copy)
    x.pf_done = event();
    m_->record(x.pf_done, s);
  }
  if (bank) {
    x.home = Home::Bank;
    bank_key_[size_t(slot) - bank_first_] = k;
    banked_.push_back(k);
    bump(g, &CacheStats::bank_serves, &LayerCounts::bank_serves);
  } else {
    x.home = Home::Coming;
    coming_.push_back(k);
    touch(k);
    ++on_device_;
  }
  count_fetch(g, prefetch);
  if (prefetch) {
    ++pf_layer_[g];
    ++pf_token_;
  }
  if (from_file && c_.disk_queue <= 1) drain_pending();  // synchronous reads: the copy now
  return true;
}

void SlotCache::cover(uint32_t g, uint32_t unit) {
  const uint32_t k = key(g, unit);
  Entry& x = e_[k];
  if (mut_ == kNoCover || x.home != Home::Coming || !x.via_pf) return;
  // only this key's copy lands before the ready: its read ends first if in flight (a file prefetch's event comes with
  // its copy), the wait is on its own event
  drain_key(k);
  if (x.home == Home::Coming && x.via_pf && x.pf_done) {
    m_->wait(Mover::kDem, x.pf_done);
    ++st_.covered_waits;
  }
}

void SlotCache::use(uint32_t g, uint32_t unit, bool was_miss) {
  enter();
  const uint32_t k = key(g, unit);
  Entry& x = e_[k];
  bump(g, &CacheStats::lookups, &LayerCounts::lookups);
  if (was_miss) {
    bump(g, &CacheStats::misses, &LayerCounts::misses);
    if (!layer_missed_[g]) ++st_.miss_layers;  // (the layer's first miss this token)
    layer_missed_[g] = 1;
  }
  if (c_.scored) x.demand_epoch = epoch_;  // a routed use (never a prefetch, a resurrection or a seed)
  if (x.via_pf && !x.used) {
    x.used = true;
    bump(g, &CacheStats::prefetch_used, &LayerCounts::prefetch_used);
  }
  if (recent_.has(k)) touch(k);
}

void SlotCache::serve_demand(uint32_t g, const uint32_t* ids, uint32_t n, uint64_t mask) {
  enter();
  const uint32_t nu = units(g);
  for (uint32_t i = 0; i < n; ++i)
    require(ids[i] < nu, SS_E_INVALID,
            "device-gated: layer " + std::to_string(g) + " exported id " + std::to_string(ids[i]) + " of " +
                std::to_string(nu));
  if (mask) m_->diag_mark(g, 0);
  // masked occurrences in export order: a repeated id is fetched at its first occurrence, covered at the others; a
  // miss whose landing read still runs is fetched after the layer's other misses (their reads start first)
  late_.clear();
  uint64_t late_covered = 0;
  poll_landings();  // (a landing read that completed is landed: only a running one is late)
  for (uint32_t i = 0; i < n; ++i) {
    if (!((mask >> i) & 1u)) continue;
    const Home h = e_[key(g, ids[i])].home;
    if (h == Home::Device || h == Home::Coming || h == Home::Bank) {
      cover(g, ids[i]);
      ++st_.covered;
    } else if (c_.landing_blocks && h == Home::Landing) {
      if (std::find(late_.begin(), late_.end(), ids[i]) != late_.end()) ++late_covered;
      else late_.push_back(ids[i]);
    } else {
      fetch(g, ids[i], false);
    }
  }
  for (uint32_t id : late_) fetch(g, id, false);
  st_.covered += late_covered;  // (a repeated late miss: covered at its later occurrences)
  if (c_.landing_blocks && c_.landing_ttl == 0) {
    served_[g] = 1;
    expire_layer_landings(g, ids, n);
  }
  drain_layer(g, ids, n);  // this layer's copies and entries (its demand reads, the prefetch reads it routes)
  if (!mask) return;
  drain_demand();  // (the ready follows every demand read's copy and entry)
  m_->ready(g, seq_);
  m_->diag_mark(g, 1);
}

void SlotCache::serve_use(uint32_t g, const uint32_t* ids, uint32_t n, uint64_t mask) {
  enter();
  const bool predicted = pred_layer_ == g;
  uniq_.assign(ids, ids + n);
  std::sort(uniq_.begin(), uniq_.end());
  uniq_.erase(std::unique(uniq_.begin(), uniq_.end()), uniq_.end());
  if (c_.scored) score_history(g);  // (the union saved before a prediction reuses uniq_)
  for (uint32_t id : uniq_) {  // placement rounds: the tokens that routed the unit since the last round
    uint32_t& hits = rhits_[key(g, id)];
    hits += hits != UINT32_MAX ? 1 : 0;
  }
  for (uint32_t id : uniq_) {
    bool missed = false;
    for (uint32_t i = 0; i < n && !missed; ++i) missed = ids[i] == id && ((mask >> i) & 1u);
    use(g, id, missed);
    if (predicted && std::find(pred_.begin(), pred_.end(), id) != pred_.end()) ++st_.predicted_true;
  }
  pred_.clear();
  pred_layer_ = kNil;
}

// The prediction for layer g_next: deduplicated in order, invalid ids dropped; each one a budgeted prefetch. The
// device running ahead does not skip it (the reference's default prediction admission).
void SlotCache::serve_prediction(uint32_t g_next, const uint32_t* pred, uint32_t n, bool ahead) {
  (void)ahead;
  enter();  // (its prefetches' file reads stay in flight past the call)
  if (g_next >= gated()) return;
  const uint32_t nu = units(g_next);
  uniq_.clear();
  for (uint32_t i = 0; i < n; ++i) {
    if (pred[i] >= nu) ++st_.pred_invalid;
    else if (std::find(uniq_.begin(), uniq_.end(), pred[i]) == uniq_.end()) uniq_.push_back(pred[i]);
  }
  st_.predicted += uniq_.size();
  pred_ = uniq_;
  pred_layer_ = g_next;
  for (uint32_t id : pred_)
    if (!advise_land(g_next, id)) fetch(g_next, id, true);  // (landings on: a file-homed unit lands instead)
}

// ---- the boundary ----
void SlotCache::end_token(const std::vector<uint32_t>& keep, uint32_t rows) {
  drain_pending();  // the end of the token: no read in flight while its streams sync and victims are chosen
  m_->sync(Mover::kDem);
  m_->sync(Mover::kPf);
  if (c_.landing_blocks) {
    // the landing reads not running are dropped, the running ones end (landed, or back to their file); every landing
    // block a promotion's copy read is free (the streams synced); a landing not demanded for landing_ttl boundaries
    // (TTL 0: one) goes back to its file, with no copy
    cancel_landings();
    end_landings();
    reclaim_lands(true);
    for (uint32_t l = 0; l < c_.landing_blocks; ++l) {
      const uint32_t k = land_owner_[l];
      if (k == kNil || ++e_[k].land_age < std::max<uint32_t>(c_.landing_ttl, 1)) continue;
      unland(k);
      ++st_.landing_expired;
    }
  }
  std::vector<uint8_t> held;
  if (!keep.empty()) {
    held.assign(keys_, 0);
    for (uint32_t k : keep)
      if (k < keys_) held[k] = 1;
  }
  auto is_held = [&held](uint32_t k) { return !held.empty() && held[k]; };
  // (1) the token's arrivals become device homes, their source blocks free (or kept as the inclusive share's clean
  // copies); pf_revert: an unused prefetch goes back to its source block at the pinned recency tail (or, read from it,
  // its file), its slot free, its entry withdrawn by the upload below
  for (uint32_t k : coming_) {
    Entry& x = e_[k];
    if (x.home != Home::Coming) continue;
    recycle(x.pf_done);
    if (c_.pf_revert && x.via_pf && !x.used && !is_held(k)) {
      ++st_.pf_reverted;
      st_.pf_revert_bytes += unit_bytes_;
      free_slots_.give(x.slot);
      to_lower(k, true);
      leave_device(k);
      x.via_pf = false;
      continue;
    }
    x.home = Home::Device;
    x.via_pf = false;
    if (x.block < 0) continue;  // (read from its file: no block)
    if (backed_ < c_.inclusive) {
      x.backed = true;
      ++backed_;
      ++st_.inclusive_kept;
    } else {
      free_blocks_.give(x.block);
      x.block = -1;
    }
  }
  coming_.clear();
  std::fill(served_.begin(), served_.end(), uint8_t(0));
  // (2) bank units go back to their blocks (or, read from it, their file)
  for (uint32_t k : banked_) {
    Entry& x = e_[k];
    if (x.home == Home::Bank) {
      to_lower(k);
      set_entry(k, -1);
    }
    recycle(x.pf_done);
    x.via_pf = false;
  }
  banked_.clear();
  std::fill(bank_key_.begin(), bank_key_.end(), kNil);
  bank_seq_[0] = bank_seq_[1] = 0;
  bank_layer_[0] = bank_layer_[1] = kNil;
  // (3) victims until free slots + write-backs still to free one reach the spare target
  collect();
  size_t freeing = deferred_.size();
  for (const Writeback& w : wbs_) freeing += w.discard ? 0u : 1u;
  const size_t have = free_slots_.size() + freeing;
  victims_.clear();
  size_t taken = 0;
  bool out_of_blocks = false;
  auto eligible = [&](uint32_t k) {
    const Entry& x = e_[k];
    return x.home == Home::Device && !x.wb_pending && !is_held(k);
  };
  // A victim leaves without a copy when its block holds a clean copy, when clean_evict drops it to its file, or (file
  // tier) when no block can be freed by dropping a pinned unit to its file; else it takes a free block and its
  // write-back is issued below. No block at all: the boundary stops short.
  auto evict = [&](uint32_t k) {
    Entry& x = e_[k];
    const bool clean = !x.backed && clean_now();
    const bool no_copy =
        x.backed || clean || (free_blocks_.empty() && !drop_host_lru() && c_.disk_tier);
    if (!no_copy && free_blocks_.empty()) {
      ++st_.evict_short;
      out_of_blocks = true;
      return false;
    }
    ++taken;
    if (no_copy) {
      ++(x.backed ? st_.inclusive_drops : st_.disk_discards);
      if (clean) count_clean();
      free_slots_.give(x.slot);
      leave_device(k);
      to_lower(k);
      count_evicted(k);
      return true;
    }
    x.block = free_blocks_.take();
    leave_device(k);
    x.home = Home::Evicting;
    x.wb_pending = true;
    victims_.push_back(k);
    return true;
  };
  // scored eviction: the lowest scores among the eligible units, when every gated layer was closed this token (a layer
  // the token did not export is closed here from its unchanged history); else the recency tail
  const bool selecting = !c_.no_admit;  // (no_admit: nothing was admitted, no boundary evicts)
  const bool want_score = selecting && c_.scored && (!c_.scored_auto || rows > 1);
  if (c_.scored)
    for (uint32_t g = 0; g < gated(); ++g)
      if (!run_[g]) sc_[g].list_epoch = epoch_;
  const bool by_score =
      want_score && std::all_of(sc_.begin(), sc_.end(), [this](const LayerScore& h) { return h.list_epoch == epoch_; });
  if (want_score && !by_score) ++st_.score_fallbacks;
  if (by_score) {
    const auto t0 = Clock::now();
    select_scored(c_.spare_target > have ? c_.spare_target - have : 0, eligible);
    for (const ScoreCand& cd : select_heap_) {
      if (!evict(cd.key)) break;
      ++st_.scored_victims;
    }
    st_.score_ns += ns_since(t0);
  } else if (selecting) {
    for (uint32_t k = recent_.back(); k != kNil && have + taken < c_.spare_target;) {
      const uint32_t newer = recent_.newer(k);  // (k may leave the list)
      if (eligible(k) && !evict(k)) break;
      k = newer;
    }
  }
  if (selecting && pressure_ && pressure_recent_ && !out_of_blocks) {  // test pressure: the most recent ones too
    uint32_t n = 0;
    for (uint32_t k = recent_.front(); k != kNil && n < pressure_recent_;) {
      const uint32_t older = recent_.older(k);
      if (eligible(k)) {
        if (!evict(k)) break;
        ++n;
      }
      k = older;
    }
  }
  // (4) the table, then the write-backs behind it: deferred ones carried by the larger of this and the last boundary's
  // evictions (the older ones flushed now), or issued at once on the write-back stream
  const size_t n_evict = victims_.size();
  upload();
  const size_t carry = std::max(n_evict, prev_evict_);
  const size_t n_flush = deferred_.size() > carry ? deferred_.size() - carry : 0;
  prev_evict_ = n_evict;
  credit_ = 0;
  if (c_.wb_defer)
    for (uint32_t k : victims_) {
      deferred_.push_back(Deferred{k, e_[k].slot, e_[k].block, 0, 0});
      ++st_.wb_deferred;
      count_evicted(k);
    }
  const uint64_t issued_before = st_.wb_issued_bytes;
  for (size_t i = 0; i < n_flush; ++i) finish_front();
  st_.wb_boundary_flushed += n_flush;
  st_.wb_boundary_flushed_bytes += st_.wb_issued_bytes - issued_before;
  if (!c_.wb_defer)
    for (uint32_t k : victims_) {
      const Entry& x = e_[k];
      m_->d2h(Mover::kD2h, x.slot, x.block, -1, k);
      void* ev = event();
      m_->record(ev, Mover::kD2h);
      wbs_.push_back(Writeback{k, x.slot, x.block, ev, false, unit_bytes_});
      outstanding_ += unit_bytes_;
      st_.wb_issued_bytes += unit_bytes_;
      count_evicted(k);
    }
  ++st_.tokens;
}

// ---- scored eviction ----
// Layer g's union of this token (uniq_, sorted) against the previous token's: every (r in the previous union, e in this
// one) cell takes one saturating increment and its row sum with it; the union enters the window ring (the oldest
// leaves once 16 are held) and becomes the previous one.
void SlotCache::score_history(uint32_t g) {
  LayerScore& h = sc_[g];
  const uint32_t n = units(g);
  require(uniq_.size() <= c_.max_ids, SS_E_BACKEND, "device-gated: a score union above max ids");
  h.cur = uniq_;
  h.served = epoch_;
  for (uint32_t r : h.prev) {
    uint32_t* row = &h.T[size_t(r) * n];
    for (uint32_t e : h.cur) {
      if (row[e] == UINT32_MAX) {
        ++st_.score_saturated;
      } else {
        row[e] += 1;
        h.rowsum[r] += 1;
      }
    }
  }
  const size_t width = c_.max_ids;
  if (h.ring_n == kWindow) {  // the oldest union leaves the window
    for (uint32_t i = 0; i < h.ring_len[h.ring_head]; ++i) h.cnt[h.ring[h.ring_head * width + i]] -= 1;
    h.ring_head = (h.ring_head + 1) % kWindow;
    h.ring_n -= 1;
  }
  const uint32_t at = (h.ring_head + h.ring_n++) % kWindow;
  std::copy(h.cur.begin(), h.cur.end(), h.ring.begin() + std::ptrdiff_t(at * width));
  h.ring_len[at] = uint8_t(h.cur.size());
  for (uint32_t e : h.cur) h.cnt[e] += 1;
  h.prev = h.cur;
}

void SlotCache::score_layer(uint32_t g) {
  enter();
  if (c_.scored && g < gated() && sc_[g].served == epoch_) sc_[g].list_epoch = epoch_;  // (not served: fall back)
}

// Unit u of layer g with cur = this token's union: N = sum over r in cur of T[r][u], D = sum over cur of the row
// sums, P = ((|cur| N) << 16) / max(1, D), F = (cnt[u] << 16) / 16, Rec = (1 << 16) / (1 + epoch - demand_epoch),
// S = w_t P + w_f F + w_r Rec in unsigned floor arithmetic (N <= D, so P <= |cur| << 16 and S < 2^33). With a cutoff
// that F and Rec alone cannot beat, the transition rows are not read.
SlotCache::ScoreCand SlotCache::score_candidate(uint32_t g, uint32_t u, uint64_t D, const ScoreCand* cutoff) const {
  const LayerScore& h = sc_[g];
  const uint32_t k = base_[g] + u;
  const Entry& x = e_[k];
  const uint64_t freq = (uint64_t(h.cnt[u]) << 16) / kWindow;
  const uint64_t rec = (uint64_t(1) << 16) / (1 + (epoch_ - x.demand_epoch));
  ScoreCand cd{uint64_t(c_.w_freq) * freq + uint64_t(c_.w_rec) * rec, x.demand_epoch, x.lru_stamp, k};
  if (cutoff != nullptr && !cand_less(cd, *cutoff)) return cd;
  uint64_t hits = 0;
  const size_t n = units(g);
  for (uint32_t r : h.cur) hits += h.T[r * n + u];
  cd.s += uint64_t(c_.w_trans) * (((uint64_t(h.cur.size()) * hits) << 16) / std::max<uint64_t>(D, 1));
  return cd;
}

// The `need` lowest candidates (cand_less) of every gated layer's eligible units, ascending in select_heap_: a bounded
// max-heap over all layers, scored from each layer's current union, epochs and stamps.
void SlotCache::select_scored(size_t need, const std::function<bool(uint32_t)>& eligible, bool count) {
  select_heap_.clear();
  auto& heap = select_heap_;
  for (uint32_t g = 0; need != 0 && g < gated(); ++g) {
    uint64_t denom = 0;
    for (uint32_t r : sc_[g].cur) denom += sc_[g].rowsum[r];
    st_.score_layers += count ? 1 : 0;
    for (uint32_t u = 0; u < units(g); ++u) {
      if (!eligible(base_[g] + u)) continue;
      st_.score_candidates += count ? 1 : 0;
      const bool full = heap.size() == need;
      const ScoreCand cd = score_candidate(g, u, denom, full ? &heap.front() : nullptr);
      if (!full) {
        heap.push_back(cd);
        std::push_heap(heap.begin(), heap.end(), cand_less);
      } else if (cand_less(cd, heap.front())) {  // the worst kept one leaves
        std::pop_heap(heap.begin(), heap.end(), cand_less);
        heap.back() = cd;
        std::push_heap(heap.begin(), heap.end(), cand_less);
      }
    }
  }
  std::sort_heap(heap.begin(), heap.end(), cand_less);
}

// The open state of every score table: the profile's counts (or zeros), an empty window, no union, epoch 0, the
// open's stamps.
void SlotCache::reset_score() {
  for (uint32_t g = 0; g < uint32_t(sc_.size()); ++g) {
    LayerScore& h = sc_[g];
    const size_t n = units(g);
    if (h.open_T.empty()) std::fill(h.T.begin(), h.T.end(), 0u);
    else h.T = h.open_T;
    for (size_t r = 0; r < n; ++r)
      h.rowsum[r] = h.open_T.empty() ? 0 : std::accumulate(h.T.begin() + std::ptrdiff_t(r * n),
                                                           h.T.begin() + std::ptrdiff_t((r + 1) * n), uint64_t(0));
    std::fill(h.cnt.begin(), h.cnt.end(), uint16_t(0));
    std::fill(h.ring.begin(), h.ring.end(), 0u);
    std::fill(h.ring_len.begin(), h.ring_len.end(), uint8_t(0));
    h.ring_head = h.ring_n = 0;
    h.prev.clear();
    h.cur.clear();
    h.served = h.list_epoch = 0;
  }
  epoch_ = 0;
  stamp_ = open_.stamp;
}

void SlotCache::set_policy(uint32_t policy) {
  require(policy <= 2, SS_E_INVALID, "device-gated: policy must be LRU, SCORED or SCORED_AUTO");
  require(!policy || !sc_.empty(), SS_E_INVALID, "device-gated: scoring must be provisioned at open");
  drain_pending();
  drain();
  collect();
  c_.scored = policy != 0;
  c_.scored_auto = policy == 2;
  reset_score();
  for (Entry& x : e_) x.demand_epoch = x.lru_stamp = 0;
  stamp_ = 0;  // the stamps follow the recency order from the back
  for (uint32_t k = recent_.back(); k != kNil; k = recent_.newer(k)) e_[k].lru_stamp = ++stamp_;
}

void SlotCache::load_counts(const std::vector<std::vector<uint32_t>>& cells) {
  require(c_.scored && cells.size() == sc_.size(), SS_E_INVALID, "device-gated: a score profile needs policy SCORED");
  for (uint32_t g = 0; g < gated(); ++g) {
    const size_t n = units(g);
    require(cells[g].size() == n * n, SS_E_INVALID, "device-gated: a profile layer is not units^2 counts");
    LayerScore& h = sc_[g];
    h.T = cells[g];
    for (size_t r = 0; r < n; ++r)
      h.rowsum[r] = std::accumulate(h.T.begin() + std::ptrdiff_t(r * n), h.T.begin() + std::ptrdiff_t((r + 1) * n),
                                    uint64_t(0));
    h.open_T = h.T;  // the reset_open state
  }
}

// ---- kept-resident layers (ss_dg_make_resident) ----
// Every refusal comes first (ids, capacity, blocks), then the cache settles, then: prefetches of the layer already
// landed are admitted; victims are chosen for the units still to copy in (scores when scored, else the recency tail);
// each unit goes into a free slot, evicting victims (a clean copy or a drop to a file costs nothing, a dirty one is
// written back first) when none is free; a pinned unit is copied from its block, a file unit read through the staging
// buffers (reads in flight up to the queue depth). The units copied in become the most recent, in the caller's order.
SlotCache::ResidentResult SlotCache::make_resident(uint32_t g, const std::vector<uint32_t>& ids,
                                                   const std::vector<uint32_t>& other_kept) {
  const auto t0 = Clock::now();
  require(g < gated(), SS_E_INVALID, "ss_dg_make_resident: gated layer out of range");
  std::vector<uint8_t> want(keys_, 0), other(keys_, 0);
  for (uint32_t u : ids) {
    require(u < units(g), SS_E_INVALID, "ss_dg_make_resident: id out of range");
    require(!want[key(g, u)], SS_E_INVALID, "ss_dg_make_resident: duplicate id " + std::to_string(u));
    want[key(g, u)] = 1;
  }
  size_t n_other = 0;
  for (uint32_t k : other_kept) {
    if (k >= keys_ || other[k] || want[k]) continue;
    other[k] = 1;
    ++n_other;
  }
  // capacity: every layer's kept units leave the spare target free for the boundaries
  const uint64_t room = uint64_t(c_.persistent_slots) - c_.spare_target;
  require(ids.size() + n_other <= room, SS_E_CAPACITY,
          "ss_dg_make_resident: " + std::to_string(ids.size()) + " units of gated layer " + std::to_string(g) + " + " +
              std::to_string(n_other) + " other kept units + the spare target " + std::to_string(c_.spare_target) +
              " exceed the " + std::to_string(c_.persistent_slots) + " persistent slots");
  size_t to_copy = 0, evictable = 0, evicting = 0;
  for (uint32_t k = 0; k < keys_; ++k) {
    const Home h = e_[k].home;
    require(h != Home::Bank, SS_E_BACKEND, "ss_dg_make_resident: a bank unit between tokens");
    evicting += h == Home::Evicting ? 1 : 0;
    if (want[k]) to_copy += h != Home::Device && h != Home::Coming ? 1 : 0;
    else evictable += h == Home::Device && !other[k] ? 1 : 0;
  }
  const size_t discards = size_t(std::count_if(wbs_.begin(), wbs_.end(), [](const Writeback& w) { return w.discard; }));
  const size_t free_after = free_slots_.size() + evicting;
  require(to_copy <= free_after + evictable, SS_E_CAPACITY,
          "ss_dg_make_resident: " + std::to_string(to_copy) + " units to copy in, " + std::to_string(free_after) +
              " free slots and " + std::to_string(evictable) +
              " evictable units (the rest hold other layers' kept units or prefetches in flight)");
  require(c_.disk_tier || to_copy <= free_after || free_after + free_blocks_.size() + discards > 0, SS_E_CAPACITY,
          "ss_dg_make_resident: no free slot and no free pinned block to start the write-backs");
  stamp_room("ss_dg_make_resident");
  settle_writebacks("ss_dg_make_resident");

  ResidentResult res;
  std::vector<uint32_t> in;  // the units to copy in, in the caller's order
  for (uint32_t u : ids) {
    const uint32_t k = key(g, u);
    Entry& x = e_[k];
    if (x.home == Home::Device) continue;
    if (x.home != Home::Coming) {
      in.push_back(k);
      continue;
    }
    x.home = Home::Device;  // a prefetch whose copy landed: admitted now
    x.via_pf = false;
    recycle(x.pf_done);
    if (x.block >= 0) free_blocks_.give(x.block);
    x.block = -1;
  }
  auto eligible = [&](uint32_t k) {
    const Entry& x = e_[k];
    return x.home == Home::Device && !x.wb_pending && !want[k] && !other[k];
  };
  std::vector<uint32_t> victims;
  const size_t n_vict = in.size() > free_slots_.size() ? in.size() - free_slots_.size() : 0;
  if (n_vict != 0 && c_.scored) {
    select_scored(n_vict, eligible, false);
    for (const ScoreCand& cd : select_heap_) victims.push_back(cd.key);
  } else {
    for (uint32_t k = recent_.back(); k != kNil && victims.size() < n_vict; k = recent_.newer(k))
      if (eligible(k)) victims.push_back(k);
  }
  if (victims.size() != n_vict) broken("ss_dg_make_resident: fewer victims than the capacity check counted");

  std::vector<uint8_t> hold = want;  // never dropped to a file here: the units to copy in, this call's write-backs
  std::vector<int32_t> released;     // source blocks of committed copies (free once the demand stream synced)
  std::vector<int32_t> released_lands;  // the same of landed units' landing blocks
  std::vector<int32_t> written;      // slots of written-back victims (free once the write-back stream synced)
  struct Read {
    uint32_t key;
    int32_t slot, stage;
    void* handle;
  };
  std::deque<Read> reads;  // file reads in flight, oldest first, each in its own staging buffer
  const size_t depth =
      c_.disk_tier ? std::max<size_t>(1, std::min<size_t>(std::max<uint32_t>(c_.disk_queue, 1), c_.disk_staging)) : 1;
  bool io_failed = false;
  uint64_t n_read = 0, n_written = 0, read_ns = 0;
  // the committed units become the most recent, in the order of `in`, on every exit
  std::vector<uint8_t> committed(in.size(), 0);
  struct Promote {
    SlotCache& cache;
    const std::vector<uint32_t>& order;
    const std::vector<uint8_t>& done;
    ~Promote() {
      for (size_t i = 0; i < order.size(); ++i)
        if (done[i]) cache.touch(order[i]);
    }
  } promote{*this, in, committed};
  std::vector<int32_t> position(keys_, -1);
  for (size_t i = 0; i < in.size(); ++i) position[in[i]] = int32_t(i);
  auto commit = [&](uint32_t k, int32_t slot) {
    Entry& x = e_[k];
    x.home = Home::Device;
    x.slot = slot;
    x.block = -1;
    committed[size_t(position[k])] = 1;
    ++on_device_;
    ++res.copied;
  };
  auto copy_in = [&](uint32_t k, int32_t slot, int32_t src) {  // the copy and its entry, or nothing owned changes
    try {
      m_->h2d(Mover::kDem, slot, src, k);
      publish(Mover::kDem, k, slot);
    } catch (...) {
      set_entry(k, -1);
      free_slots_.give(slot);
      throw;
    }
  };
  auto settle_copies = [&] {
    m_->sync(Mover::kDem);
    for (int32_t b : released) free_blocks_.give(b);
    released.clear();
    for (int32_t l : released_lands) free_lands_.give(l);
    released_lands.clear();
  };
  auto settle_writes = [&] {
    if (written.empty()) return;
    m_->sync(Mover::kD2h);
    for (int32_t s : written) free_slots_.give(s);
    written.clear();
  };
  auto end_read = [&](size_t i) {  // a read's end: its copy and entry, its staging buffer's event
    const Read rd = reads[i];
    reads.erase(reads.begin() + std::ptrdiff_t(i));
    const auto ta = Clock::now();
    try {
      m_->read_end(rd.handle);
    } catch (...) {
      read_ns += ns_since(ta);
      io_failed = true;
      free_slots_.give(rd.slot);
      throw;
    }
    read_ns += ns_since(ta);
    copy_in(rd.key, rd.slot, rd.stage);
    --on_file_;
    commit(rd.key, rd.slot);
    ++n_read;
    void*& ev = stage_ev_[uint32_t(rd.stage) - c_.blocks];
    if (ev == nullptr) ev = event();
    m_->record(ev, Mover::kDem);
  };
  auto account = [&] {
    const uint64_t copied_bytes = uint64_t(res.copied) * unit_bytes_;
    st_.resident_units += res.copied;
    st_.resident_evicted += res.evicted;
    st_.resident_bytes += copied_bytes;
    st_.mkres_file_reads += n_read;
    st_.mkres_file_bytes += n_read * unit_bytes_;
    st_.mkres_read_ns += read_ns;
    st_.mkres_h2d_bytes += copied_bytes;
    st_.mkres_wb_bytes += n_written * unit_bytes_;
    st_.resident_ns += ns_since(t0);
  };
  // With no free slot: victims evicted until the free slots and those being written back cover the units left to
  // copy; no copy for a clean one or one dropped to its file (a pinned unit dropped to its file frees a block when
  // none is free), else written back into a free block.
  size_t vi = 0;
  auto evict_for = [&](size_t left) {
    while (vi < victims.size() && free_slots_.size() + written.size() < left) {
      const uint32_t v = victims[vi];
      Entry& x = e_[v];
      if (!x.backed && free_blocks_.empty() && !released.empty()) {  // the blocks of the copies already enqueued
        settle_copies();
        continue;
      }
      if (!x.backed && free_blocks_.empty() && !c_.disk_tier) break;
      const bool clean = !x.backed && clean_now();
      const bool no_copy = x.backed || clean || (free_blocks_.empty() && !drop_host_lru(&hold, false));
      if (clean) count_clean();
      int32_t b = -1;
      if (!no_copy) {
        b = free_blocks_.items().back();
        m_->d2h(Mover::kD2h, x.slot, b, -1, v);  // the dirty unit's only copy, written back before its slot is reused
        free_blocks_.take();
        ++n_written;
      }
      ++vi;
      ++res.evicted;
      leave_device(v);
      if (no_copy) {
        free_slots_.give(x.slot);
        to_lower(v);
        continue;
      }
      written.push_back(x.slot);
      x.home = Home::Host;
      x.slot = -1;
      x.block = b;
      home_push(v);
      hold[v] = 1;
    }
  };
  try {
    for (size_t next = 0; next < in.size();) {
      if (free_slots_.empty()) evict_for(in.size() - next);
      settle_writes();
      if (free_slots_.empty()) fail(SS_E_BACKEND, "ss_dg_make_resident: no slot for a unit");
      const int32_t slot = free_slots_.take();
      const uint32_t k = in[next];
      Entry& x = e_[k];
      if (x.home == Home::Host) {
        const int32_t b = x.block;
        copy_in(k, slot, b);
        ++next;
        home_erase(k);
        released.push_back(b);
        commit(k, slot);
        continue;
      }
      if (x.home == Home::Landed) {  // its landing block is the source, as a pinned block (drained: landed)
        const int32_t l = x.land;
        copy_in(k, slot, land_block(l));
        ++next;
        released_lands.push_back(l);
        land_owner_[size_t(l)] = kNil;
        x.land = -1;
        x.land_age = 0;
        --on_land_;
        commit(k, slot);
        continue;
      }
      // its file, through the next staging buffer (its last copy landed first): at most `depth` reads in flight, the
      // finished ones ending first (any position), then the oldest; a read holding the next buffer ends before it
      try {
        if (reads.size() >= depth)
          for (size_t j = 0; j < reads.size();) {
            if (m_->read_done(reads[j].handle)) end_read(j);
            else ++j;
          }
        if (reads.size() >= depth) end_read(0);
        const uint32_t i = stage_next_;
        stage_next_ = (stage_next_ + 1) % c_.disk_staging;
        const int32_t stage = int32_t(c_.blocks + i);
        const auto holder = std::find_if(reads.begin(), reads.end(), [stage](const Read& r) { return r.stage == stage; });
        if (holder != reads.end()) end_read(size_t(holder - reads.begin()));
        if (stage_ev_[i] != nullptr && !m_->done(stage_ev_[i])) m_->event_sync(stage_ev_[i]);
        const auto tb = Clock::now();
        void* handle = nullptr;
        try {
          handle = m_->read_begin(k, stage);
        } catch (...) {
          read_ns += ns_since(tb);
          io_failed = true;
          throw;
        }
        read_ns += ns_since(tb);
        reads.push_back(Read{k, slot, stage, handle});
        ++next;
      } catch (...) {
        free_slots_.give(slot);
        throw;
      }
    }
    while (!reads.empty()) end_read(0);
    settle_writes();
    settle_copies();
    upload();  // (syncs the demand stream) every changed entry, the victims' -1 included
  } catch (...) {
    for (const Read& rd : reads) {  // reads not ended give their slots back (their keys never changed home)
      try {
        m_->read_end(rd.handle);
      } catch (...) {
      }
      free_slots_.give(rd.slot);
    }
    reads.clear();
    bool uploaded = false;
    if (io_failed) {  // the device is fine: what was enqueued lands, the table goes up
      try {
        settle_writes();
        settle_copies();
        upload();
        uploaded = true;
      } catch (...) {
      }
    }
    if (!uploaded) {  // a device failure: the host records stay one ownership (the context is poisoned by its caller)
      for (int32_t s : written) free_slots_.give(s);
      for (int32_t b : released) free_blocks_.give(b);
      for (int32_t l : released_lands) free_lands_.give(l);
      written.clear();
      released.clear();
      released_lands.clear();
    }
    account();
    throw;
  }
  account();
  return res;
}

// ---- placement rounds ----
// Decay and add the hits; order the movable units (device homes coldest first, pinned and file homes hottest first;
// ties: recency position, then key); then (a) pinned -> device: into a free slot while the device holds less than its
// share (persistent slots - spare target - kept - coming), else in place of the coldest device unit when hotter by the
// hysteresis factor (the demoted unit back to its clean block, or written back into a free block, or with the file
// tier into the block of the coldest pinned unit, dropped to its file); (b) file tier: a file unit read into the block
// of the coldest pinned unit (dropped to its file) when hotter by the hysteresis factor. A unit with no count never
// moves; every step checks the budgets and the cancellation first (dg_core.cpp:2592-2897).
RoundOut SlotCache::round(const RoundIn& in, const std::vector<uint32_t>& kept_keys) {
  const auto t0 = Clock::now();
  round_state_.store(kRoundRunning, std::memory_order_release);
  struct BackToIdle {
    std::atomic<int>& state;
    ~BackToIdle() { state.store(kRoundIdle, std::memory_order_release); }
  } idle{round_state_};
  last_round_ = RoundOut{};
  require(std::isfinite(in.decay) && in.decay >= 0 && in.decay <= 1, SS_E_INVALID, "ss_dg_round: decay must be 0..1");
  require(std::isfinite(in.hysteresis) && in.hysteresis >= 1 && in.hysteresis <= 1e6, SS_E_INVALID,
          "ss_dg_round: hysteresis must be 1..1e6");
  require(in.flags == 0, SS_E_INVALID, "ss_dg_round: unknown flags");
  std::vector<uint8_t> kept(keys_, 0);
  size_t n_kept = 0;
  for (uint32_t k : kept_keys) {
    if (k >= keys_ || kept[k]) continue;
    kept[k] = 1;
    ++n_kept;
  }
  if (std::any_of(e_.begin(), e_.end(), [](const Entry& x) { return x.home == Home::Bank; }))
    broken("a bank unit between tokens");
  stamp_room("ss_dg_round");
  settle_writebacks("ss_dg_round");
  for (uint32_t k = 0; k < keys_; ++k) {
    rs_[k] = in.decay * rs_[k] + double(rhits_[k]);
    rhits_[k] = 0;
  }

  RoundOut out;
  const uint64_t ub = unit_bytes_;
  uint64_t spent = 0;
  uint32_t moved = 0;
  auto affordable = [&](uint64_t b) {
    return in.budget_bytes == 0 || (spent <= in.budget_bytes && b <= in.budget_bytes - spent);
  };
  auto stop_asked = [&] {
    if (round_state_.load(std::memory_order_acquire) == kRoundCancel) out.cancelled = 1;
    return out.cancelled != 0;
  };
  // recency positions, least recent first (device homes; pinned homes filled before (b))
  std::vector<uint32_t> age(keys_, 0), home_age(keys_, 0);
  uint32_t next_age = 0;
  for (uint32_t k = recent_.back(); k != kNil; k = recent_.newer(k)) age[k] = next_age++;
  auto hotter = [&](uint32_t a, uint32_t b) { return rs_[a] != rs_[b] ? rs_[a] > rs_[b] : a < b; };
  auto colder = [&](const std::vector<uint32_t>& rank) {
    return [&](uint32_t a, uint32_t b) {
      if (rs_[a] != rs_[b]) return rs_[a] < rs_[b];
      return rank[a] != rank[b] ? rank[a] < rank[b] : a < b;
    };
  };
  std::vector<uint32_t> dev, host, file;
  size_t n_coming = 0;
  for (uint32_t k = 0; k < keys_; ++k) {
    const Entry& x = e_[k];
    n_coming += x.home == Home::Coming ? 1 : 0;
    if (kept[k] || x.wb_pending) continue;
    if (x.home == Home::Device) dev.push_back(k);
    else if (x.home == Home::Host) host.push_back(k);
    else if (x.home == Home::File) file.push_back(k);
  }
  std::sort(dev.begin(), dev.end(), colder(age));
  std::sort(host.begin(), host.end(), hotter);
  std::sort(file.begin(), file.end(), hotter);
  int64_t share = int64_t(c_.persistent_slots) - int64_t(c_.spare_target) - int64_t(n_kept) - int64_t(n_coming) -
                  int64_t(dev.size());
  const Mover::Stream wb_stream = c_.wb_on_d2h ? Mover::kD2h : Mover::kDem;
  auto account = [&] {
    out.ns = ns_since(t0);
    ++st_.round_count;
    st_.round_units += uint64_t(out.promoted_to_device) + out.promoted_to_pinned + out.demoted_from_device +
                       out.dropped_to_file;
    st_.round_bytes += out.bytes_read + out.bytes_h2d + out.bytes_written_back;
    st_.round_ns += out.ns;
    st_.round_cancelled += out.cancelled;
    last_round_ = out;
  };
  // a pinned unit into `slot`: its home changes once the copy and its entry were accepted and the demand stream synced;
  // a cancellation seen then drops it (the slot free again, the unit keeps its block)
  auto promote = [&](uint32_t k, int32_t slot) {
    Entry& x = e_[k];
    const int32_t src = x.block;
    try {
      m_->h2d(Mover::kDem, slot, src, k);
      publish(Mover::kDem, k, slot);
      m_->sync(Mover::kDem);
    } catch (...) {
      set_entry(k, -1);
      free_slots_.give(slot);
      throw;
    }
    spent += ub;
    out.bytes_h2d += ub;
    if (stop_asked()) {
      set_entry(k, -1);
      free_slots_.give(slot);
      return false;
    }
    home_erase(k);
    free_blocks_.give(src);
    x.block = -1;
    x.slot = slot;
    x.home = Home::Device;
    touch(k);
    ++on_device_;
    ++out.promoted_to_device;
    return true;
  };
  // a pinned unit dropped to its file (no copy: the file holds its bytes); its block is returned
  auto drop_to_file = [&](uint32_t p) {
    Entry& y = e_[p];
    home_erase(p);
    const int32_t b = y.block;
    y.block = -1;
    y.home = Home::File;
    ++on_file_;
    ++out.dropped_to_file;
    return b;
  };
  // a block for a demoted unit's write-back: a free one, else (file tier) the coldest pinned unit's, dropped to its
  // file (never `except`); -1 when none
  size_t coldest = host.size();
  auto block_for_writeback = [&](uint32_t except) -> int32_t {
    if (!free_blocks_.empty()) return free_blocks_.take();
    if (!c_.disk_tier) return -1;
    while (coldest > 0) {
      const uint32_t p = host[--coldest];
      if (p != except && e_[p].home == Home::Host) return drop_to_file(p);
    }
    return -1;
  };
  // (b)'s reads: one at a time (synchronous), each committed at the next read or at the end
  struct Landing {
    uint32_t key;
    int32_t block;
  };
  std::deque<Landing> reads;
  auto commit_read = [&] {
    const Landing rd = reads.front();
    reads.pop_front();
    out.bytes_read += ub;
    if (stop_asked()) {  // the block free again, the unit stays in its file
      free_blocks_.give(rd.block);
      return;
    }
    Entry& x = e_[rd.key];
    --on_file_;
    x.home = Home::Host;
    x.block = rd.block;
    home_push(rd.key);
    ++out.promoted_to_pinned;
  };
  try {
    size_t next_dev = 0;
    for (size_t i = 0; i < host.size() && moved < in.max_units; ++i) {  // (a) pinned -> device
      const uint32_t c = host[i];
      if (!(rs_[c] > 0)) break;
      if (e_[c].home != Home::Host) continue;  // (dropped to its file for a write-back block)
      if (stop_asked()) break;
      if (share > 0 && free_slots_.size() > c_.spare_target) {  // the device holds less than its share
        if (!affordable(ub)) break;
        if (!promote(c, free_slots_.take())) break;
        --share;
        ++moved;
        continue;
      }
      if (next_dev >= dev.size()) break;
      const uint32_t v = dev[next_dev];
      if (!(rs_[c] > in.hysteresis * rs_[v])) break;
      Entry& y = e_[v];
      const bool clean = !y.backed && clean_now();  // clean_evict: no free block, to its file (no write)
      const bool free_demotion = y.backed || clean;
      if (!affordable(ub + (free_demotion ? 0 : ub))) break;
      const int32_t slot = y.slot;
      if (free_demotion) {  // a clean copy: its block is its home again, no write (clean_evict: its file)
        leave_device(v);
        to_lower(v);
        if (clean) count_clean();
      } else {
        const int32_t b = block_for_writeback(c);
        if (b < 0) break;
        try {
          m_->d2h(wb_stream, slot, b, -1, v);
          m_->sync(wb_stream);
        } catch (...) {
          free_blocks_.give(b);  // the unit keeps its slot (its only copy)
          throw;
        }
        leave_device(v);
        y.home = Home::Host;
        y.slot = -1;
        y.block = b;
        home_push(v);
        spent += ub;
        out.bytes_written_back += ub;
      }
      ++next_dev;
      ++out.demoted_from_device;
      if (!promote(c, slot)) break;  // (cancelled: the demoted unit's slot stays free)
      ++moved;
    }
    if (c_.disk_tier && !out.cancelled) {  // (b) file -> pinned, in place of the coldest pinned units
      std::vector<uint32_t> pinned;
      for (uint32_t k = 0; k < keys_; ++k)
        if (e_[k].home == Home::Host && !kept[k] && !e_[k].wb_pending) pinned.push_back(k);
      uint32_t h_age = 0;
      for (uint32_t k = homes_.back(); k != kNil; k = homes_.newer(k)) home_age[k] = h_age++;  // after (a)'s pushes
      std::sort(pinned.begin(), pinned.end(), colder(home_age));
      size_t pv = 0;
      for (size_t i = 0; i < file.size() && moved < in.max_units && pv < pinned.size(); ++i) {
        const uint32_t c = file[i];
        if (!(rs_[c] > 0)) break;
        if (e_[c].home != Home::File) continue;
        if (stop_asked()) break;
        if (!(rs_[c] > in.hysteresis * rs_[pinned[pv]])) break;
        if (!affordable(ub)) break;
        if (!reads.empty()) commit_read();
        if (out.cancelled) break;
        const int32_t b = drop_to_file(pinned[pv++]);  // its block is quiescent
        try {
          m_->read_unit(c, b);
        } catch (...) {
          free_blocks_.give(b);
          throw;
        }
        reads.push_back(Landing{c, b});
        spent += ub;
        ++moved;
      }
      while (!reads.empty()) commit_read();
    }
    upload();  // (syncs the demand stream) every changed entry
  } catch (...) {
    for (const Landing& rd : reads) free_blocks_.give(rd.block);  // never committed: their units stay in their files
    reads.clear();
    try {  // the moves made so far go up (a failed device fails this too; the caller then poisons the context)
      upload();
    } catch (...) {
    }
    account();
    throw;
  }
  account();
  return out;
}

void SlotCache::seed_round_counts(const std::vector<uint32_t>& keys, const std::vector<float>& counts) {
  require(keys.size() == counts.size(), SS_E_INVALID, "ss_dg_round_seed_counts: keys and counts differ in length");
  for (size_t i = 0; i < keys.size(); ++i) {
    require(keys[i] < keys_, SS_E_INVALID, "ss_dg_round_seed_counts: unit out of range");
    require(std::isfinite(counts[i]) && counts[i] >= 0, SS_E_INVALID,
            "ss_dg_round_seed_counts: counts must be finite and >= 0");
  }
  for (size_t i = 0; i < keys.size(); ++i) rs_[keys[i]] = double(counts[i]);
}

// Between tokens: pinned units into free slots above the spare target, each copied and made the most recent.
uint32_t SlotCache::seed(const std::vector<uint32_t>& keys) {
  drain_pending();  // between tokens (copies, then an upload)
  stamp_room("ss_seed");
  if (!coming_.empty()) m_->sync(Mover::kPf);
  collect();
  uint32_t seeded = 0;
  for (uint32_t k : keys) {
    require(k < keys_, SS_E_INVALID, "ss_seed: unit out of range");
    Entry& x = e_[k];
    if (x.home != Home::Host || free_slots_.size() <= c_.spare_target) continue;
    const int32_t slot = free_slots_.take();
    m_->h2d(Mover::kDem, slot, x.block, k);
    home_erase(k);
    free_blocks_.give(x.block);
    x.block = -1;
    x.slot = slot;
    x.home = Home::Device;
    set_entry(k, slot);
    touch(k);
    ++on_device_;
    ++seeded;
  }
  if (seeded) upload();  // syncs kDem: the copies landed before their blocks are reused
  return seeded;
}

void SlotCache::drain() {
  drain_pending();
  cancel_landings();  // (the ones not running: back to their files; the others landed, or back on a failure)
  end_landings();
  while (!deferred_.empty()) finish_front();
  for (Mover::Stream s : {Mover::kDem, Mover::kPf, Mover::kD2h}) m_->sync(s);
  reclaim_lands(true);
}

std::vector<uint32_t> SlotCache::residency() const {
  std::vector<uint32_t> out;
  out.reserve(on_device_);
  for (uint32_t k = recent_.front(); k != kNil; k = recent_.older(k))
    if (e_[k].home == Home::Device) out.push_back(k);
  return out;
}

void SlotCache::set_wb_defer(bool on) {
  drain_pending();  // (settings: between tokens, every read ended first)
  if (on == c_.wb_defer) return;
  while (!on && !deferred_.empty()) finish_front();
  c_.wb_defer = on;
  apply_wb_defer();
  credit_ = 0;
  prev_evict_ = 0;
}

void SlotCache::set_spare_target(uint32_t n) {
  drain_pending();
  require(n <= c_.persistent_slots, SS_E_INVALID, "device-gated: spare target above the persistent slots");
  c_.spare_target = n;
  if (c_.prefetch_reserve_auto) c_.prefetch_reserve = std::min<uint32_t>(24, n / 4);
}

void SlotCache::set_clean_evict(bool on) {
  drain_pending();
  c_.clean_evict = on;
}

void SlotCache::set_pf_revert(bool on) {
  drain_pending();
  c_.pf_revert = on;
}

void SlotCache::set_prefetch_budget(uint32_t per_layer, uint32_t per_token) {
  drain_pending();
  c_.prefetch_per_layer = per_layer;
  c_.prefetch_per_token = per_token;
}

void SlotCache::set_pressure(uint32_t free_per_token, uint32_t evict_recent) {
  drain_pending();
  pressure_ = free_per_token != 0 || evict_recent != 0;
  pressure_free_ = free_per_token;
  pressure_recent_ = evict_recent;
}

// ---- reset to the open placement ----
// Locations: slots [0, P), blocks [P, P + blocks), the reset staging buffer and (file tier) the unit's file. Every
// misplaced unit moves once: units going back to their file first (no copy, their location vacated), then chains
// that end in a free location (each move fills the hole the previous one left; a unit read from its file ends its
// chain), then the remaining cycles through the staging buffer (dg_core.cpp:2976-3075). The mover executes each move
// before the next one reads its destination; consecutive slot-to-slot moves share launches, a move's wave one after
// every earlier move that reads its destination or writes its source.
void SlotCache::reset_open() {
  require(open_.ent.size() == keys_, SS_E_INVALID, "device-gated: reset before place");
  settle_writebacks("reset");
  for (Entry& x : e_)
    if (x.pf_done) {
      m_->event_sync(x.pf_done);
      recycle(x.pf_done);
    }
  for (void* ev : stage_ev_)  // every staging copy landed
    if (ev) m_->event_sync(ev);
  for (uint32_t l = 0; l < c_.landing_blocks; ++l)  // landings (ended: none reads its block) back to their files
    if (land_owner_[l] != kNil) unland(land_owner_[l]);
  const size_t P = c_.persistent_slots, N = P + c_.blocks, kStage = N, kFile = N + 1;
  std::vector<size_t> at(keys_), goal(keys_);
  std::vector<uint32_t> holder(N + 1, kNil), wants(N + 1, kNil);  // per location: its unit now, the unit it should hold
  for (uint32_t k = 0; k < keys_; ++k) {
    const Entry& x = e_[k];
    if (x.home == Home::Evicting) broken("reset left an evicting unit");
    // a unit read from its file has no block: a Coming one's slot is its only copy; a bank slot is no persistent
    // location, so a bank unit read from its file goes back to it
    const bool on_slot = x.home == Home::Device || (x.home == Home::Coming && x.block < 0);
    const bool in_file = x.home == Home::File || (x.home == Home::Bank && x.block < 0);
    at[k] = in_file ? kFile : on_slot ? size_t(x.slot) : P + size_t(x.block);
    const Entry& o = open_.ent[k];
    goal[k] = o.home == Home::File ? kFile : o.home == Home::Device ? size_t(o.slot) : P + size_t(o.block);
    if (at[k] != kFile) holder[at[k]] = k;
    if (goal[k] != kFile) wants[goal[k]] = k;
  }
  for (uint32_t k = 0; k < keys_; ++k)  // back to its file: its location is vacated, no copy
    if (goal[k] == kFile && at[k] != kFile) {
      holder[at[k]] = kNil;
      at[k] = kFile;
    }
  struct Move {
    size_t from, to;
    uint32_t key;
  };
  std::vector<Move> moves;  // planned first (bookkeeping only), executed after
  auto plan = [&](uint32_t k, size_t to) {
    const size_t from = at[k];
    if (to > N || holder[to] != kNil) broken("reset would overwrite a live source");
    moves.push_back(Move{from, to, k});
    if (from != kFile) holder[from] = kNil;
    holder[to] = k;
    at[k] = to;
  };
  for (size_t loc = 0; loc < N; ++loc)  // chains ending in a free location
    for (size_t hole = loc; hole < N && holder[hole] == kNil && wants[hole] != kNil;) {
      const uint32_t k = wants[hole];
      const size_t vacated = at[k];
      plan(k, hole);
      hole = vacated;
    }
  for (uint32_t k = 0; k < keys_; ++k) {  // cycles, through the staging buffer
    if (at[k] == goal[k]) continue;
    if (at[k] == kFile) broken("reset left a file read behind");
    size_t hole = at[k];
    plan(k, kStage);
    while (hole != goal[k]) {
      const uint32_t next = wants[hole];
      if (next == kNil) broken("reset cycle without a predecessor");
      const size_t vacated = at[next];
      plan(next, hole);
      hole = vacated;
    }
    plan(k, hole);
  }
  auto block_at = [&](size_t loc) { return loc == kStage ? -1 : int32_t(loc - P); };
  std::vector<std::pair<int32_t, int32_t>> slot_moves;
  std::vector<uint32_t> waves;
  auto run_slot_moves = [&] {
    if (slot_moves.empty()) return;
    m_->d2d_moves(slot_moves, waves);
    slot_moves.clear();
    waves.clear();
  };
  for (const Move& mv : moves) {
    ++st_.reset_moves;
    st_.reset_bytes += unit_bytes_;
    if (mv.from < P && mv.to < P) {
      uint32_t wave = 0;
      for (size_t i = 0; i < slot_moves.size(); ++i)
        if (size_t(slot_moves[i].first) == mv.to || size_t(slot_moves[i].second) == mv.from)
          wave = std::max(wave, waves[i] + 1);
      slot_moves.push_back({int32_t(mv.from), int32_t(mv.to)});
      waves.push_back(wave);
      continue;
    }
    run_slot_moves();
    if (mv.from == kFile && mv.to < P) {  // read into the reset staging buffer, then to the slot
      m_->read_unit(mv.key, -1);
      m_->h2d(Mover::kDem, int32_t(mv.to), -1, mv.key);
      m_->sync(Mover::kDem);
    } else if (mv.from == kFile) {
      m_->read_unit(mv.key, block_at(mv.to));
    } else if (mv.from < P) {
      m_->d2h(Mover::kD2h, int32_t(mv.from), block_at(mv.to), -1, mv.key);
      m_->sync(Mover::kD2h);
    } else if (mv.to < P) {
      m_->h2d(Mover::kDem, int32_t(mv.to), block_at(mv.from), mv.key);
      m_->sync(Mover::kDem);
    } else {
      m_->h2h(block_at(mv.from), block_at(mv.to), mv.key);
    }
  }
  run_slot_moves();
  // every host record back to the open's
  c_ = open_.cfg;
  apply_wb_defer();
  e_ = open_.ent;
  reset_score();  // the history's open state (a profile's counts, or none)
  std::fill(rs_.begin(), rs_.end(), 0.0);  // placement rounds: the counts start over
  std::fill(rhits_.begin(), rhits_.end(), 0u);
  backed_ = 0;  // clean copies are dropped: the open holds none
  table_ = open_.table;
  free_slots_ = open_.slots;
  free_blocks_ = open_.blocks;
  recent_ = open_.recent;
  homes_ = open_.homes;
  free_lands_ = open_.lands;  // (every landing block free, in the open's order)
  on_land_ = 0;
  std::fill(served_.begin(), served_.end(), uint8_t(0));
  on_device_ = open_.on_device;
  on_file_ = open_.on_file;
  stage_next_ = 0;
  coming_.clear();
  banked_.clear();
  std::fill(bank_key_.begin(), bank_key_.end(), kNil);
  for (int b = 0; b < 2; ++b) {
    bank_seq_[b] = bank_next_[b] = 0;
    bank_layer_[b] = kNil;
  }
  std::fill(pf_layer_.begin(), pf_layer_.end(), 0u);
  pf_token_ = 0;
  pred_.clear();
  pred_layer_ = kNil;
  std::fill(layer_missed_.begin(), layer_missed_.end(), uint8_t(0));
  pressure_ = false;
  pressure_free_ = pressure_recent_ = demand_free_used_ = 0;
  prev_evict_ = 0;
  credit_ = 0;
  outstanding_ = 0;
  m_->upload_table(table_.data(), keys_);  // the open's whole table
  clear_dirty();
  device_table_known_ = false;
}

// ---- invariants ----
void SlotCache::check() const {
  std::vector<uint8_t> slot_owner(slots_, 0), block_owner(c_.blocks, 0), land_owner(c_.landing_blocks, 0);
  auto own = [this](std::vector<uint8_t>& v, int64_t i, const char* what) {
    if (i < 0 || size_t(i) >= v.size() || v[size_t(i)]) broken(what);
    v[size_t(i)] = 1;
  };
  if (ranged_ && device_table_known_)  // every entry the device does not hold yet is marked for the next upload
    for (uint32_t k = 0; k < keys_; ++k)
      if (table_[k] != device_table_[k]) {
        const uint32_t g = gated_of(k);
        if (k < dirty_lo_[g] || k > dirty_hi_[g]) broken("a table entry changed without its mark");
      }
  uint32_t listed = 0, homes_listed = 0, dev = 0, hosts = 0, files = 0, lands = 0, landing_n = 0;
  for (uint32_t k = recent_.front(); k != kNil; k = recent_.older(k)) {
    if (++listed > keys_) broken("the recency list has a cycle");
    if (e_[k].home != Home::Device && e_[k].home != Home::Coming) broken("a listed unit is not on the device");
  }
  for (uint32_t k = homes_.front(); k != kNil; k = homes_.older(k)) {
    if (++homes_listed > keys_) broken("the pinned recency list has a cycle");
    if (e_[k].home != Home::Host) broken("a unit in the pinned recency list is not a pinned home");
  }
  if (!homes_.consistent()) broken("the pinned recency list's front-half cursor");
  for (uint32_t k = 0; k < keys_; ++k) {
    const Entry& x = e_[k];
    const bool in_recent = recent_.has(k);
    if ((x.land >= 0) != (x.home == Home::Landing || x.home == Home::Landed)) broken("a landing block outside a landing");
    switch (x.home) {
      case Home::Host:
        own(block_owner, x.block, "a host unit without its own block");
        if (table_[k] != -1) broken("a host unit with a published entry");
        if (in_recent) broken("a host unit in the recency list");
        ++hosts;
        break;
      case Home::File:
        if (!c_.disk_tier) broken("a file home without the file tier");
        if (x.slot >= 0 || x.block >= 0 || in_recent || homes_.has(k)) broken("a file home holding a slot or a block");
        if (table_[k] != -1) broken("a file home with a published entry");
        ++files;
        break;
      case Home::Device:
      case Home::Coming:
        ++dev;
        own(slot_owner, x.slot, "a device unit without its own slot");
        if (x.slot >= int32_t(c_.persistent_slots)) broken("a device unit in a bank slot");
        if (table_[k] != x.slot) broken("a device unit's entry is not its slot");
        if (!in_recent) broken("a device unit outside the recency list");
        if (x.home == Home::Coming) {
          if (x.block >= 0 || !c_.disk_tier) own(block_owner, x.block, "a coming unit without its source block");
        } else if (x.backed) {
          own(block_owner, x.block, "a clean copy without its own block");
        } else if (x.block >= 0) {
          broken("a device unit still holding a block");
        }
        if (x.backed && x.home != Home::Device) broken("a clean copy of a unit not on the device");
        break;
      case Home::Bank:
        own(slot_owner, x.slot, "a bank unit without its own slot");
        if (x.block >= 0 || !c_.disk_tier) own(block_owner, x.block, "a bank unit without its block");
        if (x.slot < int32_t(c_.persistent_slots)) broken("a bank unit in a persistent slot");
        if (table_[k] != x.slot) broken("a bank unit's entry is not its slot");
        break;
      case Home::Evicting:
        own(slot_owner, x.slot, "an evicting unit without its slot");
        own(block_owner, x.block, "an evicting unit without its destination block");
        if (table_[k] != -1) broken("an evicting unit with a published entry");
        break;
      case Home::Landing:
      case Home::Landed:
        if (!c_.disk_tier || !c_.landing_blocks) broken("a landing without landing blocks");
        if (x.slot >= 0 || x.block >= 0 || table_[k] != -1 || in_recent || homes_.has(k) || x.pf_done)
          broken("a landing holding a slot, a block, an entry or a copy event");
        own(land_owner, x.land, "a landing without its own landing block");
        if (land_owner_[size_t(x.land)] != k) broken("a landing block's owner is another unit");
        if (x.home == Home::Landed && x.land_age >= std::max<uint32_t>(c_.landing_ttl, 1))
          broken("a landing past its time to live");
        ++lands;
        landing_n += x.home == Home::Landing ? 1 : 0;
        break;
    }
  }
  for (const LandRead& r : landing_)
    if (r.key >= keys_ || e_[r.key].home != Home::Landing || e_[r.key].land != r.land)
      broken("a landing read does not match its unit");
  if (landing_.size() != landing_n) broken("the landing reads disagree with the units landing");
  for (const LandBusy& b : land_busy_) own(land_owner, b.land, "a landing block behind a copy and in use");
  for (int32_t l : free_lands_.items()) own(land_owner, l, "a free landing block that is also in use");
  for (uint32_t l = 0; l < c_.landing_blocks; ++l) {
    if (!land_owner[l]) broken("a landing block neither free nor held");
    if (land_owner_[l] != kNil && e_[land_owner_[l]].land != int32_t(l)) broken("a landing block's owner");
  }
  if (lands != on_land_) broken("the landing count disagrees with the homes");
  if (dev != on_device_ || dev != listed) broken("the device count disagrees with the homes");
  if (files != on_file_) broken("the file count disagrees with the homes");
  if (c_.disk_tier && hosts != homes_listed) broken("the pinned recency list does not hold every pinned home");
  for (int32_t s : free_slots_.items()) own(slot_owner, s, "a free slot that is also in use");
  for (int32_t b : free_blocks_.items()) own(block_owner, b, "a free block that is also in use");
  for (const Writeback& w : wbs_)
    if (w.discard) own(block_owner, w.block, "a discarded write-back block in use");
  for (uint32_t s = 0; s < c_.persistent_slots; ++s)
    if (!slot_owner[s]) broken("a persistent slot neither free nor held");
  for (uint32_t b = 0; b < c_.blocks; ++b)
    if (!block_owner[b]) broken("a block neither free nor held");
}

}  // namespace tsb
