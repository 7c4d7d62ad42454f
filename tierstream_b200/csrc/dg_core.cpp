#include "dg_core.hpp"

#include <algorithm>
#include <chrono>
#include <cmath>

#include "errors.hpp"

namespace tsb {

SlotCache::SlotCache(const CacheConfig& cfg, Mover* m) : c_(cfg), m_(m) {
  base_.assign(1, 0);
  for (uint32_t n : c_.n_units) {
    require(n >= 1, SS_E_INVALID, "device-gated: a gated layer without units");
    base_.push_back(base_.back() + n);
  }
  keys_ = base_.back();
  require(c_.persistent_slots >= 1 && c_.spare_target <= c_.persistent_slots, SS_E_INVALID,
          "device-gated: spare target above the persistent slots");
  const uint64_t slots = uint64_t(c_.persistent_slots) + 2ull * c_.bank_slots;
  require(slots < 0x7fffffffull, SS_E_INVALID, "device-gated: more than 2^31 - 1 slots");
  slots_ = uint32_t(slots);
  bank_first_ = c_.persistent_slots;
  require(c_.inclusive == 0 || c_.inclusive < c_.blocks, SS_E_INVALID,
          "device-gated: the inclusive share must leave a block for write-backs");
  require(!c_.disk_tier || c_.disk_staging >= 1, SS_E_INVALID, "device-gated: the file tier needs staging buffers");
  require(c_.disk_tier || (!c_.disk_prefetch && !c_.disk_staging && !c_.home_blocks), SS_E_INVALID,
          "device-gated: file tier options without the file tier");
  require(uint64_t(c_.blocks) + c_.disk_staging < 0x7fffffffull, SS_E_INVALID, "device-gated: too many host blocks");
  stage_ev_.assign(c_.disk_staging, nullptr);
  require(!c_.no_admit || c_.bank_slots >= c_.max_ids, SS_E_CAPACITY,
          "device-gated: dg_no_admit serves every miss through a bank slot: it needs " + std::to_string(c_.max_ids) +
              " bank slots per bank (dg_max_ids), " + std::to_string(c_.bank_slots) + " configured");
  run_.assign(c_.n_units.size(), 1);
  rs_.assign(keys_, 0.0);
  rhits_.assign(keys_, 0);
  if (c_.scored) {  // every score table allocated now (the service thread never allocates)
    require(c_.w_trans <= 1000 && c_.w_freq <= 1000 && c_.w_rec <= 1000 && c_.w_trans + c_.w_freq + c_.w_rec == 1000,
            SS_E_INVALID, "device-gated: score weights must each be 0..1000 and sum to 1000");
    require(c_.max_ids >= 1 && c_.max_ids <= 64, SS_E_INVALID, "device-gated: score unions need max ids 1..64");
    sc_.resize(c_.n_units.size());
    for (size_t g = 0; g < sc_.size(); ++g) {
      const size_t n = c_.n_units[g];
      require(n <= 65536, SS_E_INVALID,
              "device-gated: scored eviction needs at most 65536 units per gated layer (gated layer " +
                  std::to_string(g) + " has " + std::to_string(n) + ")");
      LayerScore& l = sc_[g];
      l.T.assign(n * n, 0);
      l.rowsum.assign(n, 0);
      l.cnt.assign(n, 0);
      l.ring.assign(size_t(kWindow) * c_.max_ids, 0);
      l.ring_len.assign(kWindow, 0);
      l.prev.reserve(c_.max_ids);
      l.cur.reserve(c_.max_ids);
    }
    select_heap_.reserve(c_.persistent_slots);
  }
  e_.assign(keys_, Entry{});
  table_.assign(keys_, -1);
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
  for (const Pending& p : pending_) {  // reads in flight end before anything they write into can be freed
    try {
      m_->read_end(p.handle);
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
  uint32_t n = 0;
  for (uint32_t k : coming_) n += e_[k].home == Home::Coming ? 1u : 0u;
  return n;
}

void SlotCache::apply_wb_defer() {
  if (c_.wb_defer) {
    wb_stream_ = c_.wb_on_d2h ? Mover::kD2h : Mover::kDem;
    layer_bytes_ = c_.wb_layer_bytes ? c_.wb_layer_bytes : m_->part_bytes(0);
    max_outstanding_ = c_.wb_max_outstanding ? c_.wb_max_outstanding : 2 * unit_bytes_;
    require(layer_bytes_ <= uint64_t(INT64_MAX) / 4, SS_E_INVALID, "device-gated: dg_wb_layer_bytes too large");
    if (c_.wb_on_d2h && !post_ready_ev_) post_ready_ev_ = event();
  } else {
    wb_stream_ = Mover::kDem;
    layer_bytes_ = 0;
    max_outstanding_ = 0;
  }
}

void SlotCache::place(const std::vector<uint32_t>& order, const std::vector<uint8_t>* disk) {
  drain_pending();
  const uint32_t dev_max = c_.persistent_slots - c_.spare_target;
  std::vector<uint8_t> taken(keys_, 0);
  std::vector<uint32_t> dev;
  for (uint32_t k : order) {
    require(k < keys_, SS_E_INVALID, "device-gated: resident key out of range");
    if (!taken[k] && dev.size() < dev_max) {
      taken[k] = 1;
      dev.push_back(k);
    }
  }
  // file tier: which non-resident keys get a block, as flags (the plan's pinned units first, then its disk units,
  // each by priority: the order's keys first, then key order); host_rank is their recency order
  const bool three = c_.disk_tier;
  std::vector<uint8_t> blocked(keys_, 0);
  std::vector<uint32_t> host_rank;
  if (three) {
    require(!disk || disk->size() == keys_, SS_E_INVALID, "device-gated: the disk flags do not cover the keys");
    std::vector<uint8_t> seen(keys_, 0);
    std::vector<uint32_t> prio;
    for (uint32_t k : order)
      if (!seen[k]) {
        seen[k] = 1;
        prio.push_back(k);
      }
    for (uint32_t k = 0; k < keys_; ++k)
      if (!seen[k]) prio.push_back(k);
    const uint32_t cap = std::min(c_.home_blocks, c_.blocks);
    for (uint8_t pass = 0; pass < 2; ++pass)
      for (uint32_t k : prio)
        if (!taken[k] && (disk ? (*disk)[k] : uint8_t(0)) == pass && host_rank.size() < cap) {
          blocked[k] = 1;
          host_rank.push_back(k);
        }
  } else {
    require(uint64_t(keys_) - dev.size() <= c_.blocks, SS_E_CAPACITY,
            "device-gated: fewer host blocks than non-resident units");
  }
  int32_t next_block = 0;
  on_file_ = 0;
  hhead_ = htail_ = kNil;
  for (uint32_t k = 0; k < keys_; ++k) {
    e_[k] = Entry{};
    if (!taken[k] && (!three || blocked[k])) {
      e_[k].block = next_block++;  // Host home, blocks in key order
    } else if (!taken[k]) {
      e_[k].home = Home::File;
      ++on_file_;
    }
    table_[k] = -1;
  }
  for (size_t i = host_rank.size(); i-- > 0;) hpush(host_rank[i]);  // the first by priority most recently homed
  head_ = tail_ = kNil;
  for (uint32_t i = 0; i < dev.size(); ++i) {
    Entry& x = e_[dev[i]];
    x.home = Home::Device;
    x.slot = int32_t(i);
    table_[dev[i]] = x.slot;
  }
  for (size_t i = dev.size(); i-- > 0;) push_front(dev[i]);  // dev[0] ends up most recent
  on_device_ = uint32_t(dev.size());
  free_slots_.clear();
  free_blocks_.clear();
  for (uint32_t s = c_.persistent_slots; s-- > on_device_;) free_slots_.push_back(int32_t(s));
  for (int32_t b = int32_t(c_.blocks); b-- > next_block;) free_blocks_.push_back(b);
  open_c_ = c_;
  open_e_ = e_;
  open_table_ = table_;
  open_free_slots_ = free_slots_;
  open_free_blocks_ = free_blocks_;
  open_head_ = head_;
  open_tail_ = tail_;
  open_on_device_ = on_device_;
  open_hhead_ = hhead_;
  open_htail_ = htail_;
  open_on_file_ = on_file_;
  open_stamp_ = stamp_;
}

// ---- file tier: the pinned homes' recency list (head = most recently homed; only kept with the file tier) ----
void SlotCache::hpush(uint32_t k) {
  if (!c_.disk_tier) return;
  Entry& x = e_[k];
  x.hprev = kNil;
  x.hnext = hhead_;
  if (hhead_ != kNil) e_[hhead_].hprev = k;
  else htail_ = k;
  hhead_ = k;
  x.in_hlist = true;
}

void SlotCache::hunlink(uint32_t k) {
  if (!c_.disk_tier) return;
  Entry& x = e_[k];
  if (!x.in_hlist) broken("a pinned home outside the pinned recency list");
  if (x.hprev != kNil) e_[x.hprev].hnext = x.hnext;
  else hhead_ = x.hnext;
  if (x.hnext != kNil) e_[x.hnext].hprev = x.hprev;
  else htail_ = x.hprev;
  x.hprev = x.hnext = kNil;
  x.in_hlist = false;
}

void SlotCache::hpush_tail(uint32_t k) {  // the least recently homed: the first to drop to its file
  if (!c_.disk_tier) return;
  Entry& x = e_[k];
  x.hnext = kNil;
  x.hprev = htail_;
  if (htail_ != kNil) e_[htail_].hnext = k;
  else hhead_ = k;
  htail_ = k;
  x.in_hlist = true;
}

std::vector<uint32_t> SlotCache::host_order() const {
  std::vector<uint32_t> out;
  for (uint32_t k = hhead_; k != kNil; k = e_[k].hnext) out.push_back(k);
  return out;
}

// A unit that leaves the device or a bank slot without a write-back: its block (a clean copy, or the block it was
// served from) is its home again, else (file tier) its file.
void SlotCache::to_lower(uint32_t k, bool cold) {
  Entry& x = e_[k];
  x.slot = -1;
  if (x.backed) {
    x.backed = false;
    --backed_;
  }
  if (x.block >= 0) {
    x.home = Home::Host;
    if (cold) hpush_tail(k);
    else hpush(k);
  } else {
    if (!c_.disk_tier) broken("a unit without a block left the device without a write-back");
    x.home = Home::File;
    ++on_file_;
  }
}

// The least recently homed pinned unit (not skipped) goes to its file (no copy: the file holds its bytes); its block
// is free.
bool SlotCache::drop_host_lru(const std::vector<uint8_t>* skip, bool count) {
  if (!c_.disk_tier) return false;
  uint32_t k = htail_;
  while (k != kNil && skip && (*skip)[k]) k = e_[k].hprev;
  if (k == kNil) return false;
  Entry& x = e_[k];
  hunlink(k);
  free_blocks_.push_back(x.block);
  x.block = -1;
  x.home = Home::File;
  ++on_file_;
  if (count) ++st_.disk_drops;
  return true;
}

// The next staging buffer in rotation, once a read still holding it ended and its last copy landed.
int32_t SlotCache::take_stage() {
  const uint32_t i = stage_next_;
  stage_next_ = (i + 1) % c_.disk_staging;
  const int32_t block = int32_t(c_.blocks + i);
  end_reads([block](const Pending& p) { return p.stage == block; });
  if (stage_ev_[i] && !m_->done(stage_ev_[i])) {
    m_->event_sync(stage_ev_[i]);
    ++st_.disk_stage_waits;
  }
  return block;
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
  end_reads([&n](const Pending&) {
    if (n == 0) return false;
    --n;
    return true;
  });
}

void SlotCache::drain_demand() {
  end_reads([](const Pending& p) { return !p.prefetch; });
}

void SlotCache::drain_key(uint32_t k) {
  end_reads([k](const Pending& p) { return p.key == k; });
}

// The demand reads and the prefetch reads of units layer g routes (a wrong prediction's read keeps running).
void SlotCache::drain_layer(uint32_t g, const uint32_t* ids, uint32_t n) {
  const uint32_t first = key(g, 0);
  end_reads([this, g, ids, n, first](const Pending& p) {
    return !p.prefetch || (gated_of(p.key) == g && std::find(ids, ids + n, p.key - first) != ids + n);
  });
}

// The picked records leave pending_ (the others keep their order) and end oldest first. A read that failed is undone
// (its key back in its file, its slot back); after a failed copy every record left is undone and nothing more is
// enqueued. The first failure is rethrown.
void SlotCache::end_reads(const std::function<bool(const Pending&)>& pick) {
  if (pending_.empty()) return;
  std::vector<uint8_t> picked(pending_.size());
  for (size_t i = 0; i < pending_.size(); ++i) picked[i] = pick(pending_[i]) ? 1 : 0;
  std::vector<Pending> ending;
  ending.reserve(pending_.size());
  size_t kept = 0;
  for (size_t i = 0; i < pending_.size(); ++i) {
    if (picked[i]) ending.push_back(pending_[i]);
    else pending_[kept++] = pending_[i];
  }
  pending_.resize(kept);
  std::exception_ptr first;
  bool device_failed = false;
  for (size_t i = 0; i < ending.size(); ++i) {
    const Pending p = ending[i];
    if (p.entry != entries_) {  // it ran while its fetch's caller went on
      ++st_.disk_carried;
      st_.disk_carried_bytes += unit_bytes_;
    }
    const auto t0 = std::chrono::steady_clock::now();
    bool read_ok = true;
    try {
      st_.disk_read_ns += m_->read_end(p.handle);
    } catch (...) {
      read_ok = false;
      if (!first) first = std::current_exception();
    }
    st_.disk_wait_ns += uint64_t(
        std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count());
    if (!read_ok || device_failed) {
      undo_pending(p);
      continue;
    }
    ++st_.disk_reads;
    st_.disk_read_bytes += unit_bytes_;
    try {
      finish_pending(p);
    } catch (...) {
      if (!first) first = std::current_exception();
      device_failed = true;  // (this record stays fetched, as a synchronous fetch whose copy failed)
      ending.insert(ending.end(), pending_.begin(), pending_.end());
      pending_.clear();
    }
  }
  if (first) std::rethrow_exception(first);
}

// An ended read's device work: the copy from its staging buffer and the entry, the buffer's event, a prefetch's event.
void SlotCache::finish_pending(const Pending& p) {
  Entry& x = e_[p.key];
  if (mut_ == kEntryBeforeCopy) {  // test-only fault: the entry before its bytes
    publish(p.s, p.key, p.slot);
    m_->h2d(p.s, p.slot, p.stage, p.key);
  } else {
    m_->h2d(p.s, p.slot, p.stage, p.key);
    publish(p.s, p.key, p.slot);
  }
  void*& ev = stage_ev_[uint32_t(p.stage) - c_.blocks];  // the staging buffer is reusable once this copy landed
  if (!ev) ev = event();
  m_->record(ev, p.s);
  if (p.prefetch) {
    x.pf_done = event();
    m_->record(x.pf_done, p.s);
  }
}

// A read that failed: the key goes back to its file, its slot to where it came from (a bank slot stays used for the
// layer, unpublished); nothing was enqueued for it.
void SlotCache::undo_pending(const Pending& p) {
  Entry& x = e_[p.key];
  const uint32_t g = gated_of(p.key);
  table_[p.key] = -1;
  if (p.bank) {
    bank_key_[size_t(p.slot) - bank_first_] = kNil;
    banked_.erase(std::find(banked_.begin(), banked_.end(), p.key));
    --st_.bank_serves;
    --lc_[g].bank_serves;
  } else {
    unlink(p.key);
    --on_device_;
    coming_.erase(std::find(coming_.begin(), coming_.end(), p.key));
    free_slots_.push_back(p.slot);
    if (p.free_counted) --demand_free_used_;
  }
  x.home = Home::File;
  x.slot = -1;
  x.via_pf = x.used = false;
  ++on_file_;
  if (p.prefetch) {
    --st_.prefetched;
    --lc_[g].prefetched;
  } else {
    --st_.fetched;
    --lc_[g].fetched;
  }
}

// ---- the recency list (head = most recently used) ----
void SlotCache::unlink(uint32_t k) {
  Entry& x = e_[k];
  if (!x.listed) return;
  if (x.prev != kNil) e_[x.prev].next = x.next;
  else head_ = x.next;
  if (x.next != kNil) e_[x.next].prev = x.prev;
  else tail_ = x.prev;
  x.prev = x.next = kNil;
  x.listed = false;
}

void SlotCache::push_front(uint32_t k) {
  Entry& x = e_[k];
  x.prev = kNil;
  x.next = head_;
  if (head_ != kNil) e_[head_].prev = k;
  else tail_ = k;
  head_ = k;
  x.listed = true;
  if (c_.scored) {  // unique stamps, larger nearer the head (stamp_room keeps the counter far from wrapping)
    if (stamp_ == UINT64_MAX) broken("the recency stamp counter wrapped");
    x.lru_stamp = ++stamp_;
  }
}

void SlotCache::stamp_room(const char* what) const {
  if (c_.scored && stamp_ > kStampLimit)
    fail(SS_E_BACKEND, std::string("device-gated: ") + what +
                           ": the scored eviction's recency stamp counter is exhausted (reopen the context)");
}

void* SlotCache::event() {
  if (!pool_.empty()) {
    void* ev = pool_.back();
    pool_.pop_back();
    return ev;
  }
  void* ev = m_->event_create();
  all_events_.push_back(ev);
  return ev;
}

void SlotCache::publish(Mover::Stream s, uint32_t k, int32_t v) {
  table_[k] = v;
  m_->publish(s, k, v);
}

// Finished write-backs in submission order: the unit's home becomes its block and its slot is free; a discarded one
// (the unit was resurrected) only returns its block.
uint32_t SlotCache::collect() {
  uint32_t n = 0;
  while (!wbs_.empty()) {
    Writeback& w = wbs_.front();
    if (!m_->done(w.done)) break;
    Entry& x = e_[w.key];
    x.wb_pending = false;
    if (w.discard) {
      free_blocks_.push_back(w.block);
    } else {
      x.home = Home::Host;
      x.block = w.block;
      x.slot = -1;
      hpush(w.key);
      free_slots_.push_back(w.slot);
    }
    ++n;
    outstanding_ -= w.bytes;
    st_.wb_completed_bytes += w.bytes;
    pool_.push_back(w.done);
    wbs_.pop_front();
  }
  st_.writebacks_done += n;
  return n;
}

void SlotCache::submit_part(Deferred& d) {
  const uint32_t p = d.parts_done;
  m_->d2h(wb_stream_, d.slot, d.block, int32_t(p), d.key);
  ++d.parts_done;
  const uint64_t b = m_->part_bytes(p);
  d.bytes += b;
  outstanding_ += b;
  st_.wb_issued_bytes += b;
}

void* SlotCache::record_front(bool discard) {
  Deferred& d = deferred_.front();
  void* ev = event();
  m_->record(ev, wb_stream_);
  wbs_.push_back({d.key, d.slot, d.block, ev, discard, d.bytes});
  deferred_.pop_front();
  return ev;
}

void* SlotCache::finish_front() {
  Deferred& d = deferred_.front();
  while (d.parts_done < m_->parts()) submit_part(d);
  return record_front(false);
}

void SlotCache::issue_writebacks(uint32_t g, const std::function<bool()>& ahead) {
  enter();
  if (deferred_.empty()) {
    credit_ = 0;
    return;
  }
  if (g + 1 >= gated()) return;  // never behind the last layer: the boundary's sync would wait for it
  const int64_t grant = int64_t(layer_bytes_);
  credit_ = std::min(credit_ + grant, grant);  // a debt carries over, unused credit does not
  st_.collected_mid += collect();
  bool behind_ready = false;
  while (credit_ > 0 && !deferred_.empty() && outstanding_ < max_outstanding_ && !(ahead && ahead())) {
    if (wb_stream_ == Mover::kD2h && !behind_ready) {
      m_->record(post_ready_ev_, Mover::kDem);
      m_->wait(Mover::kD2h, post_ready_ev_);
      behind_ready = true;
    }
    Deferred& d = deferred_.front();
    credit_ -= int64_t(m_->part_bytes(d.parts_done));
    if (d.parts_done + 1 == m_->parts()) finish_front();
    else submit_part(d);
  }
}

// A demand with no free slot while write-backs are deferred: wait for the oldest live write-back in flight (or finish
// the deferred front and wait for it) until a slot is free.
void SlotCache::force_free_slot() {
  while (free_slots_.empty() && !deferred_.empty()) {
    void* ev = nullptr;
    for (const Writeback& w : wbs_)
      if (!w.discard) {
        ev = w.done;
        break;
      }
    if (!ev) ev = finish_front();
    ++st_.wb_forced;
    const auto t0 = std::chrono::steady_clock::now();
    m_->event_sync(ev);
    st_.wb_forced_wait_ns += uint64_t(
        std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count());
    st_.collected_mid += collect();
  }
}

// Bank g & 1 of the demand bank slots; a bank is reused two gated layers later, when the device has finished the
// layer that used it before. The slot's previous unit goes back to its block and its entry is withdrawn first.
int32_t SlotCache::bank_slot(uint32_t g) {
  const uint32_t b = g & 1u;
  if (bank_seq_[b] != seq_ || bank_layer_[b] != g) {
    bank_seq_[b] = seq_;
    bank_layer_[b] = g;
    bank_next_[b] = 0;
  }
  if (bank_next_[b] >= c_.bank_slots) return -1;
  const uint32_t idx = b * c_.bank_slots + bank_next_[b]++;
  const int32_t slot = int32_t(bank_first_ + idx);
  const uint32_t old = bank_key_[idx];
  if (old != kNil && e_[old].home == Home::Bank && e_[old].slot == slot) {
    drain_key(old);  // (its read, were it still in flight, ends before the alias goes)
    to_lower(old);  // its block, or (read from it) its file
    publish(Mover::kDem, old, -1);
  }
  bank_key_[idx] = kNil;
  return slot;
}

void SlotCache::begin_token(uint32_t seq, const std::vector<uint8_t>* run) {
  require(!run || run->size() == gated(), SS_E_INVALID, "device-gated: the exported layers do not cover the gated layers");
  enter();
  if (run) std::copy(run->begin(), run->end(), run_.begin());
  else std::fill(run_.begin(), run_.end(), uint8_t(1));
  if (c_.scored) {  // the token's epoch (the first is 1); one token cannot push more than 2^40 stamps
    stamp_room("begin_token");
    require(epoch_ < (uint64_t(1) << 63), SS_E_BACKEND, "device-gated: the scored eviction's epoch counter is exhausted");
    ++epoch_;
  }
  seq_ = seq;
  pf_token_ = 0;
  demand_free_used_ = 0;
  std::fill(pf_layer_.begin(), pf_layer_.end(), 0u);
  std::fill(layer_missed_.begin(), layer_missed_.end(), uint8_t(0));
  pred_.clear();
  pred_layer_ = kNil;
}

bool SlotCache::fetch(uint32_t g, uint32_t unit, bool prefetch) {
  const uint32_t k = key(g, unit);
  Entry& x = e_[k];
  if (prefetch && (pf_layer_[g] >= c_.prefetch_per_layer || pf_token_ >= c_.prefetch_per_token)) return false;
  if (prefetch && c_.no_admit) return false;  // (no_admit issues no prefetch)
  switch (x.home) {
    case Home::Coming:
      drain_key(k);  // (its own prefetch read in flight: ended)
      return false;
    case Home::Device:
    case Home::Bank:
      return false;
    case Home::Evicting: {  // resurrection: the slot still holds the bytes (a write-back only reads them)
      for (auto it = deferred_.begin(); it != deferred_.end(); ++it) {
        if (it->key != k) continue;
        if (it->parts_done == 0) {  // nothing submitted: cancelled, its block free again
          free_blocks_.push_back(it->block);
          deferred_.erase(it);
          x.wb_pending = false;
          ++st_.wb_cancelled;
          st_.wb_cancelled_bytes += unit_bytes_;
        } else {  // partly submitted (only the front can be): recorded as a discard
          if (it != deferred_.begin()) broken("parts submitted behind the deferred front");
          st_.wb_cancelled_bytes += unit_bytes_ - it->bytes;
          record_front(true);
        }
        x.home = Home::Device;
        x.block = -1;
        publish(Mover::kDem, k, x.slot);
        push_front(k);
        ++on_device_;
        ++st_.resurrected;
        return true;
      }
      for (Writeback& w : wbs_)
        if (w.key == k && !w.discard) {
          w.discard = true;
          break;
        }
      x.home = Home::Device;
      x.block = -1;
      publish(Mover::kDem, k, x.slot);
      push_front(k);
      ++on_device_;
      ++st_.resurrected;
      return true;
    }
    case Home::Host:
      break;
    case Home::File:  // a file read below; a prefetch only with disk_prefetch
      if (prefetch && !c_.disk_prefetch) return false;
      break;
  }
  // a prefetch keeps the reserve free (pf_strict: the spare target's slots too)
  const size_t reserve =
      prefetch ? (c_.pf_strict ? std::max<size_t>(c_.prefetch_reserve, c_.spare_target) : c_.prefetch_reserve) : 0u;
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
  if (bank) {
    // (no_admit: taken above)
  } else if (!capped && free_slots_.size() > reserve) {
    if (!prefetch) ++demand_free_used_;
    free_counted = !prefetch;
    slot = free_slots_.back();
    free_slots_.pop_back();
  } else if (prefetch) {
    if (c_.pf_strict && free_slots_.size() > c_.prefetch_reserve) ++st_.pf_strict_refused;
    return false;
  } else {
    slot = bank_slot(g);
    if (slot >= 0) {
      bank = true;
    } else {  // more distinct misses than a bank holds: only an internal error gets here
      drain_pending();
      force_free_slot();
      while (free_slots_.empty() && !wbs_.empty()) {
        m_->event_sync(wbs_.front().done);
        collect();
        ++st_.stalled;
      }
      if (free_slots_.empty()) fail(SS_E_BACKEND, "device-gated: no free slot, no bank slot, no write-back to wait for");
      slot = free_slots_.back();
      free_slots_.pop_back();
    }
  }
  const Mover::Stream s = prefetch ? Mover::kPf : Mover::kDem;
  const bool from_file = x.home == Home::File;
  if (from_file) {  // its bytes from the file into a staging buffer, then the same copy once the read ended
    const size_t depth = std::max<uint32_t>(c_.disk_queue, 1);
    try {
      if (pending_.size() >= depth) {  // a full queue: the completed reads, then the oldest demand reads, then the oldest
        end_reads([this](const Pending& p) { return m_->read_done(p.handle); });
        if (pending_.size() >= depth) {
          size_t n = pending_.size() + 1 - depth;
          end_reads([&n](const Pending& p) {
            if (n == 0 || p.prefetch) return false;
            --n;
            return true;
          });
        }
        if (pending_.size() >= depth) drain_pending(pending_.size() + 1 - depth);
      }
      const int32_t stage = take_stage();
      const auto t0 = std::chrono::steady_clock::now();
      void* h = m_->read_begin(k, stage);
      st_.disk_read_ns += uint64_t(
          std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count());
      if (!pending_.empty()) ++st_.disk_overlapped;
      pending_.push_back({k, slot, stage, s, prefetch, bank, free_counted, h, entries_});
      st_.disk_max_in_flight = std::max<uint64_t>(st_.disk_max_in_flight, pending_.size());
    } catch (...) {  // nothing begun for this key: its slot goes back (a bank slot stays used, unpublished)
      if (!bank) {
        free_slots_.push_back(slot);
        if (free_counted) --demand_free_used_;
      }
      throw;
    }
    table_[k] = slot;  // the mirror now; the device's entry with the copy
    --on_file_;
  } else {
    if (mut_ == kEntryBeforeCopy) {  // test-only fault: the entry before its bytes
      publish(s, k, slot);
      m_->h2d(s, slot, x.block, k);
    } else {
      m_->h2d(s, slot, x.block, k);
      publish(s, k, slot);
    }
    hunlink(k);  // (a Host unit: out of the pinned recency list)
  }
  x.slot = slot;
  x.via_pf = prefetch;
  x.used = false;
  if (prefetch && !from_file) {  // (a file read's: with its copy)
    x.pf_done = event();
    m_->record(x.pf_done, s);
  }
  if (bank) {
    x.home = Home::Bank;
    bank_key_[size_t(slot) - bank_first_] = k;
    banked_.push_back(k);
    ++st_.bank_serves;
    ++lc_[g].bank_serves;
  } else {
    x.home = Home::Coming;
    coming_.push_back(k);
    push_front(k);
    ++on_device_;
  }
  if (prefetch) {
    ++st_.prefetched;
    ++lc_[g].prefetched;
    ++pf_layer_[g];
    ++pf_token_;
  } else {
    ++st_.fetched;
    ++lc_[g].fetched;
  }
  if (from_file && c_.disk_queue <= 1) drain_pending();  // synchronous reads: the copy now
  return true;
}

void SlotCache::cover(uint32_t g, uint32_t unit) {
  Entry& x = e_[key(g, unit)];
  // only this key's copy lands before the ready: its read ends first if in flight (a file prefetch's event comes
  // with its copy), the wait is on its own event
  if (x.home == Home::Coming && x.via_pf && mut_ != kNoCover) drain_key(key(g, unit));
  if (x.home == Home::Coming && x.via_pf && x.pf_done && mut_ != kNoCover) {
    m_->wait(Mover::kDem, x.pf_done);
    ++st_.covered_waits;
  }
}

void SlotCache::use(uint32_t g, uint32_t unit, bool was_miss) {
  enter();
  const uint32_t k = key(g, unit);
  Entry& x = e_[k];
  ++st_.lookups;
  ++lc_[g].lookups;
  if (was_miss) {
    ++st_.misses;
    ++lc_[g].misses;
    if (!layer_missed_[g]) {
      layer_missed_[g] = 1;
      ++st_.miss_layers;
    }
  }
  if (c_.scored) x.demand_epoch = epoch_;  // a routed use (never a prefetch, a resurrection or a seed)
  if (x.via_pf && !x.used) {
    x.used = true;
    ++st_.prefetch_used;
    ++lc_[g].prefetch_used;
  }
  if (x.listed) {
    unlink(k);
    push_front(k);
  }
}

void SlotCache::serve_demand(uint32_t g, const uint32_t* ids, uint32_t n, uint64_t mask) {
  enter();
  const uint32_t nu = units(g);
  for (uint32_t i = 0; i < n; ++i)
    require(ids[i] < nu, SS_E_INVALID,
            "device-gated: layer " + std::to_string(g) + " exported id " + std::to_string(ids[i]) + " of " +
                std::to_string(nu));
  if (mask) m_->diag_mark(g, 0);
  // masked occurrences in export order: a repeated id is fetched at its first occurrence, covered at the others
  for (uint32_t i = 0; i < n; ++i) {
    if (!(mask >> i & 1u)) continue;
    const Home h = e_[key(g, ids[i])].home;
    if (h == Home::Device || h == Home::Coming || h == Home::Bank) {
      cover(g, ids[i]);
      ++st_.covered;
    } else {
      fetch(g, ids[i], false);
    }
  }
  drain_layer(g, ids, n);  // this layer's copies and entries (its demand reads, the prefetch reads it routes)
  if (mask) {
    drain_demand();  // (the ready follows every demand read's copy and entry)
    m_->ready(g, seq_);
    m_->diag_mark(g, 1);
  }
}

void SlotCache::serve_use(uint32_t g, const uint32_t* ids, uint32_t n, uint64_t mask) {
  enter();
  const bool have_pred = pred_layer_ == g;
  uniq_.assign(ids, ids + n);
  std::sort(uniq_.begin(), uniq_.end());
  uniq_.erase(std::unique(uniq_.begin(), uniq_.end()), uniq_.end());
  if (c_.scored) score_history(g);  // (the union saved before a prediction reuses uniq_)
  for (uint32_t id : uniq_) {  // placement rounds: the tokens that routed the unit since the last round
    uint32_t& h = rhits_[key(g, id)];
    if (h != UINT32_MAX) ++h;
  }
  for (uint32_t id : uniq_) {
    bool miss = false;
    for (uint32_t i = 0; i < n; ++i)
      if (ids[i] == id && (mask >> i & 1u)) miss = true;
    use(g, id, miss);
    if (have_pred && std::find(pred_.begin(), pred_.end(), id) != pred_.end()) ++st_.predicted_true;
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
    if (pred[i] >= nu) {
      ++st_.pred_invalid;
      continue;
    }
    if (std::find(uniq_.begin(), uniq_.end(), pred[i]) == uniq_.end()) uniq_.push_back(pred[i]);
  }
  st_.predicted += uniq_.size();
  pred_.assign(uniq_.begin(), uniq_.end());
  pred_layer_ = g_next;
  for (uint32_t id : pred_) fetch(g_next, id, true);
}

void SlotCache::end_token(const std::vector<uint32_t>& keep, uint32_t rows) {
  drain_pending();  // the end of the token: no read in flight while its streams sync and victims are chosen
  m_->sync(Mover::kDem);
  m_->sync(Mover::kPf);
  std::vector<uint8_t> kept;
  if (!keep.empty()) {
    kept.assign(keys_, 0);
    for (uint32_t k : keep)
      if (k < keys_) kept[k] = 1;
  }
  auto keep_k = [&](uint32_t k) { return !kept.empty() && kept[k]; };
  for (uint32_t k : coming_) {  // arrivals become device homes; their source blocks are free
    Entry& x = e_[k];
    if (x.home != Home::Coming) continue;
    if (c_.pf_revert && x.via_pf && !x.used && !keep_k(k)) {
      // an unused prefetch goes back: to its source block (still holding the bytes) at the pinned recency tail, or
      // (read from it) to its file; no write-back, and the table upload below withdraws its entry
      ++st_.pf_reverted;
      st_.pf_revert_bytes += unit_bytes_;
      free_slots_.push_back(x.slot);
      to_lower(k, true);
      table_[k] = -1;
      unlink(k);
      --on_device_;
      x.via_pf = false;
      if (x.pf_done) {
        pool_.push_back(x.pf_done);
        x.pf_done = nullptr;
      }
      continue;
    }
    x.home = Home::Device;
    x.via_pf = false;
    if (x.pf_done) {
      pool_.push_back(x.pf_done);
      x.pf_done = nullptr;
    }
    if (x.block >= 0) {  // (a unit read from its file holds none)
      if (backed_ < c_.inclusive) {  // inclusive share: the source block stays as a clean copy of the slot's bytes
        x.backed = true;
        ++backed_;
        ++st_.inclusive_kept;
      } else {
        free_blocks_.push_back(x.block);
        x.block = -1;
      }
    }
  }
  coming_.clear();
  for (uint32_t k : banked_) {  // bank units go back to their blocks (or, read from it, their file)
    Entry& x = e_[k];
    if (x.home == Home::Bank) {
      to_lower(k);
      table_[k] = -1;
    }
    if (x.pf_done) {
      pool_.push_back(x.pf_done);
      x.pf_done = nullptr;
    }
    x.via_pf = false;
  }
  banked_.clear();
  std::fill(bank_key_.begin(), bank_key_.end(), kNil);
  bank_seq_[0] = bank_seq_[1] = 0;
  bank_layer_[0] = bank_layer_[1] = kNil;
  collect();
  size_t pending = deferred_.size();
  for (const Writeback& w : wbs_) pending += w.discard ? 0u : 1u;
  const size_t base = free_slots_.size() + pending;
  victims_.clear();
  size_t got = 0;
  bool short_blocks = false;
  auto eligible = [&](uint32_t k) {
    const Entry& x = e_[k];
    return x.home == Home::Device && !x.wb_pending && !(kept.size() && kept[k]);
  };
  auto accept = [&](uint32_t k) {
    Entry& x = e_[k];
    // a clean copy (its block is its home again) or, file tier with no block to free, its file: no copy; a pinned
    // unit dropped to its file frees a block first when none is free (clean_evict: none is dropped for it)
    const bool clean = !x.backed && clean_now();
    if (x.backed || clean || (free_blocks_.empty() && !drop_host_lru() && c_.disk_tier)) {
      if (x.backed) ++st_.inclusive_drops;
      else ++st_.disk_discards;
      if (clean) count_clean();
      unlink(k);
      --on_device_;
      free_slots_.push_back(x.slot);
      to_lower(k);
      table_[k] = -1;
      ++st_.evicted;
      ++lc_[gated_of(k)].evicted;
      ++got;
      return true;
    }
    if (free_blocks_.empty()) {
      ++st_.evict_short;
      short_blocks = true;
      return false;
    }
    const int32_t b = free_blocks_.back();
    free_blocks_.pop_back();
    unlink(k);
    --on_device_;
    x.home = Home::Evicting;
    x.block = b;
    x.wb_pending = true;
    table_[k] = -1;
    victims_.push_back(k);
    ++got;
    return true;
  };
  // scored eviction: the lowest scores among the eligible units, when every gated layer was closed this token (a
  // layer the token did not export is closed here from its unchanged history); else the recency tail
  const bool select = !c_.no_admit;  // (no_admit: nothing was admitted, no boundary evicts)
  const bool want_score = select && c_.scored && (!c_.scored_auto || rows > 1);
  for (uint32_t g = 0; c_.scored && g < gated(); ++g)
    if (!run_[g]) sc_[g].list_epoch = epoch_;
  bool by_score = want_score;
  for (uint32_t g = 0; by_score && g < gated(); ++g) by_score = sc_[g].list_epoch == epoch_;
  if (want_score && !by_score) ++st_.score_fallbacks;
  if (by_score) {
    const auto t0 = std::chrono::steady_clock::now();
    select_scored(c_.spare_target > base ? c_.spare_target - base : 0, eligible);
    for (const ScoreCand& cd : select_heap_) {
      if (!accept(cd.key)) break;
      ++st_.scored_victims;
    }
    st_.score_ns += uint64_t(
        std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count());
  } else if (select) {
    for (uint32_t k = tail_; k != kNil && base + got < c_.spare_target;) {
      const uint32_t prev = e_[k].prev;
      if (eligible(k) && !accept(k)) break;
      k = prev;
    }
  }
  if (select && pressure_ && pressure_recent_ && !short_blocks) {  // test pressure: the most recent ones too
    uint32_t n = 0;
    for (uint32_t k = head_; k != kNil && n < pressure_recent_;) {
      const uint32_t next = e_[k].next;
      if (eligible(k)) {
        if (!accept(k)) break;
        ++n;
      }
      k = next;
    }
  }
  const size_t n_evict = victims_.size();
  m_->upload_table(table_.data(), keys_);  // the table first, then the write-backs behind it
  const size_t n_old = deferred_.size(), carry = std::max(n_evict, prev_evict_);
  const size_t n_flush = n_old > carry ? n_old - carry : 0;
  prev_evict_ = n_evict;
  credit_ = 0;
  for (size_t i = 0; c_.wb_defer && i < n_evict; ++i) {
    const uint32_t k = victims_[i];
    deferred_.push_back({k, e_[k].slot, e_[k].block, 0, 0});
    ++st_.wb_deferred;
    ++st_.evicted;
    ++lc_[gated_of(k)].evicted;
  }
  const uint64_t issued0 = st_.wb_issued_bytes;
  for (size_t i = 0; i < n_flush; ++i) finish_front();
  st_.wb_boundary_flushed += n_flush;
  st_.wb_boundary_flushed_bytes += st_.wb_issued_bytes - issued0;
  for (size_t i = 0; !c_.wb_defer && i < n_evict; ++i) {
    const uint32_t k = victims_[i];
    const Entry& x = e_[k];
    m_->d2h(Mover::kD2h, x.slot, x.block, -1, k);
    void* ev = event();
    m_->record(ev, Mover::kD2h);
    wbs_.push_back({k, x.slot, x.block, ev, false, unit_bytes_});
    outstanding_ += unit_bytes_;
    st_.wb_issued_bytes += unit_bytes_;
    ++st_.evicted;
    ++lc_[gated_of(k)].evicted;
  }
  ++st_.tokens;
}

// ---- scored eviction ----
// Layer g's union of this token (uniq_, sorted) against the previous token's: every (r in the previous union, e in
// this one) cell takes one saturating increment and its row sum with it; the union enters the window ring (the oldest
// leaves it once 16 are held) and becomes the previous one.
void SlotCache::score_history(uint32_t g) {
  LayerScore& l = sc_[g];
  const uint32_t n = units(g);
  require(uniq_.size() <= c_.max_ids, SS_E_BACKEND, "device-gated: a score union above max ids");
  l.cur.assign(uniq_.begin(), uniq_.end());
  l.served = epoch_;
  for (uint32_t r : l.prev) {
    uint32_t* row = l.T.data() + size_t(r) * n;
    for (uint32_t e : l.cur) {
      if (row[e] == UINT32_MAX) {
        ++st_.score_saturated;
        continue;
      }
      ++row[e];
      ++l.rowsum[r];
    }
  }
  if (l.ring_n == kWindow) {
    const uint32_t* old = l.ring.data() + size_t(l.ring_head) * c_.max_ids;
    for (uint32_t i = 0; i < l.ring_len[l.ring_head]; ++i) --l.cnt[old[i]];
    l.ring_head = (l.ring_head + 1) % kWindow;
    --l.ring_n;
  }
  const uint32_t at = (l.ring_head + l.ring_n) % kWindow;
  std::copy(l.cur.begin(), l.cur.end(), l.ring.begin() + ptrdiff_t(size_t(at) * c_.max_ids));
  l.ring_len[at] = uint8_t(l.cur.size());
  ++l.ring_n;
  for (uint32_t e : l.cur) ++l.cnt[e];
  l.prev.assign(l.cur.begin(), l.cur.end());
}

void SlotCache::score_layer(uint32_t g) {
  enter();
  if (!c_.scored || g >= gated() || sc_[g].served != epoch_) return;  // (not served: the boundary falls back)
  sc_[g].list_epoch = epoch_;
}

// Unit u of layer g with cur = this token's union: N = sum over r in cur of T[r][u], D = sum over cur of the row
// sums, P = ((|cur| N) << 16) / max(1, D), F = (cnt[u] << 16) / 16, Rec = (1 << 16) / (1 + epoch - demand_epoch),
// S = w_t P + w_f F + w_r Rec in unsigned floor arithmetic (N <= D, so P <= |cur| << 16 and S < 2^33). With a cutoff
// that F and Rec alone cannot beat, the transition rows are not read.
SlotCache::ScoreCand SlotCache::score_candidate(uint32_t g, uint32_t u, uint64_t D, const ScoreCand* cutoff) const {
  const LayerScore& l = sc_[g];
  const Entry& x = e_[base_[g] + u];
  const uint64_t F = (uint64_t(l.cnt[u]) << 16) / kWindow;
  const uint64_t R = (uint64_t(1) << 16) / (1 + (epoch_ - x.demand_epoch));
  ScoreCand cd{uint64_t(c_.w_freq) * F + uint64_t(c_.w_rec) * R, x.demand_epoch, x.lru_stamp, base_[g] + u};
  if (cutoff && !cand_less(cd, *cutoff)) return cd;
  uint64_t N = 0;
  for (uint32_t r : l.cur) N += l.T[size_t(r) * units(g) + u];
  const uint64_t P = ((uint64_t(l.cur.size()) * N) << 16) / std::max<uint64_t>(1, D);
  cd.s += uint64_t(c_.w_trans) * P;
  return cd;
}

// The `need` lowest candidates (cand_less) of every gated layer's eligible units, ascending in select_heap_: a bounded
// max-heap over all layers, scored from each layer's current union, epochs and stamps.
void SlotCache::select_scored(size_t need, const std::function<bool(uint32_t)>& eligible, bool count) {
  select_heap_.clear();
  for (uint32_t g = 0; need && g < gated(); ++g) {
    uint64_t D = 0;
    for (uint32_t r : sc_[g].cur) D += sc_[g].rowsum[r];
    if (count) ++st_.score_layers;
    for (uint32_t u = 0; u < units(g); ++u) {
      if (!eligible(base_[g] + u)) continue;
      if (count) ++st_.score_candidates;
      const ScoreCand cd = score_candidate(g, u, D, select_heap_.size() == need ? &select_heap_.front() : nullptr);
      if (select_heap_.size() < need) {
        select_heap_.push_back(cd);
        std::push_heap(select_heap_.begin(), select_heap_.end(), cand_less);
      } else if (cand_less(cd, select_heap_.front())) {
        std::pop_heap(select_heap_.begin(), select_heap_.end(), cand_less);
        select_heap_.back() = cd;
        std::push_heap(select_heap_.begin(), select_heap_.end(), cand_less);
      }
    }
  }
  std::sort_heap(select_heap_.begin(), select_heap_.end(), cand_less);
}

// The open state of every score table: the profile's counts (or zeros), an empty window, no union, epoch 0, the
// open's stamps.
void SlotCache::reset_score() {
  for (uint32_t g = 0; g < uint32_t(sc_.size()); ++g) {
    LayerScore& l = sc_[g];
    const uint32_t n = units(g);
    if (l.open_T.empty()) std::fill(l.T.begin(), l.T.end(), 0u);
    else std::copy(l.open_T.begin(), l.open_T.end(), l.T.begin());
    for (uint32_t r = 0; r < n; ++r) {
      uint64_t sum = 0;
      for (uint32_t e = 0; e < n && !l.open_T.empty(); ++e) sum += l.T[size_t(r) * n + e];
      l.rowsum[r] = sum;
    }
    std::fill(l.cnt.begin(), l.cnt.end(), uint16_t(0));
    std::fill(l.ring.begin(), l.ring.end(), 0u);
    std::fill(l.ring_len.begin(), l.ring_len.end(), uint8_t(0));
    l.ring_head = l.ring_n = 0;
    l.prev.clear();
    l.cur.clear();
    l.served = l.list_epoch = 0;
  }
  epoch_ = 0;
  stamp_ = open_stamp_;
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
  stamp_ = 0;
  for (uint32_t k = tail_; k != kNil; k = e_[k].prev) e_[k].lru_stamp = ++stamp_;
}

void SlotCache::load_counts(const std::vector<std::vector<uint32_t>>& cells) {
  require(c_.scored && cells.size() == sc_.size(), SS_E_INVALID, "device-gated: a score profile needs policy SCORED");
  for (uint32_t g = 0; g < gated(); ++g) {
    LayerScore& l = sc_[g];
    const uint32_t n = units(g);
    require(cells[g].size() == size_t(n) * n, SS_E_INVALID, "device-gated: a profile layer is not units^2 counts");
    l.T = cells[g];
    for (uint32_t r = 0; r < n; ++r) {
      uint64_t sum = 0;
      for (uint32_t e = 0; e < n; ++e) sum += l.T[size_t(r) * n + e];
      l.rowsum[r] = sum;
    }
    l.open_T = l.T;  // the reset_open state
  }
}

// ---- kept-resident layers (ss_dg_make_resident) ----
SlotCache::ResidentResult SlotCache::make_resident(uint32_t g, const std::vector<uint32_t>& ids,
                                                   const std::vector<uint32_t>& other_kept) {
  const auto t0 = std::chrono::steady_clock::now();
  require(g < gated(), SS_E_INVALID, "ss_dg_make_resident: gated layer out of range");
  std::vector<uint8_t> want(keys_, 0), other(keys_, 0);
  for (uint32_t u : ids) {
    require(u < units(g), SS_E_INVALID, "ss_dg_make_resident: id out of range");
    require(!want[key(g, u)], SS_E_INVALID, "ss_dg_make_resident: duplicate id " + std::to_string(u));
    want[key(g, u)] = 1;
  }
  size_t n_other = 0;
  for (uint32_t k : other_kept)
    if (k < keys_ && !other[k] && !want[k]) {
      other[k] = 1;
      ++n_other;
    }
  // capacity: every layer's kept units leave the spare target free for the boundaries
  const uint64_t cap = uint64_t(c_.persistent_slots) - c_.spare_target;
  require(ids.size() + n_other <= cap, SS_E_CAPACITY,
          "ss_dg_make_resident: " + std::to_string(ids.size()) + " units of gated layer " + std::to_string(g) + " + " +
              std::to_string(n_other) + " other kept units + the spare target " + std::to_string(c_.spare_target) +
              " exceed the " + std::to_string(c_.persistent_slots) + " persistent slots");
  size_t need = 0, eligible_n = 0, evicting = 0, discarded = 0;
  for (uint32_t k = 0; k < keys_; ++k) {
    const Entry& x = e_[k];
    require(x.home != Home::Bank, SS_E_BACKEND, "ss_dg_make_resident: a bank unit between tokens");
    if (x.home == Home::Evicting) ++evicting;
    if (want[k]) need += x.home != Home::Device && x.home != Home::Coming ? 1u : 0u;
    else if (x.home == Home::Device && !other[k]) ++eligible_n;
  }
  for (const Writeback& w : wbs_) discarded += w.discard ? 1u : 0u;
  const size_t free_after = free_slots_.size() + evicting;
  require(need <= free_after + eligible_n, SS_E_CAPACITY,
          "ss_dg_make_resident: " + std::to_string(need) + " units to copy in, " + std::to_string(free_after) +
              " free slots and " + std::to_string(eligible_n) +
              " evictable units (the rest hold other layers' kept units or prefetches in flight)");
  require(c_.disk_tier || need <= free_after || free_after + free_blocks_.size() + discarded > 0, SS_E_CAPACITY,
          "ss_dg_make_resident: no free slot and no free pinned block to start the write-backs");
  stamp_room("ss_dg_make_resident");
  drain();  // everything settled: reads, copies, deferred and recorded write-backs collected
  for (const Writeback& w : wbs_) m_->event_sync(w.done);
  collect();
  if (!wbs_.empty()) broken("ss_dg_make_resident: write-backs not collected");

  ResidentResult r;
  std::vector<uint32_t> in;  // the units to copy in, in the caller's order
  for (uint32_t u : ids) {
    const uint32_t k = key(g, u);
    Entry& x = e_[k];
    if (x.home == Home::Coming) {  // a prefetch whose copy landed: admitted now
      x.home = Home::Device;
      x.via_pf = false;
      if (x.pf_done) {
        pool_.push_back(x.pf_done);
        x.pf_done = nullptr;
      }
      if (x.block >= 0) {
        free_blocks_.push_back(x.block);
        x.block = -1;
      }
    } else if (x.home != Home::Device) {
      in.push_back(k);
    }
  }
  auto eligible = [&](uint32_t k) {
    const Entry& x = e_[k];
    return x.home == Home::Device && !x.wb_pending && !want[k] && !other[k];
  };
  std::vector<uint32_t> victims;
  const size_t n_vict = in.size() > free_slots_.size() ? in.size() - free_slots_.size() : 0;
  if (n_vict && c_.scored) {
    select_scored(n_vict, eligible, false);
    for (const ScoreCand& cd : select_heap_) victims.push_back(cd.key);
  } else {
    for (uint32_t k = tail_; k != kNil && victims.size() < n_vict; k = e_[k].prev)
      if (eligible(k)) victims.push_back(k);
  }
  if (victims.size() != n_vict) broken("ss_dg_make_resident: fewer victims than the capacity check counted");

  std::vector<uint8_t> hold = want;  // never dropped to a file here: the units to copy in, this call's write-backs
  std::vector<int32_t> released;     // source blocks of committed copies (free once the demand stream synced)
  std::vector<int32_t> wb;           // slots of written-back victims (free once the write-back stream synced)
  struct Read {
    uint32_t key;
    int32_t slot, stage;
    void* handle;
  };
  std::deque<Read> reads;  // file reads in flight, oldest first, each in its own staging buffer
  const size_t depth = c_.disk_tier ? std::max<size_t>(1, std::min<size_t>(std::max<uint32_t>(c_.disk_queue, 1),
                                                                          c_.disk_staging))
                                    : 1;
  bool io_error = false;
  // the committed units become the most recent in the order of `in` on every exit
  struct Recent {
    SlotCache* cache;
    const std::vector<uint32_t>& order;
    std::vector<uint8_t> done;
    ~Recent() {
      for (size_t i = 0; i < order.size(); ++i)
        if (done[i]) cache->push_front(order[i]);
    }
  } recent{this, in, std::vector<uint8_t>(in.size(), 0)};
  std::vector<int32_t> in_pos(keys_, -1);
  for (size_t i = 0; i < in.size(); ++i) in_pos[in[i]] = int32_t(i);
  auto commit = [&](uint32_t k, int32_t slot) {
    Entry& x = e_[k];
    x.home = Home::Device;
    x.slot = slot;
    x.block = -1;
    recent.done[size_t(in_pos[k])] = 1;
    ++on_device_;
    ++r.copied;
  };
  auto transfer = [&](uint32_t k, int32_t slot, int32_t src) {  // the copy and its entry, or nothing owned changes
    try {
      m_->h2d(Mover::kDem, slot, src, k);
      publish(Mover::kDem, k, slot);
    } catch (...) {
      table_[k] = -1;
      free_slots_.push_back(slot);
      throw;
    }
  };
  auto flush_dem = [&] {
    m_->sync(Mover::kDem);
    free_blocks_.insert(free_blocks_.end(), released.begin(), released.end());
    released.clear();
  };
  auto flush_d2h = [&] {
    if (wb.empty()) return;
    m_->sync(Mover::kD2h);
    free_slots_.insert(free_slots_.end(), wb.begin(), wb.end());
    wb.clear();
  };
  uint64_t n_read = 0, n_wb = 0, read_ns = 0;
  auto timed = [&](const std::chrono::steady_clock::time_point& a) {
    read_ns += uint64_t(
        std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - a).count());
  };
  auto end_read = [&](size_t i) {  // a read's end: its copy and entry, its staging buffer's event
    const Read rd = reads[i];
    reads.erase(reads.begin() + std::ptrdiff_t(i));
    const auto ta = std::chrono::steady_clock::now();
    try {
      m_->read_end(rd.handle);
    } catch (...) {
      timed(ta);
      io_error = true;
      free_slots_.push_back(rd.slot);
      throw;
    }
    timed(ta);
    transfer(rd.key, rd.slot, rd.stage);
    --on_file_;
    commit(rd.key, rd.slot);
    ++n_read;
    void*& ev = stage_ev_[uint32_t(rd.stage) - c_.blocks];
    if (!ev) ev = event();
    m_->record(ev, Mover::kDem);
  };
  auto account = [&] {
    st_.resident_units += r.copied;
    st_.resident_evicted += r.evicted;
    st_.resident_bytes += uint64_t(r.copied) * unit_bytes_;
    st_.mkres_file_reads += n_read;
    st_.mkres_file_bytes += n_read * unit_bytes_;
    st_.mkres_read_ns += read_ns;
    st_.mkres_h2d_bytes += uint64_t(r.copied) * unit_bytes_;
    st_.mkres_wb_bytes += n_wb * unit_bytes_;
    st_.resident_ns += uint64_t(
        std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count());
  };
  try {
    size_t next = 0, vi = 0;
    while (next < in.size()) {
      // no free slot: the next victims (as many as the remaining units need and the blocks allow)
      const bool evict = free_slots_.empty();
      while (evict && vi < victims.size() && free_slots_.size() + wb.size() < in.size() - next) {
        const uint32_t v = victims[vi];
        Entry& x = e_[v];
        if (!x.backed && free_blocks_.empty() && !released.empty()) {  // the blocks of the copies already enqueued
          flush_dem();
          continue;
        }
        if (!x.backed && free_blocks_.empty() && !c_.disk_tier) break;
        // a clean copy (its block is its home again) or, file tier with no block to free (clean_evict: none
        // free), its file: no copy
        const bool clean = !x.backed && clean_now();
        const bool no_copy = x.backed || clean || (free_blocks_.empty() && !drop_host_lru(&hold, false));
        if (clean) count_clean();
        int32_t b = -1;
        if (!no_copy) {
          b = free_blocks_.back();
          m_->d2h(Mover::kD2h, x.slot, b, -1, v);  // the dirty unit's only copy, written back before its slot is reused
          free_blocks_.pop_back();
          ++n_wb;
        }
        ++vi;
        ++r.evicted;
        unlink(v);
        --on_device_;
        table_[v] = -1;
        if (no_copy) {
          free_slots_.push_back(x.slot);
          to_lower(v);
          continue;
        }
        wb.push_back(x.slot);
        x.home = Home::Host;
        x.slot = -1;
        x.block = b;
        hpush(v);
        hold[v] = 1;
      }
      flush_d2h();
      if (free_slots_.empty()) fail(SS_E_BACKEND, "ss_dg_make_resident: no slot for a unit");
      const int32_t slot = free_slots_.back();
      free_slots_.pop_back();
      const uint32_t k = in[next];
      Entry& x = e_[k];
      if (x.home == Home::Host) {
        const int32_t b = x.block;
        transfer(k, slot, b);
        ++next;
        hunlink(k);
        released.push_back(b);
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
        stage_next_ = (i + 1) % c_.disk_staging;
        const int32_t stage = int32_t(c_.blocks + i);
        for (size_t j = 0; j < reads.size(); ++j)
          if (reads[j].stage == stage) {
            end_read(j);
            break;
          }
        if (stage_ev_[i] && !m_->done(stage_ev_[i])) m_->event_sync(stage_ev_[i]);
        void* h = nullptr;
        const auto tb = std::chrono::steady_clock::now();
        try {
          h = m_->read_begin(k, stage);
        } catch (...) {
          timed(tb);
          io_error = true;
          throw;
        }
        timed(tb);
        reads.push_back({k, slot, stage, h});
        ++next;
      } catch (...) {
        free_slots_.push_back(slot);
        throw;
      }
    }
    while (!reads.empty()) end_read(0);
    flush_d2h();
    flush_dem();
    m_->upload_table(table_.data(), keys_);  // (syncs the demand stream) every changed entry, the victims' -1 included
  } catch (...) {
    for (const Read& rd : reads) {  // reads not ended give their slots back (their keys never changed home)
      try {
        m_->read_end(rd.handle);
      } catch (...) {
      }
      free_slots_.push_back(rd.slot);
    }
    reads.clear();
    bool ok = false;
    if (io_error) {  // the device is fine: what was enqueued lands, the table goes up
      try {
        flush_d2h();
        flush_dem();
        m_->upload_table(table_.data(), keys_);
        ok = true;
      } catch (...) {
      }
    }
    if (!ok) {  // a device failure: the host records stay one ownership (the context is poisoned by its caller)
      free_slots_.insert(free_slots_.end(), wb.begin(), wb.end());
      wb.clear();
      free_blocks_.insert(free_blocks_.end(), released.begin(), released.end());
      released.clear();
    }
    account();
    throw;
  }
  account();
  return r;
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
  const auto t0 = std::chrono::steady_clock::now();
  round_state_.store(kRoundRunning, std::memory_order_release);
  struct Idle {
    std::atomic<int>& s;
    ~Idle() { s.store(kRoundIdle, std::memory_order_release); }
  } idle{round_state_};
  last_round_ = RoundOut{};
  require(std::isfinite(in.decay) && in.decay >= 0 && in.decay <= 1, SS_E_INVALID, "ss_dg_round: decay must be 0..1");
  require(std::isfinite(in.hysteresis) && in.hysteresis >= 1 && in.hysteresis <= 1e6, SS_E_INVALID,
          "ss_dg_round: hysteresis must be 1..1e6");
  require(in.flags == 0, SS_E_INVALID, "ss_dg_round: unknown flags");
  std::vector<uint8_t> kept(keys_, 0);
  size_t n_kept = 0;
  for (uint32_t k : kept_keys)
    if (k < keys_ && !kept[k]) {
      kept[k] = 1;
      ++n_kept;
    }
  for (uint32_t k = 0; k < keys_; ++k)
    if (e_[k].home == Home::Bank) broken("a bank unit between tokens");
  stamp_room("ss_dg_round");
  drain();  // everything settled: copies, deferred and recorded write-backs collected
  for (const Writeback& w : wbs_) m_->event_sync(w.done);
  collect();
  if (!wbs_.empty()) broken("ss_dg_round: write-backs not collected");
  for (uint32_t k = 0; k < keys_; ++k) {
    rs_[k] = in.decay * rs_[k] + double(rhits_[k]);
    rhits_[k] = 0;
  }

  RoundOut r;
  const uint64_t ub = unit_bytes_;
  uint64_t spent = 0;
  uint32_t moved = 0;
  auto fits = [&](uint64_t b) { return !in.budget_bytes || (spent <= in.budget_bytes && b <= in.budget_bytes - spent); };
  auto cancelled = [&] {
    if (round_state_.load(std::memory_order_acquire) == kRoundCancel) r.cancelled = 1;
    return r.cancelled != 0;
  };
  std::vector<uint32_t> pos(keys_, 0), hpos(keys_, 0);  // recency positions, least recent first
  {
    uint32_t i = 0;
    for (uint32_t k = tail_; k != kNil; k = e_[k].prev) pos[k] = i++;
  }
  auto hotter = [&](uint32_t a, uint32_t b) { return rs_[a] != rs_[b] ? rs_[a] > rs_[b] : a < b; };
  auto colder_dev = [&](uint32_t a, uint32_t b) {
    if (rs_[a] != rs_[b]) return rs_[a] < rs_[b];
    return pos[a] != pos[b] ? pos[a] < pos[b] : a < b;
  };
  auto colder_host = [&](uint32_t a, uint32_t b) {
    if (rs_[a] != rs_[b]) return rs_[a] < rs_[b];
    return hpos[a] != hpos[b] ? hpos[a] < hpos[b] : a < b;
  };
  std::vector<uint32_t> dev, host, file;
  size_t n_coming = 0;
  for (uint32_t k = 0; k < keys_; ++k) {
    const Entry& x = e_[k];
    if (x.home == Home::Coming) ++n_coming;
    if (kept[k] || x.wb_pending) continue;
    if (x.home == Home::Device) dev.push_back(k);
    else if (x.home == Home::Host) host.push_back(k);
    else if (x.home == Home::File) file.push_back(k);
  }
  std::sort(dev.begin(), dev.end(), colder_dev);
  std::sort(host.begin(), host.end(), hotter);
  std::sort(file.begin(), file.end(), hotter);
  int64_t room = int64_t(c_.persistent_slots) - int64_t(c_.spare_target) - int64_t(n_kept) - int64_t(n_coming) -
                 int64_t(dev.size());
  const Mover::Stream ws = c_.wb_on_d2h ? Mover::kD2h : Mover::kDem;
  auto account = [&] {
    r.ns = uint64_t(
        std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count());
    ++st_.round_count;
    st_.round_units += uint64_t(r.promoted_to_device) + r.promoted_to_pinned + r.demoted_from_device + r.dropped_to_file;
    st_.round_bytes += r.bytes_read + r.bytes_h2d + r.bytes_written_back;
    st_.round_ns += r.ns;
    st_.round_cancelled += r.cancelled;
    last_round_ = r;
  };
  // a pinned unit into `slot`: its home changes once the copy and its entry were accepted and the demand stream synced;
  // a cancellation seen then drops it (the slot free again, the unit keeps its block)
  auto promote = [&](uint32_t k, int32_t slot) {
    Entry& x = e_[k];
    const int32_t b = x.block;
    try {
      m_->h2d(Mover::kDem, slot, b, k);
      publish(Mover::kDem, k, slot);
      m_->sync(Mover::kDem);
    } catch (...) {
      table_[k] = -1;
      free_slots_.push_back(slot);
      throw;
    }
    spent += ub;
    r.bytes_h2d += ub;
    if (cancelled()) {
      table_[k] = -1;
      free_slots_.push_back(slot);
      return false;
    }
    hunlink(k);
    free_blocks_.push_back(b);
    x.block = -1;
    x.slot = slot;
    x.home = Home::Device;
    push_front(k);
    ++on_device_;
    ++r.promoted_to_device;
    return true;
  };
  // a block for a demoted unit's write-back: a free one, else (file tier) the coldest pinned unit's, dropped to its
  // file (never `except`); -1 when none
  size_t hback = host.size();
  auto wb_block = [&](uint32_t except) -> int32_t {
    if (!free_blocks_.empty()) {
      const int32_t b = free_blocks_.back();
      free_blocks_.pop_back();
      return b;
    }
    if (!c_.disk_tier) return -1;
    while (hback > 0) {
      const uint32_t p = host[--hback];
      Entry& y = e_[p];
      if (p == except || y.home != Home::Host) continue;
      hunlink(p);
      const int32_t b = y.block;
      y.block = -1;
      y.home = Home::File;
      ++on_file_;
      ++r.dropped_to_file;
      return b;
    }
    return -1;
  };
  // (b)'s reads: one at a time (synchronous), each committed at the next read or at the end
  struct Rd {
    uint32_t key;
    int32_t block;
  };
  std::deque<Rd> reads;
  auto end_read = [&] {
    const Rd rd = reads.front();
    reads.pop_front();
    r.bytes_read += ub;
    if (cancelled()) {  // the block free again, the unit stays in its file
      free_blocks_.push_back(rd.block);
      return;
    }
    Entry& x = e_[rd.key];
    --on_file_;
    x.home = Home::Host;
    x.block = rd.block;
    hpush(rd.key);
    ++r.promoted_to_pinned;
  };
  try {
    size_t j = 0;
    for (size_t i = 0; i < host.size() && moved < in.max_units; ++i) {  // (a) pinned -> device
      const uint32_t c = host[i];
      if (!(rs_[c] > 0)) break;
      if (e_[c].home != Home::Host) continue;  // (dropped to its file for a write-back block)
      if (cancelled()) break;
      if (room > 0 && free_slots_.size() > c_.spare_target) {  // the device holds less than its share
        if (!fits(ub)) break;
        const int32_t slot = free_slots_.back();
        free_slots_.pop_back();
        if (!promote(c, slot)) break;
        --room;
        ++moved;
        continue;
      }
      if (j >= dev.size()) break;
      const uint32_t v = dev[j];
      if (!(rs_[c] > in.hysteresis * rs_[v])) break;
      Entry& y = e_[v];
      const bool clean = !y.backed && clean_now();  // clean_evict: no free block, to its file (no write)
      if (!fits(ub + (y.backed || clean ? 0 : ub))) break;
      const int32_t slot = y.slot;
      if (y.backed || clean) {  // a clean copy: its block is its home again, no write (clean_evict: its file)
        unlink(v);
        --on_device_;
        table_[v] = -1;
        to_lower(v);
        if (clean) count_clean();
      } else {
        const int32_t b = wb_block(c);
        if (b < 0) break;
        try {
          m_->d2h(ws, slot, b, -1, v);
          m_->sync(ws);
        } catch (...) {
          free_blocks_.push_back(b);  // the unit keeps its slot (its only copy)
          throw;
        }
        unlink(v);
        --on_device_;
        table_[v] = -1;
        y.home = Home::Host;
        y.slot = -1;
        y.block = b;
        hpush(v);
        spent += ub;
        r.bytes_written_back += ub;
      }
      ++j;
      ++r.demoted_from_device;
      if (!promote(c, slot)) break;  // (cancelled: the demoted unit's slot stays free)
      ++moved;
    }
    if (c_.disk_tier && !r.cancelled) {  // (b) file -> pinned, in place of the coldest pinned units
      std::vector<uint32_t> pinned;
      for (uint32_t k = 0; k < keys_; ++k)
        if (e_[k].home == Home::Host && !kept[k] && !e_[k].wb_pending) pinned.push_back(k);
      uint32_t hi = 0;
      for (uint32_t k = htail_; k != kNil; k = e_[k].hprev) hpos[k] = hi++;  // after (a)'s pushes
      std::sort(pinned.begin(), pinned.end(), colder_host);
      size_t pv = 0;
      for (size_t i = 0; i < file.size() && moved < in.max_units && pv < pinned.size(); ++i) {
        const uint32_t c = file[i];
        if (!(rs_[c] > 0)) break;
        if (e_[c].home != Home::File) continue;
        if (cancelled()) break;
        const uint32_t p = pinned[pv];
        if (!(rs_[c] > in.hysteresis * rs_[p])) break;
        if (!fits(ub)) break;
        if (!reads.empty()) end_read();
        if (r.cancelled) break;
        ++pv;
        Entry& y = e_[p];  // dropped to its file (no copy): its block is quiescent
        hunlink(p);
        const int32_t b = y.block;
        y.block = -1;
        y.home = Home::File;
        ++on_file_;
        ++r.dropped_to_file;
        try {
          m_->read_unit(c, b);
        } catch (...) {
          free_blocks_.push_back(b);
          throw;
        }
        reads.push_back({c, b});
        spent += ub;
        ++moved;
      }
      while (!reads.empty()) end_read();
    }
    m_->upload_table(table_.data(), keys_);  // (syncs the demand stream) every changed entry
  } catch (...) {
    for (const Rd& rd : reads) free_blocks_.push_back(rd.block);  // never committed: their units stay in their files
    reads.clear();
    try {  // the moves made so far go up (a failed device fails this too; the caller then poisons the context)
      m_->upload_table(table_.data(), keys_);
    } catch (...) {
    }
    account();
    throw;
  }
  account();
  return r;
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

uint32_t SlotCache::seed(const std::vector<uint32_t>& keys) {
  drain_pending();  // between tokens (copies, then an upload)
  stamp_room("ss_seed");
  if (!coming_.empty()) m_->sync(Mover::kPf);
  collect();
  uint32_t n = 0;
  for (uint32_t k : keys) {
    require(k < keys_, SS_E_INVALID, "ss_seed: unit out of range");
    Entry& x = e_[k];
    if (x.home != Home::Host || free_slots_.size() <= c_.spare_target) continue;
    const int32_t slot = free_slots_.back();
    free_slots_.pop_back();
    m_->h2d(Mover::kDem, slot, x.block, k);
    hunlink(k);
    free_blocks_.push_back(x.block);
    x.block = -1;
    x.slot = slot;
    x.home = Home::Device;
    table_[k] = slot;
    push_front(k);
    ++on_device_;
    ++n;
  }
  if (n) m_->upload_table(table_.data(), keys_);  // syncs kDem: the copies landed before their blocks are reused
  return n;
}

void SlotCache::drain() {
  drain_pending();
  while (!deferred_.empty()) finish_front();
  m_->sync(Mover::kDem);
  m_->sync(Mover::kPf);
  m_->sync(Mover::kD2h);
}

std::vector<uint32_t> SlotCache::residency() const {
  std::vector<uint32_t> out;
  out.reserve(on_device_);
  for (uint32_t k = head_; k != kNil; k = e_[k].next)
    if (e_[k].home == Home::Device) out.push_back(k);
  return out;
}

void SlotCache::set_wb_defer(bool on) {
  drain_pending();  // (settings: between tokens, every read ended first)
  if (on == c_.wb_defer) return;
  if (!on)
    while (!deferred_.empty()) finish_front();
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

// Locations: slots [0, P), blocks [P, P + blocks), the reset staging buffer and (file tier) the unit's file. Every
// misplaced unit moves once: units going back to their file first (no copy, their location vacated), then chains
// that end in a free location (each move fills the hole the previous one left; a unit read from its file ends its
// chain), then the remaining cycles through the staging buffer (dg_core.cpp:2976-3075). The mover executes each move
// before the next one reads its destination.
void SlotCache::reset_open() {
  require(open_e_.size() == keys_, SS_E_INVALID, "device-gated: reset before place");
  drain();
  for (const Writeback& w : wbs_) m_->event_sync(w.done);
  collect();
  if (!wbs_.empty()) broken("reset could not collect every write-back");
  for (Entry& x : e_)
    if (x.pf_done) {
      m_->event_sync(x.pf_done);
      pool_.push_back(x.pf_done);
      x.pf_done = nullptr;
    }
  for (void* ev : stage_ev_)  // every staging copy landed
    if (ev) m_->event_sync(ev);
  const size_t P = c_.persistent_slots, N = P + c_.blocks, stage = N, file = N + 1;
  std::vector<size_t> cur(keys_), dst(keys_);
  std::vector<uint32_t> occupant(N + 1, kNil), wanted(N + 1, kNil);
  for (uint32_t k = 0; k < keys_; ++k) {
    const Entry& x = e_[k];
    if (x.home == Home::Evicting) broken("reset left an evicting unit");
    // a unit read from its file has no block: a Coming one's slot is its only copy; a bank slot is no persistent
    // location, so a bank unit read from its file goes back to it
    const bool on_slot = x.home == Home::Device || (x.home == Home::Coming && x.block < 0);
    const bool in_file = x.home == Home::File || (x.home == Home::Bank && x.block < 0);
    cur[k] = in_file ? file : on_slot ? size_t(x.slot) : P + size_t(x.block);
    const Entry& o = open_e_[k];
    dst[k] = o.home == Home::File ? file : o.home == Home::Device ? size_t(o.slot) : P + size_t(o.block);
    if (cur[k] != file) occupant[cur[k]] = k;
    if (dst[k] != file) wanted[dst[k]] = k;
  }
  for (uint32_t k = 0; k < keys_; ++k)  // back to its file: its location is vacated, no copy
    if (dst[k] == file && cur[k] != file) {
      occupant[cur[k]] = kNil;
      cur[k] = file;
    }
  // plan every move first (bookkeeping only), then execute them in order; consecutive slot-to-slot moves share
  // launches: a move's wave is one after every earlier move that reads its destination or writes its source
  struct Move {
    size_t from, to;
    uint32_t key;
  };
  std::vector<Move> plan;
  auto move = [&](uint32_t k, size_t to) {
    const size_t from = cur[k];
    if (to > N || occupant[to] != kNil) broken("reset would overwrite a live source");
    plan.push_back({from, to, k});
    if (from != file) occupant[from] = kNil;
    occupant[to] = k;
    cur[k] = to;
  };
  for (size_t loc = 0; loc < N; ++loc) {
    size_t hole = loc;
    while (hole < N && occupant[hole] == kNil && wanted[hole] != kNil) {
      const uint32_t k = wanted[hole];
      const size_t next = cur[k];
      move(k, hole);
      hole = next;
    }
  }
  for (uint32_t k = 0; k < keys_; ++k) {
    if (cur[k] == dst[k]) continue;
    if (cur[k] == file) broken("reset left a file read behind");
    size_t hole = cur[k];
    move(k, stage);
    while (hole != dst[k]) {
      const uint32_t next = wanted[hole];
      if (next == kNil) broken("reset cycle without a predecessor");
      const size_t from = cur[next];
      move(next, hole);
      hole = from;
    }
    move(k, hole);
  }
  auto blk = [&](size_t loc) { return loc == stage ? -1 : int32_t(loc - P); };
  std::vector<std::pair<int32_t, int32_t>> d2d;
  std::vector<uint32_t> wave;
  auto flush_d2d = [&] {
    if (d2d.empty()) return;
    m_->d2d_moves(d2d, wave);
    d2d.clear();
    wave.clear();
  };
  for (const Move& mv : plan) {
    ++st_.reset_moves;
    st_.reset_bytes += unit_bytes_;
    if (mv.from < P && mv.to < P) {
      uint32_t w = 0;
      for (size_t i = 0; i < d2d.size(); ++i)
        if (size_t(d2d[i].first) == mv.to || size_t(d2d[i].second) == mv.from) w = std::max(w, wave[i] + 1);
      d2d.push_back({int32_t(mv.from), int32_t(mv.to)});
      wave.push_back(w);
      continue;
    }
    flush_d2d();
    if (mv.from == file && mv.to < P) {  // read into the reset staging buffer, then to the slot
      m_->read_unit(mv.key, -1);
      m_->h2d(Mover::kDem, int32_t(mv.to), -1, mv.key);
      m_->sync(Mover::kDem);
    } else if (mv.from == file) {
      m_->read_unit(mv.key, blk(mv.to));
    } else if (mv.from < P) {
      m_->d2h(Mover::kD2h, int32_t(mv.from), blk(mv.to), -1, mv.key);
      m_->sync(Mover::kD2h);
    } else if (mv.to < P) {
      m_->h2d(Mover::kDem, int32_t(mv.to), blk(mv.from), mv.key);
      m_->sync(Mover::kDem);
    } else {
      m_->h2h(blk(mv.from), blk(mv.to), mv.key);
    }
  }
  flush_d2d();
  c_ = open_c_;
  apply_wb_defer();
  std::copy(open_e_.begin(), open_e_.end(), e_.begin());
  reset_score();  // the history's open state (a profile's counts, or none)
  std::fill(rs_.begin(), rs_.end(), 0.0);  // placement rounds: the counts start over
  std::fill(rhits_.begin(), rhits_.end(), 0u);
  backed_ = 0;  // clean copies are dropped: the open holds none
  std::copy(open_table_.begin(), open_table_.end(), table_.begin());
  free_slots_ = open_free_slots_;
  free_blocks_ = open_free_blocks_;
  head_ = open_head_;
  tail_ = open_tail_;
  on_device_ = open_on_device_;
  hhead_ = open_hhead_;
  htail_ = open_htail_;
  on_file_ = open_on_file_;
  stage_next_ = 0;
  coming_.clear();
  banked_.clear();
  std::fill(bank_key_.begin(), bank_key_.end(), kNil);
  bank_seq_[0] = bank_seq_[1] = 0;
  bank_layer_[0] = bank_layer_[1] = kNil;
  bank_next_[0] = bank_next_[1] = 0;
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
  m_->upload_table(table_.data(), keys_);
}

void SlotCache::check() const {
  std::vector<uint8_t> slot_used(slots_, 0), block_used(c_.blocks, 0);
  auto take = [&](std::vector<uint8_t>& v, int64_t i, const char* what) {
    if (i < 0 || size_t(i) >= v.size() || v[size_t(i)]) broken(what);
    v[size_t(i)] = 1;
  };
  uint32_t listed = 0, dev = 0, hlisted = 0, hosts = 0, files = 0;
  for (uint32_t k = head_; k != kNil; k = e_[k].next) {
    if (++listed > keys_) broken("the recency list has a cycle");
    const Home h = e_[k].home;
    if (h != Home::Device && h != Home::Coming) broken("a listed unit is not on the device");
  }
  for (uint32_t k = hhead_; k != kNil; k = e_[k].hnext) {
    if (++hlisted > keys_) broken("the pinned recency list has a cycle");
    if (e_[k].home != Home::Host || !e_[k].in_hlist) broken("a unit in the pinned recency list is not a pinned home");
  }
  for (uint32_t k = 0; k < keys_; ++k) {
    const Entry& x = e_[k];
    switch (x.home) {
      case Home::Host:
        take(block_used, x.block, "a host unit without its own block");
        if (table_[k] != -1) broken("a host unit with a published entry");
        if (x.listed) broken("a host unit in the recency list");
        ++hosts;
        break;
      case Home::File:
        if (!c_.disk_tier) broken("a file home without the file tier");
        if (x.slot >= 0 || x.block >= 0 || x.listed || x.in_hlist) broken("a file home holding a slot or a block");
        if (table_[k] != -1) broken("a file home with a published entry");
        ++files;
        break;
      case Home::Device:
      case Home::Coming:
        ++dev;
        take(slot_used, x.slot, "a device unit without its own slot");
        if (x.slot >= int32_t(c_.persistent_slots)) broken("a device unit in a bank slot");
        if (table_[k] != x.slot) broken("a device unit's entry is not its slot");
        if (!x.listed) broken("a device unit outside the recency list");
        if (x.home == Home::Coming && (x.block >= 0 || !c_.disk_tier))
          take(block_used, x.block, "a coming unit without its source block");
        else if (x.home == Home::Coming) {  // (read from its file)
        } else if (x.backed) take(block_used, x.block, "a clean copy without its own block");
        else if (x.block >= 0) broken("a device unit still holding a block");
        if (x.backed && x.home != Home::Device) broken("a clean copy of a unit not on the device");
        break;
      case Home::Bank:
        take(slot_used, x.slot, "a bank unit without its own slot");
        if (x.block >= 0 || !c_.disk_tier) take(block_used, x.block, "a bank unit without its block");
        if (x.slot < int32_t(c_.persistent_slots)) broken("a bank unit in a persistent slot");
        if (table_[k] != x.slot) broken("a bank unit's entry is not its slot");
        break;
      case Home::Evicting:
        take(slot_used, x.slot, "an evicting unit without its slot");
        take(block_used, x.block, "an evicting unit without its destination block");
        if (table_[k] != -1) broken("an evicting unit with a published entry");
        break;
    }
  }
  if (dev != on_device_ || dev != listed) broken("the device count disagrees with the homes");
  if (files != on_file_) broken("the file count disagrees with the homes");
  if (c_.disk_tier && hosts != hlisted) broken("the pinned recency list does not hold every pinned home");
  for (int32_t s : free_slots_) take(slot_used, s, "a free slot that is also in use");
  for (int32_t b : free_blocks_) take(block_used, b, "a free block that is also in use");
  for (const Writeback& w : wbs_)
    if (w.discard) take(block_used, w.block, "a discarded write-back block in use");
  for (uint32_t s = 0; s < c_.persistent_slots; ++s)
    if (!slot_used[s]) broken("a persistent slot neither free nor held");
  for (uint32_t b = 0; b < c_.blocks; ++b)
    if (!block_used[b]) broken("a block neither free nor held");
}

}  // namespace tsb
