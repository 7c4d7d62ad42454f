// The slot cache driven as the device-gated context drives it, on a host mover with the device's concurrency (the
// test hook tsb_test_dg_async_replay; no context uses it). The deterministic replay (dg_host_mover.cpp) copies when a
// copy is enqueued and answers every event as complete, which is what the reference's own replay does and what table
// parity needs, but it cannot show an ordering mistake. Here:
// - three copy streams are worker threads that run their operations (copies, entry and ready writes, event records,
//   event waits, the table upload) in order, each after a random delay, as the CUDA streams of the context's mover do;
// - events complete when their stream reaches them; a wait holds its stream until the event completes;
// - reads in flight run on their own threads and land after a random delay;
// - an engine thread exports each layer's ids with the export kernel's rule on the device table as it is at that
//   moment, waits for the layer's ready word when the export saw a miss (the wait kernel), reads every routed unit
//   through the device table (the engine's kernels) and only then exports the next layer, while the service (this
//   thread) serves the layer, its prediction, its write-backs and its scoring.
// The engine's reads are checked against the units' bytes by the caller, and the mover counts every hazard it sees: a
// host write into a block that a copy still pending reads or writes, a host read of a block a pending copy writes, two
// moves of one wave on the same slot, an engine read of a slot a pending copy writes, a copy enqueued on a block whose
// file read has not ended. Every wait gives up after 20 s with an error instead of hanging. The cache's test mutations
// (an entry published before its bytes, a demand that does not wait for the prefetch bringing its unit) plant the
// ordering faults these checks exist to catch.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <climits>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <exception>
#include <memory>
#include <mutex>
#include <random>
#include <thread>
#include <vector>

#include "dg_core.hpp"
#include "errors.hpp"
#include "tierstream/tsb.h"

namespace tsb {
namespace {

using Clock = std::chrono::steady_clock;
constexpr auto kLimit = std::chrono::seconds(20);
enum Race { kHostWriteBusyBlock, kHostReadWrittenBlock, kWaveOverlap, kReadWrittenSlot, kCopyOnReadingBlock, kRaces };

struct Ev {
  uint64_t recorded = 0, completed = 0;
};

struct Op {
  enum Kind { Copy, Write, Record, Wait, Table } kind = Copy;
  uint8_t* dst = nullptr;
  const uint8_t* src = nullptr;
  uint64_t bytes = 0;
  int32_t ref_block = INT_MIN;    // a block the copy reads or writes (INT_MIN: none)
  bool writes_block = false;
  int32_t dst_slot = -1;          // the slot a copy writes
  int32_t* word = nullptr;
  int32_t val = 0;
  Ev* ev = nullptr;
  uint64_t n = 0;
  std::vector<int32_t> table;  // (Table: the entries from table_first on)
  uint32_t table_first = 0;
};

uint64_t checksum(const uint8_t* p, uint64_t n) {
  uint64_t s = 0;
  for (uint64_t i = 0; i < n; ++i) s += uint64_t(p[i]) * (i % 251 + 1);
  return s;
}

class AsyncMover final : public Mover {
 public:
  AsyncMover(const std::vector<uint64_t>& parts, uint32_t keys, uint32_t slots, uint32_t blocks, uint32_t gated,
             const uint8_t* files, uint32_t seed, uint32_t delay_us)
      : parts_(parts), files_(files), delay_(delay_us), rng_(seed), dtab_(keys, -1), ready_(gated, 0) {
    for (uint64_t b : parts_) unit_ += b;
    arena_.assign(size_t(slots) * unit_, 0);
    blocks_.assign(size_t(blocks + 1) * unit_, 0);  // the last one is the reset staging buffer (block -1)
    nblocks_ = blocks;
    block_refs_.assign(blocks + 1, 0);
    block_writes_.assign(blocks + 1, 0);
    reading_.assign(blocks + 1, 0);
    slot_writes_.assign(slots, 0);
    for (int s = 0; s < 3; ++s) th_[s] = std::thread([this, s] { loop(s); });
  }
  ~AsyncMover() override { halt(); }
  // The streams run what they hold (a wait no longer holds them) and stop, reads in flight land; before the cache
  // that owns the events goes away.
  void halt() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
      cv_.notify_all();
    }
    for (auto& t : th_)
      if (t.joinable()) t.join();
    for (Read* r : reads_) {  // (only on an error path: the cache ends every read it begins)
      if (r->th.joinable()) r->th.join();
      delete r;
    }
    reads_.clear();
  }

  uint8_t* slot_ptr(int32_t s) { return arena_.data() + size_t(s) * unit_; }
  uint8_t* block_ptr(int32_t b) { return blocks_.data() + size_t(bi(b)) * unit_; }
  uint64_t unit() const { return unit_; }
  uint64_t races(int i) const { return races_[i]; }

  uint32_t parts() const override { return uint32_t(parts_.size()); }
  uint64_t part_bytes(uint32_t p) const override { return parts_[p]; }
  void h2d(Stream s, int32_t slot, int32_t block, uint32_t) override {
    Op op;
    op.dst = slot_ptr(slot);
    op.src = block_ptr(block);
    op.bytes = unit_;
    op.ref_block = block;
    op.dst_slot = slot;
    enqueue(s, std::move(op));
  }
  void d2h(Stream s, int32_t slot, int32_t block, int32_t p, uint32_t) override {
    uint64_t off = 0;
    for (uint32_t i = 0; i < parts_.size(); ++i) {
      if (p < 0 || uint32_t(p) == i) {
        Op op;
        op.dst = block_ptr(block) + off;
        op.src = slot_ptr(slot) + off;
        op.bytes = parts_[i];
        op.ref_block = block;
        op.writes_block = true;
        enqueue(s, std::move(op));
      }
      off += parts_[i];
    }
  }
  void d2d_moves(const std::vector<std::pair<int32_t, int32_t>>& moves, const std::vector<uint32_t>& wave) override {
    uint32_t top = 0;
    for (uint32_t w : wave) top = std::max(top, w);
    for (uint32_t w = 0; w <= top; ++w) {
      std::vector<int32_t> touched;
      for (size_t i = 0; i < moves.size(); ++i) {
        if (wave[i] != w) continue;
        touched.push_back(moves[i].first);
        touched.push_back(moves[i].second);
        Op op;
        op.dst = slot_ptr(moves[i].second);
        op.src = slot_ptr(moves[i].first);
        op.bytes = unit_;
        op.dst_slot = moves[i].second;
        enqueue(kDem, std::move(op));
      }
      std::sort(touched.begin(), touched.end());
      if (std::adjacent_find(touched.begin(), touched.end()) != touched.end()) race(kWaveOverlap);
    }
    sync(kDem);
  }
  void h2h(int32_t src, int32_t dst, uint32_t) override {
    {
      std::lock_guard<std::mutex> lk(mu_);
      if (block_refs_[bi(dst)] || reading_[bi(dst)]) ++races_[kHostWriteBusyBlock];
      if (block_writes_[bi(src)] || reading_[bi(src)]) ++races_[kHostReadWrittenBlock];
    }
    std::memmove(block_ptr(dst), block_ptr(src), unit_);
  }
  void read_unit(uint32_t key, int32_t block) override {
    {
      std::lock_guard<std::mutex> lk(mu_);
      if (block_refs_[bi(block)] || reading_[bi(block)]) ++races_[kHostWriteBusyBlock];
    }
    std::memcpy(block_ptr(block), files_ + size_t(key) * unit_, unit_);
  }
  void* read_begin(uint32_t key, int32_t block) override {
    Read* r = new Read;
    r->block = block;
    uint32_t d = 0;
    {
      std::lock_guard<std::mutex> lk(mu_);
      if (block_refs_[bi(block)] || reading_[bi(block)]) ++races_[kHostWriteBusyBlock];
      reading_[bi(block)] = 1;
      reads_.push_back(r);
      d = delay_ ? uint32_t(rng_() % (delay_ + 1)) : 0;
    }
    uint8_t* dst = block_ptr(block);
    const uint8_t* src = files_ + size_t(key) * unit_;
    const uint64_t n = unit_;
    r->th = std::thread([r, dst, src, n, d] {
      if (d) std::this_thread::sleep_for(std::chrono::microseconds(d));
      std::memcpy(dst, src, n);
      r->done.store(true, std::memory_order_release);
    });
    return r;
  }
  uint64_t read_end(void* h) override {
    Read* r = static_cast<Read*>(h);
    r->th.join();
    std::lock_guard<std::mutex> lk(mu_);
    reading_[bi(r->block)] = 0;
    reads_.erase(std::find(reads_.begin(), reads_.end(), r));
    delete r;
    return 0;
  }
  bool read_done(void* h) override { return static_cast<Read*>(h)->done.load(std::memory_order_acquire); }
  void publish(Stream s, uint32_t key, int32_t v) override {
    Op op;
    op.kind = Op::Write;
    op.word = &dtab_[key];
    op.val = v;
    enqueue(s, std::move(op));
  }
  void ready(uint32_t g, uint32_t seq) override {
    Op op;
    op.kind = Op::Write;
    op.word = reinterpret_cast<int32_t*>(&ready_[g]);
    op.val = int32_t(seq);
    enqueue(kDem, std::move(op));
  }
  void* event_create() override { return new Ev; }
  void event_destroy(void* ev) override { delete static_cast<Ev*>(ev); }
  void record(void* ev, Stream s) override {
    Op op;
    op.kind = Op::Record;
    op.ev = static_cast<Ev*>(ev);
    std::lock_guard<std::mutex> lk(mu_);
    op.n = ++op.ev->recorded;
    push_locked(s, std::move(op));
  }
  void wait(Stream s, void* ev) override {
    Op op;
    op.kind = Op::Wait;
    op.ev = static_cast<Ev*>(ev);
    std::lock_guard<std::mutex> lk(mu_);
    op.n = op.ev->recorded;
    if (op.n) push_locked(s, std::move(op));
  }
  bool done(void* ev) override {
    std::lock_guard<std::mutex> lk(mu_);
    const Ev* e = static_cast<Ev*>(ev);
    return e->completed >= e->recorded;
  }
  void event_sync(void* ev) override {
    Ev* e = static_cast<Ev*>(ev);
    std::unique_lock<std::mutex> lk(mu_);
    const uint64_t n = e->recorded;
    if (!cv_.wait_until(lk, Clock::now() + kLimit, [&] { return e->completed >= n || failed_; }) || failed_)
      fail(SS_E_BACKEND, "async replay: an event never completed");
  }
  void sync(Stream s) override {
    std::unique_lock<std::mutex> lk(mu_);
    if (!cv_.wait_until(lk, Clock::now() + kLimit, [&] { return (q_[s].empty() && !busy_[s]) || failed_; }) ||
        failed_)
      fail(SS_E_BACKEND, "async replay: a stream never drained");
  }
  void upload_table(const int32_t* t, uint32_t n) override {
    Op op;
    op.kind = Op::Table;
    op.table.assign(t, t + n);
    enqueue(kDem, std::move(op));
    sync(kDem);
  }
  void upload_table_ranges(const int32_t* t, const uint32_t* ranges, uint32_t n) override {
    for (uint32_t i = 0; i < n; ++i) {
      Op op;
      op.kind = Op::Table;
      op.table_first = ranges[2 * i];
      op.table.assign(t + ranges[2 * i], t + ranges[2 * i] + ranges[2 * i + 1]);
      enqueue(kDem, std::move(op));
    }
    sync(kDem);
  }
  void sync_all() {
    for (int s = 0; s < 3; ++s) sync(Stream(s));
  }

  // The engine's side, under the mover's lock: the device table and ready words as the streams left them.
  std::mutex mu_;
  std::condition_variable cv_;
  bool failed_ = false;
  int32_t dtab(uint32_t key) const { return dtab_[key]; }
  uint32_t ready_word(uint32_t g) const { return ready_[g]; }
  bool slot_written(int32_t s) const { return slot_writes_[size_t(s)] != 0; }
  void race_locked(int i) { ++races_[i]; }

 private:
  struct Read {
    int32_t block = 0;
    std::thread th;
    std::atomic<bool> done{false};
  };
  size_t bi(int32_t b) const { return b < 0 ? nblocks_ : size_t(b); }
  void race(int i) {
    std::lock_guard<std::mutex> lk(mu_);
    ++races_[i];
  }
  void enqueue(Stream s, Op&& op) {
    std::lock_guard<std::mutex> lk(mu_);
    push_locked(s, std::move(op));
  }
  void push_locked(Stream s, Op&& op) {
    if (op.ref_block != INT_MIN) {
      if (reading_[bi(op.ref_block)]) ++races_[kCopyOnReadingBlock];
      ++block_refs_[bi(op.ref_block)];
      if (op.writes_block) ++block_writes_[bi(op.ref_block)];
    }
    if (op.dst_slot >= 0) ++slot_writes_[size_t(op.dst_slot)];
    q_[s].push_back(std::move(op));
    cv_.notify_all();
  }
  void loop(int s) {
    std::unique_lock<std::mutex> lk(mu_);
    for (;;) {
      cv_.wait(lk, [&] { return stop_ || !q_[s].empty(); });
      if (q_[s].empty()) return;  // (stop_)
      Op op = std::move(q_[s].front());
      q_[s].pop_front();
      busy_[s] = true;
      if (op.kind == Op::Wait &&
          !cv_.wait_until(lk, Clock::now() + kLimit, [&] { return op.ev->completed >= op.n || stop_; })) {
        failed_ = true;  // a wait that never ends: the replay fails instead of hanging
        cv_.notify_all();
      }
      // a copy takes up to the whole delay, a word write, record or wait a quarter of it (copies are the slow ones)
      const uint32_t top = op.kind == Op::Copy ? delay_ : delay_ / 4;
      const uint32_t d = top ? uint32_t(rng_() % (top + 1)) : 0;
      lk.unlock();
      if (d) std::this_thread::sleep_for(std::chrono::microseconds(d));
      if (op.kind == Op::Copy) std::memmove(op.dst, op.src, size_t(op.bytes));
      lk.lock();
      switch (op.kind) {
        case Op::Write: *op.word = op.val; break;
        case Op::Record: op.ev->completed = std::max(op.ev->completed, op.n); break;
        case Op::Table: std::copy(op.table.begin(), op.table.end(), dtab_.begin() + op.table_first); break;
        default: break;
      }
      if (op.ref_block != INT_MIN) {
        --block_refs_[bi(op.ref_block)];
        if (op.writes_block) --block_writes_[bi(op.ref_block)];
      }
      if (op.dst_slot >= 0) --slot_writes_[size_t(op.dst_slot)];
      busy_[s] = false;
      cv_.notify_all();
    }
  }

  std::vector<uint64_t> parts_;
  const uint8_t* files_;
  uint64_t unit_ = 0;
  uint32_t delay_;
  std::mt19937 rng_;
  size_t nblocks_ = 0;
  std::vector<uint8_t> arena_, blocks_;
  std::vector<int32_t> dtab_;
  std::vector<uint32_t> ready_;
  std::vector<uint32_t> block_refs_, block_writes_, slot_writes_;
  std::vector<uint8_t> reading_;
  std::vector<Read*> reads_;
  std::deque<Op> q_[3];
  bool busy_[3] = {false, false, false};
  bool stop_ = false;
  uint64_t races_[kRaces] = {};
  std::thread th_[3];
};

}  // namespace

void dg_async_replay(const tsb_dg_replay_config* c, const int32_t* ids, const int32_t* preds,
                     const uint8_t* src_units, uint32_t seed, uint32_t delay_us, int32_t mutation, uint64_t* read_sum,
                     uint64_t* races) {
  require(c && c->n_units && c->part_bytes && ids && src_units && read_sum, SS_E_INVALID,
          "tsb_test_dg_async_replay: null argument");
  require(c->n_ids >= 1 && c->n_ids <= 64 && c->n_pred <= 64, SS_E_INVALID, "tsb_test_dg_async_replay: 1..64 ids");
  require(c->policy <= 2, SS_E_INVALID, "tsb_test_dg_async_replay: policy 0..2");
  require(mutation >= 0 && mutation <= 2, SS_E_INVALID, "tsb_test_dg_async_replay: mutation 0..2");
  CacheConfig cfg;
  cfg.n_units.assign(c->n_units, c->n_units + c->n_gated);
  cfg.persistent_slots = c->persistent_slots;
  cfg.bank_slots = c->bank_slots;
  cfg.blocks = c->blocks;
  cfg.spare_target = c->spare_target;
  cfg.prefetch_reserve_auto = c->prefetch_reserve == 0xFFFFFFFFu;
  cfg.prefetch_reserve = cfg.prefetch_reserve_auto ? 0 : c->prefetch_reserve;
  cfg.prefetch_per_layer = c->prefetch_per_layer;
  cfg.prefetch_per_token = c->prefetch_per_token;
  cfg.wb_defer = c->wb_defer != 0;
  cfg.wb_on_d2h = c->wb_on_d2h != 0;
  cfg.wb_layer_bytes = c->wb_layer_bytes;
  cfg.wb_max_outstanding = c->wb_max_outstanding;
  cfg.inclusive = c->inclusive;
  cfg.disk_tier = c->disk_tier != 0;
  cfg.disk_prefetch = c->disk_prefetch != 0;
  cfg.home_blocks = c->home_blocks;
  cfg.disk_staging = c->disk_staging;
  cfg.disk_queue = c->disk_queue ? c->disk_queue : 1;
  cfg.scored = c->policy != 0;
  cfg.scored_auto = c->policy == 2;
  if (c->w_trans || c->w_freq || c->w_rec) {
    cfg.w_trans = c->w_trans;
    cfg.w_freq = c->w_freq;
    cfg.w_rec = c->w_rec;
  }
  cfg.max_ids = c->n_ids;
  cfg.no_admit = c->no_admit != 0;
  cfg.clean_evict = c->clean_evict != 0;
  cfg.pf_revert = c->pf_revert != 0;
  cfg.pf_strict = c->pf_strict != 0;
  cfg.bank_keep = c->bank_keep;
  cfg.landing_blocks = c->landing_blocks;
  cfg.landing_ttl = c->landing_ttl;
  const uint32_t G = c->n_gated;
  uint32_t keys = 0;
  for (uint32_t g = 0; g < G; ++g) keys += c->n_units[g];
  AsyncMover m(std::vector<uint64_t>(c->part_bytes, c->part_bytes + c->n_parts), keys,
               c->persistent_slots + 2 * c->bank_slots + 1, c->blocks + c->disk_staging + c->landing_blocks, G,
               src_units, seed, delay_us);
  auto core = std::make_unique<SlotCache>(cfg, &m);
  core->set_mutation(mutation);  // a planted ordering fault (the entry before its bytes, a demand not covered)
  std::vector<uint32_t> order(c->order, c->order + c->n_order);
  for (uint32_t k = 0; k < keys; ++k) order.push_back(k);
  std::vector<uint8_t> disk;
  if (cfg.disk_tier && c->disk) disk.assign(c->disk, c->disk + keys);
  core->place(order, disk.empty() ? nullptr : &disk);
  if (c->profile && cfg.scored) {
    std::vector<std::vector<uint32_t>> cells(G);
    const uint32_t* p = c->profile;
    for (uint32_t g = 0; g < G; ++g) {
      cells[g].assign(p, p + size_t(c->n_units[g]) * c->n_units[g]);
      p += size_t(c->n_units[g]) * c->n_units[g];
    }
    core->load_counts(cells);
  }
  for (uint32_t k = 0; k < keys; ++k) {  // the open's fill
    if (core->slot_of(k) < 0 && core->block_of(k) < 0) continue;
    uint8_t* dst = core->slot_of(k) >= 0 ? m.slot_ptr(core->slot_of(k)) : m.block_ptr(core->block_of(k));
    std::memcpy(dst, src_units + size_t(k) * m.unit(), m.unit());
  }
  m.upload_table(core->table().data(), keys);

  std::vector<std::vector<uint32_t>> held_keys(G);
  std::vector<uint8_t> held(G, 0);
  auto kept_all = [&] {
    std::vector<uint32_t> v;
    for (const auto& h : held_keys) v.insert(v.end(), h.begin(), h.end());
    return v;
  };
  // the engine's exports, seen by the service under the mover's lock
  std::vector<uint32_t> exported(G, 0);
  std::vector<uint64_t> masks(G, 0);
  bool engine_failed = false, service_failed = false;
  std::string engine_err;
  std::vector<uint32_t> row(c->n_ids), pred(c->n_pred);
  std::mt19937 erng(seed ^ 0x9e3779b9u);
  try {
    for (uint32_t t = 0; t < c->tokens; ++t) {
      const uint32_t seq = t + 1;
      std::vector<uint8_t> run(G, 1);
      for (uint32_t g = 0; g < G; ++g) run[g] = held[g] ? 0 : 1;
      core->begin_token(seq, &run);
      std::thread engine([&] {
        std::vector<uint8_t> buf;
        for (uint32_t g = 0; g < G; ++g) {
          if (!run[g]) continue;
          const int32_t* r = ids + (size_t(t) * G + g) * c->n_ids;
          const uint32_t d = delay_us ? uint32_t(erng() % (delay_us + 1)) : 0;  // the previous layer's compute
          if (d) std::this_thread::sleep_for(std::chrono::microseconds(d));
          std::unique_lock<std::mutex> lk(m.mu_);
          uint64_t mask = 0;
          for (uint32_t i = 0; i < c->n_ids; ++i)  // the export kernel's rule on the device table
            if (uint32_t(r[i]) < c->n_units[g] && m.dtab(core->key(g, uint32_t(r[i]))) < 0) mask |= 1ull << i;
          masks[g] = mask;
          exported[g] = seq;
          m.cv_.notify_all();
          if (mask && !m.cv_.wait_until(lk, Clock::now() + kLimit, [&] {
                return m.ready_word(g) == seq || m.failed_ || service_failed;
              })) {
            engine_failed = true;
            engine_err = "the engine's wait for a ready word timed out";
            m.cv_.notify_all();
            return;
          }
          if (m.failed_ || service_failed) return;
          for (uint32_t i = 0; i < c->n_ids; ++i) {  // the engine's reads through the device table
            const int32_t s = uint32_t(r[i]) < c->n_units[g] ? m.dtab(core->key(g, uint32_t(r[i]))) : -1;
            if (s >= 0 && m.slot_written(s)) m.race_locked(kReadWrittenSlot);
            read_sum[(size_t(t) * G + g) * c->n_ids + i] = s < 0 ? 0 : checksum(m.slot_ptr(s), m.unit());
          }
        }
      });
      try {
        for (uint32_t g = 0; g < G; ++g) {
          if (!run[g]) continue;
          uint32_t nx = g + 1;
          while (nx < G && !run[nx]) ++nx;
          uint64_t mask = 0;
          {
            std::unique_lock<std::mutex> lk(m.mu_);
            if (!m.cv_.wait_until(lk, Clock::now() + kLimit, [&] { return exported[g] == seq || engine_failed; }) ||
                engine_failed)
              fail(SS_E_BACKEND, "async replay: " + (engine_err.empty() ? std::string("no export") : engine_err));
            mask = masks[g];
          }
          const int32_t* r = ids + (size_t(t) * G + g) * c->n_ids;
          for (uint32_t i = 0; i < c->n_ids; ++i) row[i] = uint32_t(r[i]);
          core->serve_demand(g, row.data(), c->n_ids, mask);
          core->serve_use(g, row.data(), c->n_ids, mask);
          auto ahead = [&](uint32_t l) {
            std::lock_guard<std::mutex> lk(m.mu_);
            return exported[l] == seq;
          };
          if (preds && c->n_pred && g + 1 < G && run[g + 1]) {
            const int32_t* p = preds + (size_t(t) * G + g) * c->n_pred;
            for (uint32_t i = 0; i < c->n_pred; ++i) pred[i] = uint32_t(p[i]);
            core->serve_prediction(g + 1, pred.data(), c->n_pred, ahead(g + 1));
          }
          if (core->deferred() && nx < G) core->issue_writebacks(g, [&] { return ahead(nx); });
          if (core->scored()) core->score_layer(g);
        }
      } catch (...) {
        {
          std::lock_guard<std::mutex> lk(m.mu_);
          service_failed = true;
          m.cv_.notify_all();
        }
        engine.join();
        throw;
      }
      engine.join();
      if (engine_failed) fail(SS_E_BACKEND, "async replay: " + engine_err);
      core->end_token(kept_all(), c->rows ? c->rows : 1);
      core->check();
      if (c->reset_at && t + 1 == c->reset_at) {
        core->reset_open();
        for (auto& h : held_keys) h.clear();
        std::fill(held.begin(), held.end(), uint8_t(0));
      }
      if (c->round_every && (t + 1) % c->round_every == 0) {
        RoundIn in;
        in.budget_bytes = c->round_budget;
        in.max_units = c->round_max_units;
        in.hysteresis = double(c->round_hysteresis);
        in.decay = double(c->round_decay);
        core->round(in, kept_all());
      }
      for (uint32_t i = 0, at = 0; i < c->mr_n; at += c->mr_count[i], ++i) {
        if (c->mr_token[i] != t) continue;
        const uint32_t lg = c->mr_layer[i];
        std::vector<uint32_t> want(c->mr_ids + at, c->mr_ids + at + c->mr_count[i]), held_now;
        if (want.empty()) {
          held_keys[lg].clear();
          held[lg] = 0;
          continue;
        }
        core->make_resident(lg, want, kept_all());
        for (uint32_t u : want) held_now.push_back(core->key(lg, u));
        held_keys[lg] = held_now;
        held[lg] = 1;
      }
      core->set_range_uploads(std::any_of(held.begin(), held.end(), [](auto h) { return h != 0; }));
    }
    m.sync_all();
  } catch (...) {
    m.halt();
    core.reset();
    throw;
  }
  m.halt();
  core.reset();
  if (races)
    for (int i = 0; i < kRaces; ++i) races[i] = m.races(i);
}

}  // namespace tsb
