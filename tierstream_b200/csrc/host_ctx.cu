// Host forward mode on a B200: the context behind ss_open(forward_mode = SS_FORWARD_HOST).
//
// Per layer a pool of persistent device slots (planned residents + dynamic slots) with LRU admission
// (resident_set.cpp), and unit-sized ring slots shared by every layer of a stride for the transient units. Per forward:
// ss_layer_routes / ss_layer_all admit the routed units and start their copies (pinned tier -> slot on the copy
// stream; file -> staging -> slot on a reader thread), ss_acquire makes the engine stream wait for them and uploads the
// layer's uint64 address table, ss_release records where the layer's readers end (ring slots are reused after it),
// ss_end folds the counters. The admission, the slot choice and the ring cursor follow the reference's host-mode
// context (stream_ctx.cpp:1105-1156, 1303-1400, 1459-1527 there), so tables match it unit for unit.
//
// Copies from the pinned tier go through the copy engines for units of at least 8 MiB (they measured faster there on
// B200) and through the land kernel (kernels.cu, one launch for every unit of a routes call) below that.
//
// Exclusive tier mode (budget tier_mode EXCLUSIVE; stream_ctx.cpp:1030-1126, 1640-1665 there): a unit lives in a slot
// or in a pinned block, never both. An admission evicts at most as many victims as the layer's block class has free
// blocks (the rest of its misses stay transient and count as deferred), writes each victim back into a free block on
// the write-back stream before the admitted unit's copy into that slot starts, and a unit promoted from its block
// frees the block at ss_end. With exclusive_discard the evictions are uncapped and victims past the free blocks are
// discarded to their files.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <iterator>
#include <deque>
#include <memory>
#include <mutex>
#include <thread>

#include "ctx.hpp"
#include "errors.hpp"
#include "kernels.hpp"
#include "pinned.hpp"
#include "read_ahead.hpp"
#include "resident_set.hpp"
#include "source_file.hpp"
#include "xxh64.hpp"

namespace tsb {
namespace {

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    fail(e == cudaErrorMemoryAllocation ? SS_E_NOMEM : SS_E_BACKEND,
         std::string(what) + ": " + cudaGetErrorString(e));
  }
}
char* at(void* p, uint64_t off) { return static_cast<char*>(p) + off; }
uint64_t now_ns() {
  return uint64_t(
      std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now().time_since_epoch()).count());
}

struct Job {
  enum State { Queued = 0, Done = 1, Failed = 2, Cancelled = 3 };  // Cancelled: a queued read dropped unread
  int layer = 0, unit = 0;
  char* dst = nullptr;             // device slot
  const char* pinned = nullptr;    // pinned tier source, null = its file
  cudaEvent_t wait_ev = nullptr;   // the copy waits for it (the slot's last readers)
  cudaEvent_t src_wait_ev = nullptr;  // exclusive: the write-back into its block that has to land first
  cudaEvent_t dst_wb_ev = nullptr;    // exclusive: the write-back of the victim whose slot it lands in
  cudaEvent_t done_ev = nullptr;   // recorded on the copy stream after the copy
  bool spec = false;               // a speculative prefetch's read, behind every demand read
  ReadAhead::EntryPtr ra;          // host read-ahead: the unit's bytes come from this read's buffer
  std::atomic<int> state{Queued};
  ss_status err_status = SS_OK;
  std::string err;
};
using JobPtr = std::shared_ptr<Job>;

class HostCtx final : public HostContext {
 public:
  HostCtx(const Desc& d, const ss_budget& b, const Plan& p, const ss_options& o) : d_(d), b_(b), plan_(p), o_(o) {
    try {
      init();
    } catch (...) {
      close();
      throw;
    }
  }
  ~HostCtx() override { close(); }

  bool poisoned() const override { return poisoned_; }
  void poison() override { poisoned_ = true; }
  int device() const override { return o_.device; }
  int n_sources() const override { return int(files_.size()); }
  bool source_direct(int i) const override { return files_[size_t(i)]->direct(); }

  void seed(int layer, const int32_t* units, int n) override {
    check_layer(layer, "seed");
    require(!in_fwd_ && !fwd_open_, SS_E_INVALID, "seed: only between forwards");
    Lay& s = L_[size_t(layer)];
    require(s.rs != nullptr, SS_E_INVALID, "seed: layer has no units");
    require(n >= 0 && (units || n == 0), SS_E_INVALID, "seed: bad unit list");
    for (int i = 0; i < n; ++i)
      require(units[i] >= 0 && units[i] < d_.layers[size_t(layer)].n_units, SS_E_INVALID, "seed: unit out of range");
    std::vector<JobPtr> jobs;
    for (int i = 0; i < n; ++i) {
      const int u = units[i];
      if (s.rs->slot(u) >= 0 || plan_.tier[size_t(gidx(layer, u))] == SS_TIER_PAIR) continue;
      const int slot = s.rs->place(u, false);
      if (slot < 0) break;
      JobPtr j = make_job(layer, u, at(s.pool, uint64_t(slot) * stride(layer)));
      jobs.push_back(j);
      submit(j);
    }
    flush_copies();
    std::string err;
    ss_status st = SS_OK;
    for (const JobPtr& j : jobs) {
      wait_quiet(*j);
      if (j->state.load() != Job::Done) {
        s.rs->drop(j->unit);
        if (st == SS_OK) {
          st = j->err_status;
          err = j->err;
        }
      }
    }
    ck(cudaStreamSynchronize(copy_), "cudaStreamSynchronize (seed)");
    for (const JobPtr& j : jobs) pool_ev(j->done_ev);
    // exclusive: a seeded unit's copy out of its block has completed (stream sync): the block is free at once
    if (excl_)
      for (const JobPtr& j : jobs)
        if (j->state.load() == Job::Done) free_block(layer, j->unit);
    if (st != SS_OK) fail(st, err);
  }

  // The next forward's state, opened by ss_begin or by a prefetch between forwards (stream_ctx.cpp:1194-1213 there).
  void open_forward() {
    if (fwd_open_) return;
    for (size_t L = 0; L < L_.size(); ++L) {
      Lay& s = L_[L];
      std::fill(s.loc.begin(), s.loc.end(), int8_t(kNone));
      std::fill(s.slot.begin(), s.slot.end(), -1);
      std::fill(s.job.begin(), s.job.end(), nullptr);
      std::fill(s.count.begin(), s.count.end(), 0u);
      std::fill(s.spec_unclaimed.begin(), s.spec_unclaimed.end(), char(0));
      s.routed.clear();
      s.pending.clear();
      s.hits.clear();
      s.groups.clear();
      s.gview.clear();
      s.routes_given = s.acquired = s.released = s.skip = false;
    }
    std::fill(fwd_.begin(), fwd_.end(), ss_layer_stats{});
    fwd_open_ = true;
  }

  void begin(const uint32_t* rows, int n_layers) override {
    require(!in_fwd_, SS_E_INVALID, "begin: previous forward not ended");
    require(rows == nullptr || n_layers == int(L_.size()), SS_E_INVALID, "begin: rows_per_layer needs one per layer");
    open_forward();
    if (rows)
      for (size_t L = 0; L < L_.size(); ++L) L_[L].skip = rows[L] == 0;
    if (excl_) {
      xst_.free_blocks = free_block_count();
      xst_.min_free_blocks = std::min(xst_.min_free_blocks, xst_.free_blocks);
    }
    stream_set_ = false;
    in_fwd_ = true;
  }

  void routes(int layer, const int32_t* ids, int n) override {
    check_layer(layer, "routes");
    require(in_fwd_, SS_E_INVALID, "routes: outside a forward (call ss_begin)");
    require(n >= 0 && (ids || n == 0), SS_E_INVALID, "routes: bad ids");
    ingest(layer, ids, n);
  }

  void routes_dev(int layer, const int32_t* ids_dev, int n, void* stream) override {
    check_layer(layer, "routes_dev");
    require(in_fwd_, SS_E_INVALID, "routes_dev: outside a forward (call ss_begin)");
    require(n >= 0, SS_E_INVALID, "routes_dev: bad count");
    check_stream(stream, "routes_dev");
    std::vector<int32_t> ids(static_cast<size_t>(n), 0);
    if (n) {  // the routes are read back on the engine stream, right behind the router that wrote them
      ck(cudaMemcpyAsync(ids.data(), ids_dev, size_t(n) * 4, cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream)),
         "cudaMemcpyAsync (routes)");
      ck(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "cudaStreamSynchronize (routes)");
    }
    ingest(layer, ids.data(), n);
  }

  void routes_all(int layer) override {
    check_layer(layer, "layer_all");
    require(in_fwd_, SS_E_INVALID, "layer_all: outside a forward (call ss_begin)");
    const int n = d_.layers[size_t(layer)].n_units;
    std::vector<int32_t> ids(static_cast<size_t>(n), 0);
    for (int u = 0; u < n; ++u) ids[size_t(u)] = u;
    ingest(layer, ids.data(), n);
  }

  // stream_ctx.cpp:1401-1440 there: certain prefetches are admitted as demands (ring when no slot), speculative ones
  // take the stream ring only, at most lookahead_budget per call, and stop at a full ring; a later route claims them.
  // ss_host_prefetch / ss_host_prefetch_layer (n < 0: every unit): read these file-backed units into read-ahead
  // buffers ahead of their fetch (stream_ctx.cpp:1441-1449); a no-op without read-ahead buffers. Allowed between
  // forwards: the requests belong to the next forward.
  void host_prefetch(int layer, const int32_t* ids, int n) override {
    check_layer(layer, "host_prefetch");
    require(n < 0 || ids || n == 0, SS_E_INVALID, "host_prefetch: bad ids");
    if (!ra_) return;
    open_forward();
    require(L_[size_t(layer)].rs != nullptr, SS_E_INVALID, "host_prefetch: layer has no units");
    if (n < 0)
      for (int u = 0; u < d_.layers[size_t(layer)].n_units; ++u) ra_request(layer, u, false);
    else
      for (int i = 0; i < n; ++i) ra_request(layer, ids[i], false);
  }
  // A unit the read-ahead may read (stream_ctx.cpp:850-865): streamable, without a pinned copy, not resident, no fetch
  // of it this forward (or one waiting for a ring slot, pending_ok), at most a buffer's bytes; once per forward.
  void ra_request(int layer, int unit, bool pending_ok) {
    if (!ra_) return;
    const Lay& s = L_[size_t(layer)];
    const Layer& l = d_.layers[size_t(layer)];
    if (!s.rs || !l.streamable || unit < 0 || unit >= l.n_units) return;
    const int64_t g = gidx(layer, unit);
    if (plan_.tier[size_t(g)] == SS_TIER_PAIR || pinned_of_[size_t(g)] || s.rs->slot(unit) >= 0) return;
    if (host_stride(l.unit_bytes) > ra_bytes_ || s.job[size_t(unit)]) return;
    if (s.loc[size_t(unit)] != kNone && !(pending_ok && s.loc[size_t(unit)] == kRing)) return;
    ra_->request(layer, unit);
  }

  void prefetch(int layer, const int32_t* ids, int n, bool speculative) override {
    check_layer(layer, "prefetch");
    const Layer& l = d_.layers[size_t(layer)];
    std::vector<int32_t> all;
    if (n < 0) {  // the whole layer (ss_prefetch_layer)
      for (int u = 0; u < l.n_units; ++u) all.push_back(u);
      ids = all.data();
      n = int(all.size());
    }
    open_forward();  // allowed between forwards: the copies belong to the next forward
    Lay& s = L_[size_t(layer)];
    require(s.rs != nullptr, SS_E_INVALID, "prefetch: layer has no units");
    if (s.routes_given || s.acquired) return;  // too late to help
    ss_layer_stats& st = fwd_[size_t(layer)];
    uint32_t issued = 0;
    std::vector<char> busy(size_t(l.n_units), 0);
    for (int u = 0; u < l.n_units; ++u) busy[size_t(u)] = s.loc[size_t(u)] != kNone;
    for (int i = 0; i < n; ++i) {
      if (speculative && issued >= o_.lookahead_budget) break;
      const int32_t u = ids[i];
      if (u < 0 || u >= l.n_units) continue;
      if (s.loc[size_t(u)] != kNone || s.rs->slot(u) >= 0) continue;
      if (plan_.tier[size_t(gidx(layer, u))] == SS_TIER_PAIR) continue;
      // a speculative read never evicts a resident on a guess: the ring only
      const Admission a = speculative ? Admission{} : s.rs->admit({u}, busy, true, eviction_cap(layer));
      xst_.deferred += uint64_t(a.deferred);
      if (!a.admitted.empty()) {
        fetch_admitted(layer, a);
        st.evicted += a.evicted.size();
      } else if (!fetch_into_ring(layer, u, speculative)) {
        if (speculative) break;  // ring full: speculation never waits
        s.pending.push_back(u);
        s.loc[size_t(u)] = kRing;  // placed when a ring slot frees
        ra_request(layer, u, true);
      }
      busy[size_t(u)] = 1;
      if (speculative) {
        s.spec_unclaimed[size_t(u)] = 1;
        ++st.spec_issued;
      }
      ++issued;
    }
    flush_copies();
  }

  void acquire(int layer, void* stream, bool wait_all, ss_layer_view* out) override {
    check_layer(layer, "acquire");
    require(in_fwd_, SS_E_INVALID, "acquire: outside a forward");
    Lay& s = L_[size_t(layer)];
    const Layer& l = d_.layers[size_t(layer)];
    require(s.rs != nullptr, SS_E_INVALID, "acquire: layer has no units");
    require(!s.acquired, SS_E_INVALID, "acquire: layer acquired twice in one forward");
    check_stream(stream, "acquire");
    require(s.routes_given, SS_E_INVALID,
            "acquire: no routes for layer " + std::to_string(layer) + " (ss_layer_routes / ss_layer_all first)");
    dispatch_pending();
    require(s.pending.empty(), SS_E_CAPACITY,
            "acquire: the stream ring cannot hold layer " + std::to_string(layer) + "'s " +
                std::to_string(s.pending.size()) + " remaining transient units (release earlier layers or plan more "
                "ring slots)");
    cudaStream_t es = static_cast<cudaStream_t>(stream);
    if (s.ready_wait) {
      ck(cudaStreamWaitEvent(es, s.ready_ev, 0), "cudaStreamWaitEvent (ready)");
      s.ready_wait = false;
    }
    // groups: the hits (on the device already) first, then the units fetched for this layer, most routed rows first,
    // in chunks of group_units (one chunk when 0), each chunk in unit order
    std::vector<int32_t> fetched;
    std::copy_if(s.routed.begin(), s.routed.end(), std::back_inserter(fetched),
                 [&](int32_t u) { return bool(s.job[size_t(u)]); });
    std::stable_sort(fetched.begin(), fetched.end(),
                     [&](int32_t a, int32_t b) { return s.count[size_t(a)] > s.count[size_t(b)]; });
    s.groups.assign(1, s.hits);
    const size_t chunk = o_.group_units ? size_t(o_.group_units) : std::max<size_t>(fetched.size(), 1);
    for (auto from = fetched.begin(); from != fetched.end();) {
      const auto to = from + std::ptrdiff_t(std::min<size_t>(chunk, size_t(fetched.end() - from)));
      s.groups.emplace_back(from, to);
      std::sort(s.groups.back().begin(), s.groups.back().end());
      from = to;
    }
    if (wait_all) {
      const uint64_t t0 = now_ns();
      for (int32_t u : fetched) join(*s.job[size_t(u)], es);
      fwd_[size_t(layer)].wait_ns += now_ns() - t0;
    }
    s.version ^= 1;
    const int v = s.version;
    ck(cudaEventSynchronize(s.table_ev[v]), "cudaEventSynchronize (table)");
    uint64_t* t = s.table_host[v];
    for (int u = 0; u < l.n_units; ++u) {
      const void* a = nullptr;
      if (s.job[size_t(u)] ? s.count[size_t(u)] != 0 : s.rs->slot(u) >= 0) a = unit_addr(layer, u);
      t[u] = uint64_t(reinterpret_cast<uintptr_t>(a));
    }
    ck(cudaMemcpyAsync(s.table_dev[v], t, sizeof(uint64_t) * size_t(l.n_units), cudaMemcpyHostToDevice, es),
       "cudaMemcpyAsync (table)");
    s.gview.clear();
    for (const auto& g : s.groups) s.gview.push_back({g.data(), int(g.size())});
    s.acquired = true;
    out->table_dev = s.table_dev[v];
    out->table_host = t;
    out->n_units = l.n_units;
    out->groups = s.gview.data();
    out->n_groups = int(s.gview.size());
  }

  void group_wait(int layer, int group, void* stream) override {
    check_layer(layer, "group_wait");
    Lay& s = L_[size_t(layer)];
    require(s.acquired && !s.released, SS_E_INVALID, "group_wait: layer not acquired");
    require(group >= 0 && size_t(group) < s.groups.size(), SS_E_INVALID, "group_wait: no such group");
    check_stream(stream, "group_wait");
    if (group == 0) return;
    const uint64_t t0 = now_ns();
    for (int32_t u : s.groups[size_t(group)]) join(*s.job[size_t(u)], static_cast<cudaStream_t>(stream));
    fwd_[size_t(layer)].wait_ns += now_ns() - t0;
  }

  void release(int layer, void* stream) override {
    check_layer(layer, "release");
    Lay& s = L_[size_t(layer)];
    require(s.acquired && !s.released, SS_E_INVALID, "release: layer not acquired or already released");
    check_stream(stream, "release");
    cudaStream_t es = static_cast<cudaStream_t>(stream);
    ck(cudaEventRecord(s.release_ev, es), "cudaEventRecord (release)");
    ck(cudaEventRecord(s.table_ev[s.version], es), "cudaEventRecord (table)");
    s.released = true;
    for (int u = 0; u < d_.layers[size_t(layer)].n_units; ++u)
      if (s.spec_unclaimed[size_t(u)]) {
        s.spec_unclaimed[size_t(u)] = 0;
        ++fwd_[size_t(layer)].spec_dropped;
      }
    for (size_t i = 0; i < ring_.size(); ++i) {
      if (ring_[i].owner != layer) continue;
      if (ring_[i].job && !cancel(ring_[i].job)) wait_quiet(*ring_[i].job);  // a read not started is dropped
      ring_owner_ev_[i] = s.release_ev;
      ring_[i].owner = -1;
      ring_[i].job.reset();
    }
    dispatch_pending();
  }

  void end() override {
    require(in_fwd_, SS_E_INVALID, "end: no forward open");
    for (size_t L = 0; L < L_.size(); ++L)
      require(!L_[L].acquired || L_[L].released, SS_E_INVALID,
              "end: layer " + std::to_string(L) + " acquired but not released");
    flush_copies();
    ss_status failed = SS_OK;
    std::string err;
    for (const JobPtr& j : fwd_jobs_) {
      if (j->spec && cancel(j)) continue;  // a speculative read that has not started is dropped
      wait_quiet(*j);
      if (j->state.load() == Job::Failed && failed == SS_OK) {
        failed = j->err_status;
        err = j->err;
      }
    }
    if (ra_) {  // every fetch ended: the forward's read-ahead ends, each request counted once
      const RaStats f = ra_->end_forward();
      ra_st_.requested += f.requested;
      ra_st_.read += f.read;
      ra_st_.landed += f.landed;
      ra_st_.unused += f.unused;
      ra_st_.failed += f.failed;
      ra_st_.bytes += f.bytes;
      ra_st_.fallback = ra_->totals().fallback;
    }
    for (size_t L = 0; L < L_.size(); ++L) {
      Lay& s = L_[L];
      if (!s.rs) continue;
      bool any = false;
      for (int u = 0; u < d_.layers[L].n_units; ++u) {
        if (s.spec_unclaimed[size_t(u)]) ++fwd_[L].spec_dropped;  // a layer never released: its unused guesses
        if (s.loc[size_t(u)] != kPersistent || !s.job[size_t(u)]) continue;
        if (s.job[size_t(u)]->state.load() != Job::Done) s.rs->drop(u);  // a failed read is read again at next use
        else any = true;
      }
      for (size_t i = 0; i < ring_.size(); ++i)
        if (ring_[i].owner == int(L)) {
          ring_[i].owner = -1;
          ring_[i].job.reset();
        }
      if (any) {  // persistent copies issued this forward: the layer's next acquire waits for them
        std::lock_guard<std::mutex> lk(copy_mu_);
        ck(cudaEventRecord(s.ready_ev, copy_), "cudaEventRecord (layer ready)");
        s.ready_wait = true;
      }
    }
    // exclusive: promotions free their blocks; the copy stream waits for this forward's write-backs (every block
    // they wrote is complete before a later forward reads it), then marks blocks_ev_ after every copy of this forward
    // (the next forward's first write-back waits for it before reusing a freed block or reading a slot filled now)
    if (excl_) {
      for (size_t L = 0; L < L_.size(); ++L) {
        Lay& s = L_[L];
        if (!s.rs) continue;
        for (int u = 0; u < d_.layers[L].n_units; ++u)
          if (s.loc[size_t(u)] == kPersistent && s.job[size_t(u)] && s.job[size_t(u)]->pinned &&
              s.job[size_t(u)]->state.load() == Job::Done)
            free_block(int(L), u);
      }
      {
        std::lock_guard<std::mutex> lk(copy_mu_);
        if (!wb_evs_.empty()) {
          ck(cudaEventRecord(wb_mark_ev_, wb_stream_), "cudaEventRecord (write-back mark)");
          ck(cudaStreamWaitEvent(copy_, wb_mark_ev_, 0), "cudaStreamWaitEvent (write-back mark)");
        }
        ck(cudaEventRecord(blocks_ev_, copy_), "cudaEventRecord (blocks)");
        wb_gate_ = true;
      }
      for (int64_t g : wb_units_) wb_pending_[size_t(g)] = nullptr;
      wb_units_.clear();
      for (cudaEvent_t e : wb_evs_) pool_ev(e);
      wb_evs_.clear();
      xst_.free_blocks = free_block_count();
    }
    for (const JobPtr& j : fwd_jobs_) pool_ev(j->done_ev);
    fwd_jobs_.clear();
    ss_layer_stats tot{};
    for (size_t L = 0; L < L_.size(); ++L) {
      add(stats_[L], fwd_[L]);
      add(tot, fwd_[L]);
    }
    if (hook_) hook_(hook_user_, &tot, fwd_.data(), int(L_.size()));
    in_fwd_ = false;
    fwd_open_ = false;
    ++forwards_;
    if (failed != SS_OK) fail(failed, err);
  }

  void check_unit(int layer, int unit) override {
    check_layer(layer, "check_unit");
    Lay& s = L_[size_t(layer)];
    const Layer& l = d_.layers[size_t(layer)];
    require(s.acquired && !s.released, SS_E_INVALID, "check_unit: layer not acquired");
    require(unit >= 0 && unit < l.n_units, SS_E_INVALID, "check_unit: unit out of range");
    const void* a = reinterpret_cast<const void*>(uintptr_t(s.table_host[s.version][unit]));
    require(a != nullptr, SS_E_INVALID, "check_unit: unit not available in this forward");
    if (s.job[size_t(unit)]) {
      wait_quiet(*s.job[size_t(unit)]);
      require(s.job[size_t(unit)]->state.load() == Job::Done, s.job[size_t(unit)]->err_status,
              s.job[size_t(unit)]->err);
    }
    ck(cudaStreamSynchronize(copy_), "cudaStreamSynchronize (check)");
    std::vector<char> got(size_t(l.unit_bytes)), want(size_t(l.unit_bytes));
    ck(cudaMemcpy(got.data(), a, got.size(), cudaMemcpyDeviceToHost), "cudaMemcpy (check)");
    read_unit(layer, unit, want.data());
    require(std::memcmp(got.data(), want.data(), got.size()) == 0, SS_E_HASH,
            "check_unit: the bytes of (" + std::to_string(layer) + ", " + std::to_string(unit) +
                ") differ from the source");
    if (!l.hash.empty())
      require(xxh64(got.data(), got.size()) == l.hash[size_t(unit)], SS_E_HASH,
              "check_unit: (" + std::to_string(layer) + ", " + std::to_string(unit) + ") differs from its hash");
  }

  void layer_stats(int layer, ss_layer_stats* out) const override {
    require(layer >= 0 && size_t(layer) < L_.size(), SS_E_INVALID, "ss_stats_layer: layer out of range");
    *out = stats_[size_t(layer)];
  }
  void total_stats(ss_layer_stats* out) const override {
    *out = ss_layer_stats{};
    for (const auto& s : stats_) add(*out, s);
  }
  void reset_stats() override { std::fill(stats_.begin(), stats_.end(), ss_layer_stats{}); }
  void set_hook(ss_stats_hook hook, void* user) override {
    hook_ = hook;
    hook_user_ = user;
  }
  void exclusive_stats(ss_exclusive_stats* out) const override {
    *out = xst_;
    out->struct_size = uint32_t(sizeof *out);
  }
  std::string stats_json() const override {
    ss_layer_stats t;
    total_stats(&t);
    char buf[1024];
    std::snprintf(buf, sizeof buf,
                  "{\"schema\":\"strix-stream/stats-v1\",\"mode\":\"host\",\"forwards\":%llu,\"total\":{\"routed\":%llu,"
                  "\"hits\":%llu,\"admitted\":%llu,\"transient\":%llu,\"evicted\":%llu,\"bytes_pinned\":%llu,"
                  "\"bytes_disk\":%llu,\"wait_ns\":%llu},\"land_launches\":%llu,\"exclusive\":{\"on\":%d,"
                  "\"writebacks\":%llu,\"writeback_bytes\":%llu,\"deferred\":%llu,\"promoted\":%llu,"
                  "\"free_blocks\":%llu,\"min_free_blocks\":%llu,\"rereads\":%llu,\"discards\":%llu}}",
                  (unsigned long long)forwards_, (unsigned long long)t.routed, (unsigned long long)t.hits,
                  (unsigned long long)t.admitted, (unsigned long long)t.transient, (unsigned long long)t.evicted,
                  (unsigned long long)t.bytes_pinned, (unsigned long long)t.bytes_disk, (unsigned long long)t.wait_ns,
                  (unsigned long long)land_launches_, excl_ ? 1 : 0, (unsigned long long)xst_.writebacks,
                  (unsigned long long)xst_.writeback_bytes, (unsigned long long)xst_.deferred,
                  (unsigned long long)xst_.promoted, (unsigned long long)xst_.free_blocks,
                  (unsigned long long)xst_.min_free_blocks, (unsigned long long)xst_.rereads,
                  (unsigned long long)xst_.discards);
    std::string js = buf;
    if (ra_) {  // (readahead_units = 0: the JSON stays as it was, as the reference's does)
      char r[512];
      std::snprintf(r, sizeof r,
                    ",\"readahead\":{\"buffers\":%llu,\"buffer_bytes\":%llu,\"requested\":%llu,\"read\":%llu,"
                    "\"landed\":%llu,\"unused\":%llu,\"failed\":%llu,\"fallback\":%llu,\"bytes\":%llu}}",
                    (unsigned long long)ra_bufs_.size(), (unsigned long long)ra_bytes_,
                    (unsigned long long)ra_st_.requested, (unsigned long long)ra_st_.read,
                    (unsigned long long)ra_st_.landed, (unsigned long long)ra_st_.unused,
                    (unsigned long long)ra_st_.failed, (unsigned long long)ra_->totals().fallback,
                    (unsigned long long)ra_st_.bytes);
      js.pop_back();  // the closing brace
      js += r;
    }
    return js;
  }

  void test_locs(int layer, int32_t* out, int n) const override {
    check_layer(layer, "tsb_test_host_locs");
    const Lay& s = L_[size_t(layer)];
    require(s.acquired && !s.released, SS_E_INVALID, "tsb_test_host_locs: layer not acquired");
    require(n == d_.layers[size_t(layer)].n_units, SS_E_INVALID, "tsb_test_host_locs: n must be the layer's units");
    for (int u = 0; u < n; ++u) {
      out[2 * u] = 0;
      out[2 * u + 1] = -1;
      if (!s.table_host[s.version][u]) continue;
      const bool ring = s.loc[size_t(u)] == kRing;
      out[2 * u] = ring ? 2 : 1;
      out[2 * u + 1] = ring ? s.slot[size_t(u)] : s.rs->slot(u);
    }
  }

  void test_unit(int layer, int unit, void** pinned, void** device) const override {
    check_layer(layer, "tsb_test_host_unit");
    require(!in_fwd_, SS_E_INVALID, "tsb_test_host_unit: between forwards only");
    const Lay& s = L_[size_t(layer)];
    require(s.rs != nullptr && unit >= 0 && unit < d_.layers[size_t(layer)].n_units, SS_E_INVALID,
            "tsb_test_host_unit: unit out of range");
    *pinned = const_cast<char*>(pinned_of_[size_t(gidx(layer, unit))]);
    const int slot = s.rs->slot(unit);
    *device = slot < 0 ? nullptr : at(s.pool, uint64_t(slot) * stride(layer));
  }

 private:
  enum Loc : int8_t { kNone = 0, kPersistent = 1, kRing = 2 };
  struct Ring {
    char* dev = nullptr;
    uint64_t stride = 0;
    int owner = -1;
    JobPtr job;
  };
  struct RingClass {
    uint64_t stride;
    size_t first, count, cursor;
  };
  struct Lay {
    std::unique_ptr<ResidentSet> rs;
    char* pool = nullptr;
    cudaEvent_t release_ev = nullptr, ready_ev = nullptr;
    bool ready_wait = false;
    uint64_t* table_dev[2] = {nullptr, nullptr};
    uint64_t* table_host[2] = {nullptr, nullptr};
    cudaEvent_t table_ev[2] = {nullptr, nullptr};
    std::vector<int8_t> loc;
    std::vector<int32_t> slot;
    std::vector<JobPtr> job;
    std::vector<uint32_t> count;
    std::vector<char> spec_unclaimed;  // speculative prefetches no route claimed yet
    std::vector<int32_t> routed, pending, hits;
    std::vector<std::vector<int32_t>> groups;
    std::vector<ss_group> gview;
    bool routes_given = false, acquired = false, released = false, skip = false;
    int version = 0;
  };

  // a += b, counter by counter (the struct is twelve uint64_t counters and nothing else)
  static void add(ss_layer_stats& a, const ss_layer_stats& b) {
    constexpr size_t kCounters = sizeof(ss_layer_stats) / sizeof(uint64_t);
    static_assert(kCounters == 12 && sizeof(ss_layer_stats) == kCounters * sizeof(uint64_t), "counters only");
    uint64_t sum[kCounters], more[kCounters];
    std::memcpy(sum, &a, sizeof sum);
    std::memcpy(more, &b, sizeof more);
    for (size_t i = 0; i < kCounters; ++i) sum[i] += more[i];
    std::memcpy(&a, sum, sizeof sum);
  }
  int64_t gidx(int layer, int unit) const { return d_.unit_base[size_t(layer)] + unit; }
  uint64_t stride(int layer) const { return d_.unit_stride(layer); }
  void check_layer(int layer, const char* what) const {
    require(layer >= 0 && size_t(layer) < L_.size(), SS_E_INVALID, std::string(what) + ": layer out of range");
  }
  void check_stream(void* stream, const char* what) {
    if (!stream_set_) {
      stream_ = stream;
      stream_set_ = true;
      return;
    }
    require(stream == stream_, SS_E_INVALID,
            std::string(what) + ": a forward must use one engine stream (join other streams into it first)");
  }
  const void* unit_addr(int layer, int unit) const {
    const Lay& s = L_[size_t(layer)];
    if (s.loc[size_t(unit)] == kRing) return ring_[size_t(s.slot[size_t(unit)])].dev;
    const int slot = s.rs->slot(unit);
    return slot < 0 ? nullptr : at(s.pool, uint64_t(slot) * stride(layer));
  }
  cudaEvent_t event() {
    if (!ev_pool_.empty()) {
      cudaEvent_t e = ev_pool_.back();
      ev_pool_.pop_back();
      return e;
    }
    cudaEvent_t e = nullptr;
    ck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
    all_ev_.push_back(e);
    return e;
  }
  void pool_ev(cudaEvent_t e) {
    if (e) ev_pool_.push_back(e);
  }
  JobPtr make_job(int layer, int unit, char* dst, bool spec = false) {
    JobPtr j = std::make_shared<Job>();
    j->layer = layer;
    j->unit = unit;
    j->dst = dst;
    j->spec = spec;
    j->wait_ev = L_[size_t(layer)].release_ev;
    j->pinned = pinned_of_[size_t(gidx(layer, unit))];
    if (excl_ && j->pinned) {
      j->src_wait_ev = wb_pending_[size_t(gidx(layer, unit))];
      if (j->src_wait_ev) ++xst_.rereads;
    }
    j->done_ev = event();
    return j;
  }

  // A pinned-tier job joins the routes call's batch (issued by flush_copies); a file job goes to the readers.
  void submit(const JobPtr& j) {
    if (j->pinned) {
      batch_.push_back(j);
      return;
    }
    if (ra_ && !j->spec) j->ra = ra_->claim(j->layer, j->unit);  // a speculative read takes the ordinary path
    {
      std::lock_guard<std::mutex> lk(q_mu_);
      (j->spec ? spec_queue_ : queue_).push_back(j);
    }
    q_cv_.notify_one();
  }
  // A speculative read that is now a demand goes to the front of the demand queue if it has not started.
  void promote(const JobPtr& j) {
    std::lock_guard<std::mutex> lk(q_mu_);
    if (!j->spec) return;
    auto it = std::find(spec_queue_.begin(), spec_queue_.end(), j);
    j->spec = false;
    if (it == spec_queue_.end()) return;  // started (or a pinned copy, issued at once)
    spec_queue_.erase(it);
    queue_.push_front(j);
  }
  // A queued (not started) read is dropped: true; false when it started, so the caller waits for it.
  bool cancel(const JobPtr& j) {
    {
      std::lock_guard<std::mutex> lk(q_mu_);
      for (auto* q : {&queue_, &spec_queue_}) {
        auto it = std::find(q->begin(), q->end(), j);
        if (it == q->end()) continue;
        q->erase(it);
        j->state.store(Job::Cancelled);
        done_cv_.notify_all();
        return true;
      }
    }
    return j->state.load() == Job::Cancelled;
  }
  void flush_copies() {
    if (batch_.empty()) return;
    std::lock_guard<std::mutex> lk(copy_mu_);
    for (const JobPtr& j : batch_) {
      if (j->wait_ev) ck(cudaStreamWaitEvent(copy_, j->wait_ev, 0), "cudaStreamWaitEvent (slot reuse)");
      if (j->src_wait_ev) ck(cudaStreamWaitEvent(copy_, j->src_wait_ev, 0), "cudaStreamWaitEvent (block written)");
      if (j->dst_wb_ev) ck(cudaStreamWaitEvent(copy_, j->dst_wb_ev, 0), "cudaStreamWaitEvent (victim written back)");
    }
    // the land kernel for small units (one launch for the batch), the copy engines for large ones
    auto kb = std::make_unique<dev::Batch>();
    auto launch = [&] {
      if (!kb->n_copies) return;
      uint64_t chunks = 0;
      for (uint32_t i = 0; i < kb->n_copies; ++i) chunks += (kb->copies[i].bytes + (64u << 10) - 1) >> 16;
      ck(cudaError_t(dev::launch_batch(*kb, int(std::min<uint64_t>(std::max<uint64_t>(chunks, 1), 296)), copy_)),
         "land kernel");
      ++land_launches_;
      kb->n_copies = 0;
    };
    for (const JobPtr& j : batch_) {
      const uint64_t n = d_.layers[size_t(j->layer)].unit_bytes;
      if (n >= ce_min_) {
        for (uint64_t off = 0; off < n; off += o_.copy_piece_bytes)
          ck(cudaMemcpyAsync(j->dst + off, j->pinned + off, size_t(std::min<uint64_t>(o_.copy_piece_bytes, n - off)),
                             cudaMemcpyHostToDevice, copy_),
             "cudaMemcpyAsync (fetch)");
      } else {
        if (kb->n_copies == dev::kMaxCopies) launch();
        kb->copies[kb->n_copies++] = {j->pinned, j->dst, n};
      }
    }
    launch();
    for (const JobPtr& j : batch_) {
      ck(cudaEventRecord(j->done_ev, copy_), "cudaEventRecord (fetch)");
      j->state.store(Job::Done);
    }
    batch_.clear();
    done_cv_.notify_all();
  }

  void read_unit(int layer, int unit, char* dst) const {
    const Layer& l = d_.layers[size_t(layer)];
    uint64_t off = 0;
    for (const Part& p : l.parts) {
      files_[size_t(p.source)]->read(dst + off, p.offset + uint64_t(unit) * p.stride, p.bytes);
      off += p.bytes;
    }
  }
  // Reader thread: the unit's file bytes into a staging buffer (hash-checked with verify_hash), then to its slot.
  void worker() {
    if (cudaSetDevice(o_.device) != cudaSuccess) (void)cudaGetLastError();  // its copies run on the context's device
    for (;;) {
      JobPtr j;
      {
        std::unique_lock<std::mutex> lk(q_mu_);
        q_cv_.wait(lk, [&] { return stop_ || !queue_.empty() || !spec_queue_.empty(); });
        if (stop_ && queue_.empty() && spec_queue_.empty()) return;
        std::deque<JobPtr>& q = queue_.empty() ? spec_queue_ : queue_;  // speculative reads only when no demand waits
        j = q.front();
        q.pop_front();
      }
      if (j->ra) {  // its bytes are in a read-ahead buffer (or will be once that read ends)
        land_read_ahead(*j);
        continue;
      }
      size_t buf = 0;
      {
        std::unique_lock<std::mutex> lk(st_mu_);
        st_cv_.wait(lk, [&] { return !st_free_.empty(); });
        buf = st_free_.back();
        st_free_.pop_back();
      }
      const Layer& l = d_.layers[size_t(j->layer)];
      try {
        char* s = staging_[buf];
        read_unit(j->layer, j->unit, s);
        if (o_.verify_hash && !l.hash.empty())
          require(xxh64(s, size_t(l.unit_bytes)) == l.hash[size_t(j->unit)], SS_E_HASH,
                  "read: unit (" + std::to_string(j->layer) + ", " + std::to_string(j->unit) +
                      ") differs from its descriptor hash");
        {
          std::lock_guard<std::mutex> lk(copy_mu_);
          if (j->wait_ev) ck(cudaStreamWaitEvent(copy_, j->wait_ev, 0), "cudaStreamWaitEvent (slot reuse)");
          if (j->dst_wb_ev)
            ck(cudaStreamWaitEvent(copy_, j->dst_wb_ev, 0), "cudaStreamWaitEvent (victim written back)");
          ck(cudaMemcpyAsync(j->dst, s, size_t(l.unit_bytes), cudaMemcpyHostToDevice, copy_), "cudaMemcpyAsync (read)");
          ck(cudaEventRecord(j->done_ev, copy_), "cudaEventRecord (read)");
        }
        ck(cudaEventSynchronize(j->done_ev), "cudaEventSynchronize (staging reuse)");
        j->state.store(Job::Done);
      } catch (const Error& e) {
        j->err_status = e.status();
        j->err = e.what();
        j->state.store(Job::Failed);
      } catch (const std::exception& e) {
        j->err_status = SS_E_BACKEND;
        j->err = e.what();
        j->state.store(Job::Failed);
      }
      {
        std::lock_guard<std::mutex> lk(st_mu_);
        st_free_.push_back(buf);
      }
      st_cv_.notify_one();
      {
        std::lock_guard<std::mutex> lk(q_mu_);
      }
      done_cv_.notify_all();
    }
  }
  // A fetch whose unit the read-ahead reads: its copy comes out of that buffer once the read ended; the buffer comes
  // back after the copy (a copy that failed after it started keeps it out of use); a failed read fails the fetch.
  void land_read_ahead(Job& j) {
    const Layer& l = d_.layers[size_t(j.layer)];
    bool issued = false;
    try {
      ss_status st = SS_OK;
      std::string msg;
      const char* src = ra_->wait(*j.ra, &st, &msg);
      if (!src) fail(st, msg);
      {
        std::lock_guard<std::mutex> lk(copy_mu_);
        if (j.wait_ev) ck(cudaStreamWaitEvent(copy_, j.wait_ev, 0), "cudaStreamWaitEvent (slot reuse)");
        if (j.dst_wb_ev) ck(cudaStreamWaitEvent(copy_, j.dst_wb_ev, 0), "cudaStreamWaitEvent (victim written back)");
        issued = true;
        ck(cudaMemcpyAsync(j.dst, src, size_t(l.unit_bytes), cudaMemcpyHostToDevice, copy_),
           "cudaMemcpyAsync (read-ahead)");
        ck(cudaEventRecord(j.done_ev, copy_), "cudaEventRecord (read-ahead)");
      }
      ck(cudaEventSynchronize(j.done_ev), "cudaEventSynchronize (read-ahead buffer reuse)");
      ra_->done(*j.ra, true, true);
      j.state.store(Job::Done);
    } catch (const Error& e) {
      ra_->done(*j.ra, false, issued);
      j.err_status = e.status();
      j.err = e.what();
      j.state.store(Job::Failed);
    } catch (const std::exception& e) {
      ra_->done(*j.ra, false, issued);
      j.err_status = SS_E_BACKEND;
      j.err = e.what();
      j.state.store(Job::Failed);
    }
    {
      std::lock_guard<std::mutex> lk(q_mu_);
    }
    done_cv_.notify_all();
  }
  void wait_quiet(Job& j) {
    std::unique_lock<std::mutex> lk(q_mu_);
    done_cv_.wait(lk, [&] { return j.state.load() != Job::Queued; });
  }
  // The engine stream waits (device side) for the job's copy; a failed read is the call's error.
  void join(Job& j, cudaStream_t es) {
    if (j.state.load() == Job::Queued && j.pinned) flush_copies();
    wait_quiet(j);
    if (j.state.load() == Job::Failed) fail(j.err_status, j.err);
    ck(cudaStreamWaitEvent(es, j.done_ev, 0), "cudaStreamWaitEvent (unit)");
  }

  bool fetch_into_ring(int layer, int unit, bool spec = false) {
    const uint64_t st = stride(layer);
    auto rc = std::find_if(rings_.begin(), rings_.end(), [&](const RingClass& r) { return r.stride == st; });
    if (rc == rings_.end()) return false;
    for (size_t k = 0; k < rc->count; ++k) {
      const size_t i = rc->first + (rc->cursor + k) % rc->count;
      if (ring_[i].owner >= 0) continue;
      rc->cursor = (i - rc->first + 1) % rc->count;
      Lay& s = L_[size_t(layer)];
      JobPtr j = make_job(layer, unit, ring_[i].dev, spec);
      fwd_jobs_.push_back(j);
      j->wait_ev = ring_owner_ev_[i];
      ring_[i].owner = layer;
      ring_[i].job = j;
      s.loc[size_t(unit)] = kRing;
      s.slot[size_t(unit)] = int32_t(i);
      s.job[size_t(unit)] = j;
      (j->pinned ? fwd_[size_t(layer)].bytes_pinned : fwd_[size_t(layer)].bytes_disk) +=
          d_.layers[size_t(layer)].unit_bytes;
      submit(j);
      return true;
    }
    return false;
  }
  void fetch_into_persistent(int layer, int unit, int slot, cudaEvent_t dst_wb_ev = nullptr) {
    Lay& s = L_[size_t(layer)];
    JobPtr j = make_job(layer, unit, at(s.pool, uint64_t(slot) * stride(layer)));
    j->dst_wb_ev = dst_wb_ev;
    fwd_jobs_.push_back(j);
    s.loc[size_t(unit)] = kPersistent;
    s.slot[size_t(unit)] = slot;
    s.job[size_t(unit)] = j;
    (j->pinned ? fwd_[size_t(layer)].bytes_pinned : fwd_[size_t(layer)].bytes_disk) +=
        d_.layers[size_t(layer)].unit_bytes;
    submit(j);
  }
  // ---- exclusive tier mode ----
  int block_class(int layer) const { return excl_ ? layer_class_[size_t(layer)] : -1; }
  uint64_t free_block_count() const {
    uint64_t f = 0;
    for (const auto& v : free_blocks_) f += v.size();
    return f;
  }
  // Evictions an admission may make: one free block per victim; uncapped with exclusive_discard.
  int eviction_cap(int layer) const {
    if (!excl_) return -1;
    const int cls = block_class(layer);
    if (cls < 0) return 0;
    if (o_.exclusive_discard) return -1;
    return int(std::min<uint64_t>(free_blocks_[size_t(cls)].size(), uint64_t(INT32_MAX)));
  }
  // The admission's victims into free blocks on the write-back stream (the first ones, in ascending unit order, while
  // blocks last; with exclusive_discard the rest are discarded to their files). Returns the event the admitted units'
  // copies into those slots wait for, null when nothing is written back.
  cudaEvent_t write_back(int layer, const Admission& a, size_t* n_wb) {
    const Layer& l = d_.layers[size_t(layer)];
    const Lay& s = L_[size_t(layer)];
    const int cls = block_class(layer);
    const uint64_t room = cls < 0 ? 0 : free_blocks_[size_t(cls)].size();
    if (cls < 0 || (!o_.exclusive_discard && room < a.evicted.size()))
      fail(SS_E_BACKEND, "exclusive: more victims than free blocks (internal)");
    const size_t nw = size_t(std::min<uint64_t>(room, a.evicted.size()));
    *n_wb = nw;
    for (int32_t u : a.evicted)
      if (pinned_of_[size_t(gidx(layer, u))])
        fail(SS_E_BACKEND, "exclusive: an evicted resident still owns a block (internal)");
    xst_.discards += a.evicted.size() - nw;  // a discard copies nothing and takes no block
    if (!nw) return nullptr;
    std::lock_guard<std::mutex> lk(copy_mu_);
    if (wb_gate_) {  // the copies of earlier forwards (into these slots, out of these blocks) come first
      ck(cudaStreamWaitEvent(wb_stream_, blocks_ev_, 0), "cudaStreamWaitEvent (blocks)");
      wb_gate_ = false;
    }
    cudaEvent_t ev = event();
    wb_evs_.push_back(ev);
    auto kb = std::make_unique<dev::Batch>();
    for (size_t i = 0; i < nw; ++i) {
      const int64_t g = gidx(layer, a.evicted[i]);
      char* b = free_blocks_[size_t(cls)].back();
      free_blocks_[size_t(cls)].pop_back();
      pinned_of_[size_t(g)] = b;
      const char* src = at(s.pool, uint64_t(a.evicted_slot[i]) * stride(layer));
      if (l.unit_bytes >= ce_min_) {
        ck(cudaMemcpyAsync(b, src, size_t(l.unit_bytes), cudaMemcpyDeviceToHost, wb_stream_),
           "cudaMemcpyAsync (write-back)");
      } else {
        if (kb->n_copies == dev::kMaxCopies) launch_batch_on(*kb, wb_stream_);
        kb->copies[kb->n_copies++] = {src, b, l.unit_bytes};
      }
      ++xst_.writebacks;
      xst_.writeback_bytes += l.unit_bytes;
    }
    launch_batch_on(*kb, wb_stream_);
    ck(cudaEventRecord(ev, wb_stream_), "cudaEventRecord (write-back)");
    for (size_t i = 0; i < nw; ++i) {  // published after the record: a read of one of these blocks waits for it
      const int64_t g = gidx(layer, a.evicted[i]);
      wb_pending_[size_t(g)] = ev;
      wb_units_.push_back(g);
    }
    return ev;
  }
  // A unit that landed in a slot from its block no longer owns the block (its copy was issued; the block's next
  // writer waits for that copy through blocks_ev_ or a stream sync).
  void free_block(int layer, int unit) {
    const int64_t g = gidx(layer, unit);
    char* b = const_cast<char*>(pinned_of_[size_t(g)]);
    if (!b) return;
    free_blocks_[size_t(block_class(layer))].push_back(b);
    pinned_of_[size_t(g)] = nullptr;
    ++xst_.promoted;
  }
  void launch_batch_on(dev::Batch& kb, cudaStream_t st) {
    if (!kb.n_copies) return;
    uint64_t chunks = 0;
    for (uint32_t i = 0; i < kb.n_copies; ++i) chunks += (kb.copies[i].bytes + (64u << 10) - 1) >> 16;
    ck(cudaError_t(dev::launch_batch(kb, int(std::min<uint64_t>(std::max<uint64_t>(chunks, 1), 296)), st)),
       "land kernel");
    ++land_launches_;
    kb.n_copies = 0;
  }

  void dispatch_pending() {
    for (size_t L = 0; L < L_.size(); ++L) {
      Lay& s = L_[L];
      if (s.pending.empty()) continue;
      size_t k = 0;
      while (k < s.pending.size() && fetch_into_ring(int(L), s.pending[k])) ++k;
      s.pending.erase(s.pending.begin(), s.pending.begin() + std::ptrdiff_t(k));
      flush_copies();
      if (!s.pending.empty()) return;  // layer order: a later layer never overtakes an earlier one
    }
  }
  // The admitted units' copies into their slots; exclusive: the victims go back to free blocks first, and only a copy
  // into a written-back victim's slot waits for that write-back.
  void fetch_admitted(int layer, const Admission& a) {
    size_t n_wb = 0;
    cudaEvent_t wb_ev = excl_ && !a.evicted.empty() ? write_back(layer, a, &n_wb) : nullptr;
    for (size_t k = 0; k < a.admitted.size(); ++k) {
      cudaEvent_t wait = nullptr;
      for (size_t i = 0; wb_ev && i < n_wb && !wait; ++i)
        if (a.evicted_slot[i] == a.slot_of[k]) wait = wb_ev;
      fetch_into_persistent(layer, a.admitted[k], a.slot_of[k], wait);
    }
  }

  void ingest(int layer, const int32_t* ids, int n) {
    Lay& s = L_[size_t(layer)];
    const Layer& l = d_.layers[size_t(layer)];
    require(s.rs != nullptr, SS_E_INVALID, "routes: layer " + std::to_string(layer) + " has no units");
    require(!s.routes_given, SS_E_INVALID, "routes: given twice for layer " + std::to_string(layer));
    require(!s.skip, SS_E_INVALID, "routes: layer " + std::to_string(layer) + " is skipped in this forward");
    for (int i = 0; i < n; ++i)
      require(ids[i] < l.n_units, SS_E_INVALID, "routes: unit id " + std::to_string(ids[i]) + " out of range");
    s.routes_given = true;
    for (int i = 0; i < n; ++i)
      if (ids[i] >= 0) ++s.count[size_t(ids[i])];
    ss_layer_stats& st = fwd_[size_t(layer)];
    std::vector<int32_t> to_admit, misses;  // misses: prefetched this forward or not resident (SCORED's recency)
    std::vector<char> busy(size_t(l.n_units), 0);
    for (int u = 0; u < l.n_units; ++u) {
      const size_t x = size_t(u);
      const bool in_flight = s.loc[x] != kNone;  // fetched or prefetched in this forward already
      const bool wanted = s.count[x] != 0 && plan_.tier[size_t(gidx(layer, u))] != SS_TIER_PAIR;
      busy[x] = char(in_flight || wanted);
      if (!wanted) continue;
      s.routed.push_back(u);
      if (!in_flight && s.rs->slot(u) >= 0) {  // resident: a hit
        s.hits.push_back(u);
        continue;
      }
      misses.push_back(u);  // (SCORED's recency: prefetched in this forward, or not resident)
      if (!in_flight) {
        to_admit.push_back(u);
      } else if (s.spec_unclaimed[x]) {  // a speculative read the routes now claim: it moves up the queue
        s.spec_unclaimed[x] = 0;
        ++st.spec_used;
        if (s.job[x]) promote(s.job[x]);
      } else {
        ++st.prefetched;
      }
    }
    st.routed += s.routed.size();
    st.hits += s.hits.size();
    const Admission a = s.rs->admit(to_admit, busy, true, eviction_cap(layer));
    xst_.deferred += uint64_t(a.deferred);
    fetch_admitted(layer, a);
    for (int32_t u : a.transient)
      if (!fetch_into_ring(layer, u)) {
        s.pending.push_back(u);
        s.loc[size_t(u)] = kRing;  // placed when a ring slot frees
        ra_request(layer, u, true);
      }
    flush_copies();
    st.admitted += a.admitted.size();
    st.transient += a.transient.size();
    st.evicted += a.evicted.size();
    s.rs->observe(s.routed, misses);
  }

  void init() {
    require(int64_t(plan_.tier.size()) == d_.total_units, SS_E_INVALID, "open: plan does not match the descriptor");
    excl_ = b_.tier_mode == SS_TIER_MODE_EXCLUSIVE;
    // a resident's slot is the only copy an eviction writes back: it must hold the unit's bytes from open
    require(!(excl_ && !o_.fill_residents), SS_E_INVALID, "open: the exclusive tier mode needs fill_residents = 1");
    require(!(excl_ && o_.exclusive_discard && d_.tiers == Tiers::Pinned), SS_E_INVALID,
            "open: exclusive_discard needs a descriptor whose tiers allow disk (tiers = \"pinned\" refuses it)");
    require(o_.readahead_units <= 64, SS_E_INVALID, "open: readahead_units must be <= 64");
    require(!o_.spec_persistent, SS_E_UNSUPPORTED,
            "open: spec_persistent is not in this build (speculative prefetches take the stream ring)");
    ck(cudaSetDevice(o_.device), "cudaSetDevice");
    ck_launch_preload();
    ck(cudaStreamCreateWithFlags(&copy_, cudaStreamNonBlocking), "cudaStreamCreate (copy)");
    if (!o_.reader_threads) o_.reader_threads = 2;
    if (!o_.staging_buffers) o_.staging_buffers = 4;
    if (!o_.copy_piece_bytes) o_.copy_piece_bytes = uint64_t(64) << 20;
    ce_min_ = uint64_t(8) << 20;
    if (const char* e = std::getenv("TSB_CE_MIN_BYTES")) ce_min_ = std::strtoull(e, nullptr, 10);
    if (const char* e = std::getenv("TSB_COPY_MODE")) {
      if (!std::strcmp(e, "kernel")) ce_min_ = UINT64_MAX;
      else if (!std::strcmp(e, "ce")) ce_min_ = 0;
    }
    for (const Source& s : d_.sources) files_.push_back(std::make_unique<SourceFile>(s.path, s.align, o_.direct_io != 0));
    // pinned tier (the planner's layout, mapped: the land kernel reads it)
    pinned_of_.assign(size_t(d_.total_units), nullptr);
    const PinnedLayout pl = pinned_layout(d_, plan_.tier);
    {
      std::vector<size_t> sizes;
      for (uint64_t bytes : pl.chunk_bytes) sizes.push_back(size_t(bytes));
      pinned_ = alloc_pinned(sizes, o_.device);  // pinned.cu: mapped, populated in parallel, huge pages
      for (const PinnedChunk& c : pinned_) chunks_.push_back(c.ptr);
    }
    for (int64_t g = 0; g < d_.total_units; ++g)
      if (pl.chunk_of[size_t(g)] >= 0) pinned_of_[size_t(g)] = at(chunks_[size_t(pl.chunk_of[size_t(g)])], pl.offset_of[size_t(g)]);
    // exclusive: one block class per host stride, the plan's spare blocks (<= 1 GiB chunks, mapped: the land kernel
    // writes victims into them), the write-back stream and its events
    if (excl_) {
      ck(cudaStreamCreateWithFlags(&wb_stream_, cudaStreamNonBlocking), "cudaStreamCreate (write-back)");
      ck(cudaEventCreateWithFlags(&blocks_ev_, cudaEventDisableTiming), "cudaEventCreate");
      ck(cudaEventCreateWithFlags(&wb_mark_ev_, cudaEventDisableTiming), "cudaEventCreate");
      wb_pending_.assign(size_t(d_.total_units), nullptr);
      std::vector<uint64_t> block_bytes;
      for (const tsb::SpareClass& c : plan_.spares) block_bytes.push_back(c.block_bytes);
      free_blocks_.resize(block_bytes.size());
      layer_class_.assign(d_.layers.size(), -1);
      std::vector<uint64_t> class_total(block_bytes.size(), 0);
      for (size_t L = 0; L < d_.layers.size(); ++L) {
        const Layer& l = d_.layers[L];
        if (!l.streamable || !l.n_units) continue;
        const auto it = std::find(block_bytes.begin(), block_bytes.end(), host_stride(l.unit_bytes));
        require(it != block_bytes.end(), SS_E_INVALID, "open: exclusive plan without a block class (internal)");
        layer_class_[L] = int(it - block_bytes.begin());
        for (int u = 0; u < l.n_units; ++u)
          if (pinned_of_[size_t(gidx(int(L), u))]) ++class_total[size_t(layer_class_[L])];
      }
      for (size_t k = 0; k < plan_.spares.size(); ++k) {
        const uint64_t bytes = plan_.spares[k].block_bytes;
        const uint64_t per_chunk = std::max<uint64_t>(1, (uint64_t(1) << 30) / bytes);
        free_blocks_[k].reserve(size_t(class_total[k] + plan_.spares[k].blocks));  // never reallocates later
        std::vector<char*> blocks;
        std::vector<size_t> sizes;
        std::vector<uint64_t> units;
        for (uint64_t left = plan_.spares[k].blocks; left > 0;) {
          units.push_back(std::min(per_chunk, left));
          sizes.push_back(size_t(units.back() * bytes));
          left -= units.back();
        }
        std::vector<PinnedChunk> got = alloc_pinned(sizes, o_.device);
        for (size_t c = 0; c < got.size(); ++c) {
          for (uint64_t i = 0; i < units[c]; ++i) blocks.push_back(at(got[c].ptr, i * bytes));
          spare_pinned_.push_back(got[c]);
        }
        for (size_t i = blocks.size(); i-- > 0;) free_blocks_[k].push_back(blocks[i]);
        xst_.free_blocks += plan_.spares[k].blocks;
      }
      xst_.min_free_blocks = xst_.free_blocks;
      wb_units_.reserve(size_t(d_.total_units));
    }
    // staging for file reads: one unit of the largest file-tier unit each
    uint64_t disk_unit = 0;
    for (size_t L = 0; L < d_.layers.size(); ++L)
      for (int u = 0; u < d_.layers[L].n_units; ++u) {
        const uint8_t t = plan_.tier[size_t(gidx(int(L), u))];
        if (t == SS_TIER_DISK || (t == SS_TIER_RESIDENT && o_.fill_residents))
          disk_unit = std::max(disk_unit, host_stride(d_.layers[L].unit_bytes));
      }
    for (uint32_t i = 0; disk_unit && i < o_.staging_buffers; ++i) {
      void* p = nullptr;
      ck(cudaHostAlloc(&p, size_t(disk_unit), cudaHostAllocPortable), "cudaHostAlloc (staging)");
      staging_.push_back(static_cast<char*>(p));
      st_free_.push_back(i);
    }
    // host read-ahead: readahead_units pinned buffers of the largest streamable unit that has no pinned copy (none
    // when every such unit is pinned or a pair's), read by reader threads of their own
    if (o_.readahead_units) {
      for (size_t L = 0; L < d_.layers.size(); ++L) {
        if (!d_.layers[L].streamable) continue;
        for (int u = 0; u < d_.layers[L].n_units; ++u) {
          const uint8_t t = plan_.tier[size_t(gidx(int(L), u))];
          if (t == SS_TIER_PINNED || t == SS_TIER_PAIR) continue;
          ra_bytes_ = std::max(ra_bytes_, host_stride(d_.layers[L].unit_bytes));
          break;
        }
      }
      if (ra_bytes_) {
        for (uint32_t i = 0; i < o_.readahead_units; ++i) {
          void* p = nullptr;
          ck(cudaHostAlloc(&p, size_t(ra_bytes_), cudaHostAllocPortable), "cudaHostAlloc (read-ahead)");
          ra_bufs_.push_back(static_cast<char*>(p));
        }
        ra_ = std::make_unique<ReadAhead>(ra_bufs_, o_.reader_threads, [this](int layer, int unit, char* dst) {
          const Layer& l = d_.layers[size_t(layer)];
          read_unit(layer, unit, dst);
          if (o_.verify_hash && !l.hash.empty())
            require(xxh64(dst, size_t(l.unit_bytes)) == l.hash[size_t(unit)], SS_E_HASH,
                    "read: unit (" + std::to_string(layer) + ", " + std::to_string(unit) +
                        ") differs from its descriptor hash");
          return l.unit_bytes;
        });
      }
    }
    // layers: pools, events, tables
    L_.resize(d_.layers.size());
    for (size_t L = 0; L < d_.layers.size(); ++L) {
      const Layer& l = d_.layers[L];
      Lay& s = L_[L];
      ck(cudaEventCreateWithFlags(&s.release_ev, cudaEventDisableTiming), "cudaEventCreate");
      ck(cudaEventCreateWithFlags(&s.ready_ev, cudaEventDisableTiming), "cudaEventCreate");
      if (l.n_units == 0) continue;
      int planned = 0;
      for (int u = 0; u < l.n_units; ++u) {
        const uint8_t t = plan_.tier[size_t(gidx(int(L), u))];
        if (t == SS_TIER_RESIDENT || t == SS_TIER_RESIDENT_BACKED) ++planned;
      }
      const int cap = l.streamable ? std::min(l.n_units, planned + int(plan_.dynamic_slots_per_layer)) : l.n_units;
      s.rs = std::make_unique<ResidentSet>(l.n_units, cap, o_.policy == SS_POLICY_SCORED, o_.score_window);
      if (cap) {
        void* p = nullptr;
        ck(cudaMalloc(&p, size_t(uint64_t(cap) * stride(int(L)))), "cudaMalloc (pool)");
        s.pool = static_cast<char*>(p);
      }
      for (int v = 0; v < 2; ++v) {
        void* h = nullptr;
        ck(cudaHostAlloc(&h, sizeof(uint64_t) * size_t(l.n_units), cudaHostAllocPortable), "cudaHostAlloc (table)");
        std::memset(h, 0, sizeof(uint64_t) * size_t(l.n_units));
        s.table_host[v] = static_cast<uint64_t*>(h);
        void* dptr = nullptr;
        ck(cudaMalloc(&dptr, sizeof(uint64_t) * size_t(l.n_units)), "cudaMalloc (table)");
        s.table_dev[v] = static_cast<uint64_t*>(dptr);
        ck(cudaEventCreateWithFlags(&s.table_ev[v], cudaEventDisableTiming), "cudaEventCreate");
      }
      s.loc.assign(size_t(l.n_units), kNone);
      s.slot.assign(size_t(l.n_units), -1);
      s.job.assign(size_t(l.n_units), nullptr);
      s.count.assign(size_t(l.n_units), 0);
      s.spec_unclaimed.assign(size_t(l.n_units), 0);
    }
    for (const tsb::RingClass& rc : plan_.rings) {
      if (!rc.slots) continue;
      void* base = nullptr;
      ck(cudaMalloc(&base, size_t(rc.stride * rc.slots)), "cudaMalloc (ring)");
      ring_bases_.push_back(base);
      rings_.push_back({rc.stride, ring_.size(), rc.slots, 0});
      for (uint32_t i = 0; i < rc.slots; ++i) ring_.push_back({at(base, rc.stride * i), rc.stride, -1, nullptr});
    }
    ring_owner_ev_.assign(ring_.size(), nullptr);
    stats_.assign(d_.layers.size(), ss_layer_stats{});
    fwd_.assign(d_.layers.size(), ss_layer_stats{});
    for (uint32_t i = 0; i < o_.reader_threads; ++i) workers_.emplace_back([this] { worker(); });
    // fill: the pinned tier from the files (reader threads of our own here), then the residents
    fill_pinned();
    std::vector<JobPtr> fill;
    for (size_t L = 0; L < d_.layers.size(); ++L) {
      const Layer& l = d_.layers[L];
      Lay& s = L_[L];
      if (!s.rs) continue;
      for (int u = 0; u < l.n_units; ++u) {
        const uint8_t t = plan_.tier[size_t(gidx(int(L), u))];
        const bool res = !l.streamable || t == SS_TIER_RESIDENT || t == SS_TIER_RESIDENT_BACKED;
        if (!res) continue;
        const int slot = s.rs->place(u, !l.streamable || o_.pin_planned != 0);
        require(slot >= 0, SS_E_CAPACITY, "open: resident pool full (internal)");
        if (o_.fill_residents) {
          JobPtr j = make_job(int(L), u, at(s.pool, uint64_t(slot) * stride(int(L))));
          j->wait_ev = nullptr;
          fill.push_back(j);
          submit(j);
        }
      }
    }
    flush_copies();
    for (const JobPtr& j : fill) {
      wait_quiet(*j);
      if (j->state.load() == Job::Failed) fail(j->err_status, j->err);
    }
    ck(cudaStreamSynchronize(copy_), "cudaStreamSynchronize (fill)");
    for (const JobPtr& j : fill) pool_ev(j->done_ev);
  }
  void ck_launch_preload() { ck(cudaError_t(dev::preload()), "loading the kernels"); }
  void fill_pinned() {
    std::vector<std::pair<int, int>> units;
    for (size_t L = 0; L < d_.layers.size(); ++L)
      for (int u = 0; u < d_.layers[L].n_units; ++u)
        if (pinned_of_[size_t(gidx(int(L), u))]) units.push_back({int(L), u});
    std::atomic<size_t> next{0};
    std::mutex mu;
    std::string err;
    ss_status st = SS_OK;
    const unsigned n = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    std::vector<std::thread> th;
    for (unsigned t = 0; t < n; ++t)
      th.emplace_back([&] {
        for (;;) {
          const size_t i = next.fetch_add(1);
          if (i >= units.size()) return;
          const auto [L, u] = units[i];
          try {
            char* dst = const_cast<char*>(pinned_of_[size_t(gidx(L, u))]);
            read_unit(L, u, dst);
            const Layer& l = d_.layers[size_t(L)];
            if (o_.verify_hash && !l.hash.empty())
              require(xxh64(dst, size_t(l.unit_bytes)) == l.hash[size_t(u)], SS_E_HASH,
                      "open: unit (" + std::to_string(L) + ", " + std::to_string(u) + ") differs from its hash");
          } catch (const Error& e) {
            std::lock_guard<std::mutex> lk(mu);
            if (st == SS_OK) {
              st = e.status();
              err = e.what();
            }
          }
        }
      });
    for (auto& t : th) t.join();
    if (st != SS_OK) fail(st, err);
  }
  void close() noexcept {
    {
      std::lock_guard<std::mutex> lk(q_mu_);
      stop_ = true;
    }
    q_cv_.notify_all();
    st_cv_.notify_all();
    for (auto& t : workers_)
      if (t.joinable()) t.join();
    workers_.clear();
    ra_.reset();  // its readers end before their buffers go
    if (copy_) cudaStreamSynchronize(copy_);
    if (wb_stream_) cudaStreamSynchronize(wb_stream_);
    cudaDeviceSynchronize();
    for (Lay& s : L_) {
      if (s.pool) cudaFree(s.pool);
      for (int v = 0; v < 2; ++v) {
        if (s.table_dev[v]) cudaFree(s.table_dev[v]);
        if (s.table_host[v]) cudaFreeHost(s.table_host[v]);
        if (s.table_ev[v]) cudaEventDestroy(s.table_ev[v]);
      }
      if (s.release_ev) cudaEventDestroy(s.release_ev);
      if (s.ready_ev) cudaEventDestroy(s.ready_ev);
    }
    L_.clear();
    for (void* b : ring_bases_) cudaFree(b);
    ring_bases_.clear();
    free_pinned(pinned_);
    chunks_.clear();
    free_pinned(spare_pinned_);
    if (wb_stream_) cudaStreamDestroy(wb_stream_);
    wb_stream_ = nullptr;
    if (blocks_ev_) cudaEventDestroy(blocks_ev_);
    if (wb_mark_ev_) cudaEventDestroy(wb_mark_ev_);
    blocks_ev_ = wb_mark_ev_ = nullptr;
    for (char* s : staging_) cudaFreeHost(s);
    staging_.clear();
    for (char* s : ra_bufs_) cudaFreeHost(s);
    ra_bufs_.clear();
    for (cudaEvent_t e : all_ev_) cudaEventDestroy(e);
    all_ev_.clear();
    if (copy_) cudaStreamDestroy(copy_);
    copy_ = nullptr;
  }

  Desc d_;
  ss_budget b_;
  Plan plan_;
  ss_options o_;
  std::vector<std::unique_ptr<SourceFile>> files_;
  std::vector<Lay> L_;
  std::vector<Ring> ring_;
  std::vector<RingClass> rings_;
  std::vector<void*> ring_bases_;
  std::vector<cudaEvent_t> ring_owner_ev_;
  std::vector<void*> chunks_;       // the pinned tier's chunks (host addresses)
  std::vector<PinnedChunk> pinned_;  // their allocation
  std::vector<const char*> pinned_of_;
  std::vector<char*> staging_;
  std::vector<size_t> st_free_;
  std::unique_ptr<ReadAhead> ra_;  // host read-ahead (readahead_units > 0 and a unit without a pinned copy)
  std::vector<char*> ra_bufs_;
  uint64_t ra_bytes_ = 0;
  RaStats ra_st_;
  std::mutex st_mu_;
  std::condition_variable st_cv_;
  cudaStream_t copy_ = nullptr;
  std::mutex copy_mu_;
  std::mutex q_mu_;
  std::condition_variable q_cv_, done_cv_;
  std::deque<JobPtr> queue_, spec_queue_;
  std::vector<std::thread> workers_;
  bool stop_ = false;
  std::vector<JobPtr> batch_, fwd_jobs_;
  std::vector<cudaEvent_t> ev_pool_, all_ev_;
  std::vector<ss_layer_stats> stats_, fwd_;
  ss_stats_hook hook_ = nullptr;
  void* hook_user_ = nullptr;
  bool in_fwd_ = false, fwd_open_ = false, poisoned_ = false, stream_set_ = false;
  void* stream_ = nullptr;
  uint64_t forwards_ = 0, ce_min_ = 0, land_launches_ = 0;
  // exclusive tier mode
  bool excl_ = false, wb_gate_ = false;
  cudaStream_t wb_stream_ = nullptr;
  cudaEvent_t blocks_ev_ = nullptr, wb_mark_ev_ = nullptr;
  std::vector<cudaEvent_t> wb_pending_;  // per unit: the write-back into its block this forward
  std::vector<int64_t> wb_units_;
  std::vector<cudaEvent_t> wb_evs_;
  std::vector<int> layer_class_;                 // per layer: its block class (-1: none)
  std::vector<std::vector<char*>> free_blocks_;  // per class, the lowest address last (taken first)
  std::vector<PinnedChunk> spare_pinned_;
  ss_exclusive_stats xst_{};
};

}  // namespace

std::unique_ptr<HostContext> open_host_context(const Desc& d, const ss_budget& b, const Plan& p, const ss_options& o) {
  require(o.backend == SS_BACKEND_CUDA, SS_E_UNSUPPORTED, "ss_open: this build has the CUDA backend only");
  return std::make_unique<HostCtx>(d, b, p, o);
}

}  // namespace tsb
