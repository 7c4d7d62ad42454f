// Reference harness (TEST INFRASTRUCTURE): drives the reference library's own DgCore, compiled from its sources, the
// way its DgService::serve_token drives it (dg_service.cpp:269-365), with a host transport in the pattern of its
// tests' immediate transport (tests/test_dg_service.cpp:33-85): every event complete when queried, copies done at
// once. The product library never links this file.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <exception>
#include <thread>
#include <vector>

#include "dg_core.hpp"
#include "dg_score.hpp"
#include "oref.h"
#include "xxh64.hpp"

namespace {

// Copies of the host transport on every host thread (the timed baseline uses what the machine has): pieces of at
// least 4 MiB each, one thread per piece.
unsigned copy_threads() {
  static const unsigned n = std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
  return n;
}
void pcopy(void* dst, const void* src, size_t n) {
  const unsigned t = std::min<unsigned>(copy_threads(), unsigned(std::max<size_t>(1, n >> 22)));
  if (t <= 1) {
    std::memcpy(dst, src, n);
    return;
  }
  const size_t per = (n / t + 4095) / 4096 * 4096;
  std::vector<std::thread> th;
  for (unsigned i = 0; i < t; ++i) {
    const size_t lo = size_t(i) * per, hi = std::min(n, lo + per);
    if (lo >= hi) break;
    th.emplace_back([=] { std::memcpy(static_cast<char*>(dst) + lo, static_cast<const char*>(src) + lo, hi - lo); });
  }
  for (auto& x : th) x.join();
}

class HostTransport final : public ts::DgTransport {
 public:
  HostTransport(const oref_dg_config& c, uint32_t keys, uint32_t slots)
      : parts_(c.part_bytes, c.part_bytes + c.n_parts), table_(keys, -1), move_(c.move_bytes != 0) {
    for (uint64_t b : parts_) unit_ += b;
    // move_bytes 2: a timing sample, every copy moves its real bytes but slots and blocks alias a ring of 16 unit
    // buffers each, far above a host's last-level cache for the benchmark's units (the bytes read back through the
    // table are then not meaningful)
    alias_slots_ = c.move_bytes == 2 ? 16 : slots;
    alias_blocks_ = c.move_bytes == 2 ? 16 : c.blocks + c.disk_staging + c.landing_blocks;
    if (move_) {
      arena_.assign(size_t(alias_slots_) * unit_, 1);
      blocks_.assign(size_t(alias_blocks_) * unit_, 2);
      stage_.assign(unit_, 0);
    }
  }
  uint8_t* slot_ptr(int32_t s) { return arena_.data() + size_t(uint32_t(s) % alias_slots_) * unit_; }
  uint8_t* block_ptr(int32_t b) {
    return b < 0 ? stage_.data() : blocks_.data() + size_t(uint32_t(b) % alias_blocks_) * unit_;
  }
  uint32_t alias_slots_ = 1, alias_blocks_ = 1;
  void h2d(Stream, int32_t slot, int32_t block) override {
    if (move_) pcopy(slot_ptr(slot), block_ptr(block), unit_);
  }
  void d2h(int32_t slot, int32_t block) override {
    if (move_) pcopy(block_ptr(block), slot_ptr(slot), unit_);
  }
  void d2d(int32_t src, int32_t dst) override {
    if (move_) std::memmove(slot_ptr(dst), slot_ptr(src), unit_);
  }
  void h2h(int32_t src, int32_t dst) override {
    if (move_) std::memmove(block_ptr(dst), block_ptr(src), unit_);
  }
  // three-tier: the unit's bytes as its file holds them (synchronous, the transport's read_unit contract)
  void read_unit(uint32_t key, int32_t block) override {
    if (move_ && files_) pcopy(block_ptr(block), files_ + size_t(key) * unit_, unit_);
  }
  const uint8_t* files_ = nullptr;
  void d2h_part(Stream, int32_t slot, int32_t block, uint32_t p) override {
    if (!move_) return;
    uint64_t off = 0;
    for (uint32_t i = 0; i < p; ++i) off += parts_[i];
    pcopy(block_ptr(block) + off, slot_ptr(slot) + off, parts_[p]);
  }
  uint32_t parts() const override { return uint32_t(parts_.size()); }
  uint64_t part_bytes(uint32_t p) const override { return parts_[p]; }
  void write_entry(Stream, uint32_t key, int32_t v) override { table_[key] = v; }
  void signal_ready(uint32_t, uint32_t) override {}
  void* event_create() override { return new int(0); }
  void event_destroy(void* ev) override { delete static_cast<int*>(ev); }
  void record(void*, Stream) override {}
  void wait(Stream, void*) override {}
  bool done(void*) override { return true; }
  void event_sync(void*) override {}
  void sync(Stream) override {}
  void upload_table(const int32_t* t, uint32_t n) override { std::memcpy(table_.data(), t, size_t(n) * 4); }
  void upload_table_ranges(const int32_t* t, const uint32_t* r, uint32_t n) override {
    for (uint32_t i = 0; i < n; ++i) std::memcpy(table_.data() + r[2 * i], t + r[2 * i], size_t(r[2 * i + 1]) * 4);
  }
  std::vector<uint64_t> parts_;
  std::vector<int32_t> table_;  // the "device" table the export rule reads
  std::vector<uint8_t> arena_, blocks_, stage_;
  uint64_t unit_ = 0;
  bool move_;
};

uint64_t checksum(const uint8_t* p, uint64_t n) {
  uint64_t s = 0;
  for (uint64_t i = 0; i < n; ++i) s += uint64_t(p[i]) * (i % 251 + 1);
  return s;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) uint64_t oref_xxh64(const void* data, size_t len, uint64_t seed) {
  return ts::xxh64(data, len, seed);
}

extern "C" __attribute__((visibility("default"))) int oref_dg_replay(const oref_dg_config* c, const int32_t* ids,
                                                                      const int32_t* preds, int32_t* tables,
                                                                      uint64_t* stats, const uint8_t* src_units,
                                                                      uint64_t* read_sum, char* err, size_t errlen) {
  try {
    ts::DgConfig cfg;
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
    cfg.max_ids = c->n_ids ? c->n_ids : 1;
    cfg.inclusive = c->inclusive;
    cfg.disk_tier = c->disk_tier != 0;
    cfg.disk_prefetch = c->disk_prefetch != 0;
    cfg.home_blocks = c->home_blocks;
    cfg.disk_staging = c->disk_staging;
    cfg.disk_queue = c->disk_queue ? c->disk_queue : 1;  // (its transport's begin is the synchronous read)
    cfg.scored = c->policy != 0;  // the bounded boundary selection, as its device-gated context configures it
    cfg.scored_auto = c->policy == 2;
    cfg.boundary_score = true;
    cfg.no_admit = c->no_admit != 0;
    cfg.clean_evict = c->clean_evict != 0;
    cfg.pf_revert = c->pf_revert != 0;
    cfg.pf_strict = c->pf_strict != 0;
    cfg.bank_keep = c->bank_keep;
    cfg.landing_blocks = c->landing_blocks;
    cfg.landing_ttl = c->landing_ttl;
    if (c->w_trans || c->w_freq || c->w_rec) {
      cfg.w_trans = c->w_trans;
      cfg.w_freq = c->w_freq;
      cfg.w_rec = c->w_rec;
    }
    uint32_t keys = 0;
    for (uint32_t g = 0; g < c->n_gated; ++g) keys += c->n_units[g];
    const uint32_t slots = c->persistent_slots + 2 * c->bank_slots + 1;
    HostTransport t(*c, keys, slots);
    t.files_ = src_units;
    ts::DgCore core(cfg, &t);
    std::vector<uint32_t> order(c->order, c->order + c->n_order);
    for (uint32_t k = 0; k < keys; ++k) order.push_back(k);
    std::vector<uint8_t> disk;
    if (cfg.disk_tier && c->disk) disk.assign(c->disk, c->disk + keys);
    core.place(order, disk.empty() ? nullptr : &disk);
    if (c->profile && cfg.scored) {  // through the profile format: written, then checked and loaded
      std::vector<std::vector<uint32_t>> cells(c->n_gated);
      const uint32_t* p = c->profile;
      for (uint32_t g = 0; g < c->n_gated; ++g) {
        cells[g].assign(p, p + size_t(c->n_units[g]) * c->n_units[g]);
        p += size_t(c->n_units[g]) * c->n_units[g];
      }
      const std::string id(32, '\x5a');
      const std::string blob = ts::dg_profile_write(cfg.n_units, id, "replay", cells);
      core.load_profile(blob.data(), blob.size(), id);
    }
    t.upload_table(core.table().data(), keys);
    if (t.move_ && src_units && c->move_bytes == 1)  // the open's fill: every unit into its slot or block
      for (uint32_t k = 0; k < keys; ++k) {
        if (core.slot_of(k) < 0 && core.block_of(k) < 0) continue;  // (three-tier: a file home stays in its file)
        uint8_t* dst = core.slot_of(k) >= 0 ? t.slot_ptr(core.slot_of(k)) : t.block_ptr(core.block_of(k));
        std::memcpy(dst, src_units + size_t(k) * t.unit_, t.unit_);
      }
    std::vector<uint32_t> row(c->n_ids), pred(c->n_pred);
    uint64_t rsum[6] = {0, 0, 0, 0, 0, 0};
      std::vector<std::vector<uint32_t>> held_keys(c->n_gated);  // kept-resident layers
      std::vector<uint8_t> held(c->n_gated, 0);
      auto kept_all = [&] {
        std::vector<uint32_t> v;
        for (const auto& h : held_keys) v.insert(v.end(), h.begin(), h.end());
        return v;
      };
    for (uint32_t tok = 0; tok < c->tokens; ++tok) {
      std::vector<uint8_t> run(c->n_gated, 1);  // a held layer is not exported
      for (uint32_t g = 0; g < c->n_gated; ++g) run[g] = held[g] ? 0 : 1;
      core.begin_token(tok + 1, &run);
      for (uint32_t g = 0; g < c->n_gated; ++g) {
        if (!run[g]) continue;
        uint32_t nx = g + 1;
        while (nx < c->n_gated && !run[nx]) ++nx;
        const int32_t* r = ids + (size_t(tok) * c->n_gated + g) * c->n_ids;
        uint64_t mask = 0;
        for (uint32_t i = 0; i < c->n_ids; ++i) {  // the export kernel's rule on the device table
          row[i] = uint32_t(r[i]);
          if (row[i] < c->n_units[g] && t.table_[core.key(g, row[i])] < 0) mask |= 1ull << i;
        }
        core.serve_demand(g, row.data(), c->n_ids, mask);
        if (read_sum && t.move_)
          for (uint32_t i = 0; i < c->n_ids; ++i) {
            const int32_t s = t.table_[core.key(g, row[i])];
            read_sum[(size_t(tok) * c->n_gated + g) * c->n_ids + i] = s < 0 ? 0 : checksum(t.slot_ptr(s), t.unit_);
          }
        core.serve_use(g, row.data(), c->n_ids, mask);
        if (preds && c->n_pred && g + 1 < c->n_gated && run[g + 1]) {
          const int32_t* p = preds + (size_t(tok) * c->n_gated + g) * c->n_pred;
          for (uint32_t i = 0; i < c->n_pred; ++i) pred[i] = uint32_t(p[i]);
          core.serve_prediction(g + 1, pred.data(), c->n_pred, c->n_ids, false);
        }
        if (core.deferred() && nx < c->n_gated) core.issue_writebacks(g, [] { return false; });
        if (core.scored()) core.score_layer(g);  // (the service closes each layer after its work, scored only)
      }
      core.end_token(kept_all(), c->rows ? c->rows : 1);
      if (c->reset_at && tok + 1 == c->reset_at) {  // every keep and hold dropped
        core.reset_open();
        for (auto& h : held_keys) h.clear();
        std::fill(held.begin(), held.end(), uint8_t(0));
      }
      if (c->round_every && (tok + 1) % c->round_every == 0) {  // ss_dg_round between tokens, nothing kept
        ts::DgRoundIn in;
        in.budget_bytes = c->round_budget;
        in.max_units = c->round_max_units;
        in.hysteresis = double(c->round_hysteresis);
        in.decay = double(c->round_decay);
        const ts::DgRoundOut r = core.round(in, kept_all());
        rsum[0] += 1;
        rsum[1] += r.promoted_to_device;
        rsum[2] += r.promoted_to_pinned;
        rsum[3] += r.demoted_from_device;
        rsum[4] += r.dropped_to_file;
        rsum[5] += r.bytes_read + r.bytes_h2d + r.bytes_written_back;
      }
      for (uint32_t i = 0, at = 0; i < c->mr_n; at += c->mr_count[i], ++i) {  // kept-resident events
        if (c->mr_token[i] != tok) continue;
        const uint32_t lg = c->mr_layer[i];
        std::vector<uint32_t> want(c->mr_ids + at, c->mr_ids + at + c->mr_count[i]), held_now;
        if (want.empty()) {
          held_keys[lg].clear();
          held[lg] = 0;
          continue;
        }
        core.make_resident(lg, want, kept_all());
        for (uint32_t u : want) held_now.push_back(core.key(lg, u));
        held_keys[lg] = held_now;
        held[lg] = 1;
      }
      if (c->rstats) std::memcpy(c->rstats + size_t(tok) * 6, rsum, sizeof rsum);
      if (c->mstats) {
        const auto& q = core.stats();
        const uint64_t mv[4] = {q.resident_units, q.resident_evicted, q.mkres_file_reads, q.mkres_wb_bytes};
        std::memcpy(c->mstats + size_t(tok) * 4, mv, sizeof mv);
      }
      if (c->sstats) {
        const ts::DgStats& q = core.stats();
        const uint64_t sv[5] = {q.score_fallbacks, q.scored_victims, q.score_layers, q.score_candidates,
                                q.score_saturated};
        std::memcpy(c->sstats + size_t(tok) * 5, sv, sizeof sv);
      }
      if (c->qstats) {
        const ts::DgStats& q = core.stats();
        const uint64_t qv[4] = {q.disk_overlapped, q.disk_max_in_flight, q.disk_carried, q.disk_carried_bytes};
        std::memcpy(c->qstats + size_t(tok) * 4, qv, sizeof qv);
      }
      if (c->pstats) {
        const ts::DgStats& q = core.stats();
        const uint64_t pv[5] = {q.clean_drops, q.clean_drop_bytes, q.pf_reverted, q.pf_revert_bytes,
                                q.pf_strict_refused};
        std::memcpy(c->pstats + size_t(tok) * 5, pv, sizeof pv);
      }
      if (c->kstats) {  // FNV-1a 64 of the pinned recency order, each key's 4 little-endian bytes
        const ts::DgStats& q = core.stats();
        uint64_t h = 0xcbf29ce484222325ull;
        for (uint32_t k : core.host_order())
          for (int b = 0; b < 4; ++b) h = (h ^ ((k >> (8 * b)) & 0xffu)) * 0x100000001b3ull;
        const uint64_t kv[4] = {q.bank_kept, q.bank_keep_drops, q.bank_keep_rereads, h};
        std::memcpy(c->kstats + size_t(tok) * 4, kv, sizeof kv);
      }
      if (c->lstats) {
        const ts::DgStats& q = core.stats();
        const uint64_t lv[9] = {q.landing_issued,  q.landing_promoted,     q.landing_late,
                                q.landing_expired, q.landing_dropped_full, q.landing_read_bytes,
                                q.landing_expired_layer, q.landing_skipped_passed, core.landing_units()};
        std::memcpy(c->lstats + size_t(tok) * 9, lv, sizeof lv);
      }
      std::memcpy(tables + size_t(tok) * keys, t.table_.data(), size_t(keys) * 4);
      const ts::DgStats& s = core.stats();
      const uint64_t v[OREF_NSTATS] = {s.tokens,          s.lookups,     s.misses,        s.covered,
                                       s.fetched,         s.prefetched,  s.prefetch_used, s.resurrected,
                                       s.bank_serves,     s.collected_mid, s.evicted,     s.evict_short,
                                       s.writebacks_done, s.wb_deferred, s.wb_cancelled,  s.wb_forced};
      std::memcpy(stats + size_t(tok) * OREF_NSTATS, v, sizeof v);
      if (c->xstats) {
        const uint64_t xv[OREF_NXSTATS] = {s.disk_reads, s.disk_read_bytes, s.disk_stage_waits, s.disk_drops,
                                           s.disk_discards, core.file_units()};
        std::memcpy(c->xstats + size_t(tok) * OREF_NXSTATS, xv, sizeof xv);
      }
      core.check();
    }
    return 0;
  } catch (const std::exception& e) {
    if (err && errlen) std::snprintf(err, errlen, "%s", e.what());
    return -1;
  }
}

extern "C" __attribute__((visibility("default"))) unsigned oref_copy_threads(void) { return copy_threads(); }

// The reference's adaptive read depth controller (src/dg_load.hpp:151-206) fed busy periods: the same outputs as
// tsb_test_read_depth (depth after each period, 11 counters, the verdict ring as 7 doubles each).
#include "dg_load.hpp"
extern "C" __attribute__((visibility("default"))) int oref_read_depth(uint32_t bound, const double* params, uint32_t n,
                                                                       const uint64_t* reads, const uint64_t* bytes,
                                                                       const uint64_t* ns, uint32_t* depth,
                                                                       uint64_t* counters, double* verdicts,
                                                                       uint32_t* n_verdicts) {
  ts::DgDepthCtl::Params p;
  if (params) {
    p.min_reads = uint64_t(params[0]);
    p.recheck_u = uint64_t(params[1]);
    p.backoff_1 = uint64_t(params[2]);
    p.backoff_max = uint64_t(params[3]);
    p.bar = params[4];
    p.drift = params[5];
  }
  ts::DgDepthCtl c(bound, p);
  for (uint32_t i = 0; i < n; ++i) depth[i] = c.on_busy(reads[i], bytes[i], ns[i]);
  const uint64_t v[11] = {c.changes, c.calibrations, c.windows, c.reads1, c.bytes1, c.ns1,
                          c.readsu, c.bytesu, c.nsu, c.decisions(), c.calibrating() ? 1u : 0u};
  std::memcpy(counters, v, sizeof v);
  uint32_t at = 0;
  for (const ts::DgDepthCtl::Decision& d : c.ring()) {
    const double row[7] = {double(d.seq), double(d.reads), double(d.from), double(d.to), d.rate_u, d.rate_1,
                           double(d.reason)};
    std::memcpy(verdicts + size_t(at) * 7, row, sizeof row);
    ++at;
  }
  *n_verdicts = at;
  return 0;
}
