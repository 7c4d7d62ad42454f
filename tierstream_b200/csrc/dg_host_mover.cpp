// A host mover for the slot cache (dg_core.hpp): the arena and the blocks are host arrays, every copy happens when
// enqueued, every event is complete when queried. It runs the deterministic replay test hook (tsb_test_dg_replay),
// which the CPU tests compare with the reference's own DgCore on the same trace; no context uses it.
#include <cstdio>
#include <cstring>
#include <vector>

#include "dg_core.hpp"
#include "errors.hpp"
#include "tierstream/tsb.h"

namespace tsb {
namespace {

class HostMover final : public Mover {
 public:
  HostMover(const std::vector<uint64_t>& parts, uint32_t keys, uint32_t slots, uint32_t blocks, bool move,
            const uint8_t* files)
      : parts_(parts), table_(keys, -1), move_(move), files_(files) {
    for (uint64_t b : parts_) unit_ += b;
    if (move_) {
      arena_.assign(size_t(slots) * unit_, 0);
      blocks_.assign(size_t(blocks) * unit_, 0);
      stage_.assign(unit_, 0);
    }
  }
  uint8_t* slot_ptr(int32_t s) { return arena_.data() + size_t(s) * unit_; }
  uint8_t* block_ptr(int32_t b) { return b < 0 ? stage_.data() : blocks_.data() + size_t(b) * unit_; }
  uint32_t parts() const override { return uint32_t(parts_.size()); }
  uint64_t part_bytes(uint32_t p) const override { return parts_[p]; }
  void h2d(Stream, int32_t slot, int32_t block, uint32_t) override {
    if (move_) std::memcpy(slot_ptr(slot), block_ptr(block), unit_);
  }
  void d2h(Stream, int32_t slot, int32_t block, int32_t p, uint32_t) override {
    if (!move_) return;
    uint64_t off = 0;
    for (uint32_t i = 0; i < parts_.size(); ++i) {
      if (p < 0 || uint32_t(p) == i) std::memcpy(block_ptr(block) + off, slot_ptr(slot) + off, parts_[i]);
      off += parts_[i];
    }
  }
  void d2d_moves(const std::vector<std::pair<int32_t, int32_t>>& moves, const std::vector<uint32_t>& wave) override {
    uint32_t top = 0;
    for (uint32_t w : wave) top = std::max(top, w);
    for (uint32_t w = 0; w <= top; ++w)
      for (size_t i = 0; i < moves.size(); ++i)
        if (wave[i] == w && move_) std::memmove(slot_ptr(moves[i].second), slot_ptr(moves[i].first), unit_);
  }
  void h2h(int32_t src, int32_t dst, uint32_t) override {
    if (move_) std::memmove(block_ptr(dst), block_ptr(src), unit_);
  }
  void read_unit(uint32_t key, int32_t block) override {
    if (move_ && files_) std::memcpy(block_ptr(block), files_ + size_t(key) * unit_, unit_);
  }
  void publish(Stream, uint32_t key, int32_t v) override { table_[key] = v; }
  void ready(uint32_t, uint32_t) override {}
  void* event_create() override { return new int(0); }
  void event_destroy(void* ev) override { delete static_cast<int*>(ev); }
  void record(void*, Stream) override {}
  void wait(Stream, void*) override {}
  bool done(void*) override { return true; }
  void event_sync(void*) override {}
  void sync(Stream) override {}
  void upload_table(const int32_t* t, uint32_t n) override { std::memcpy(table_.data(), t, size_t(n) * 4); }
  void upload_table_ranges(const int32_t* t, const uint32_t* ranges, uint32_t n) override {
    for (uint32_t i = 0; i < n; ++i)
      std::memcpy(table_.data() + ranges[2 * i], t + ranges[2 * i], size_t(ranges[2 * i + 1]) * 4);
  }

  std::vector<uint64_t> parts_;
  std::vector<int32_t> table_;
  std::vector<uint8_t> arena_, blocks_, stage_;
  uint64_t unit_ = 0;
  bool move_;
  const uint8_t* files_;  // each unit's bytes as its file holds them (file tier)
};

uint64_t checksum(const uint8_t* p, uint64_t n) {
  uint64_t s = 0;
  for (uint64_t i = 0; i < n; ++i) s += uint64_t(p[i]) * (i % 251 + 1);
  return s;
}

}  // namespace

void dg_replay(const tsb_dg_replay_config* c, const int32_t* ids, const int32_t* preds, int32_t* tables,
               uint64_t* stats, const uint8_t* src_units, uint64_t* read_sum) {
  require(c && c->n_units && c->part_bytes && ids && tables && stats, SS_E_INVALID, "tsb_test_dg_replay: null argument");
  require(c->n_ids >= 1 && c->n_ids <= 64 && c->n_pred <= 64, SS_E_INVALID, "tsb_test_dg_replay: 1..64 ids");
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
  require(c->policy <= 2, SS_E_INVALID, "tsb_test_dg_replay: policy 0..2");
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
  uint32_t keys = 0;
  for (uint32_t g = 0; g < c->n_gated; ++g) keys += c->n_units[g];
  HostMover m(std::vector<uint64_t>(c->part_bytes, c->part_bytes + c->n_parts), keys,
              c->persistent_slots + 2 * c->bank_slots + 1, c->blocks + c->disk_staging + c->landing_blocks,
              c->move_bytes != 0, src_units);
  SlotCache core(cfg, &m);
  std::vector<uint32_t> order(c->order, c->order + c->n_order);
  for (uint32_t k = 0; k < keys; ++k) order.push_back(k);
  std::vector<uint8_t> disk;
  if (cfg.disk_tier && c->disk) disk.assign(c->disk, c->disk + keys);
  core.place(order, disk.empty() ? nullptr : &disk);
  if (c->profile && cfg.scored) {
    std::vector<std::vector<uint32_t>> cells(c->n_gated);
    const uint32_t* p = c->profile;
    for (uint32_t g = 0; g < c->n_gated; ++g) {
      cells[g].assign(p, p + size_t(c->n_units[g]) * c->n_units[g]);
      p += size_t(c->n_units[g]) * c->n_units[g];
    }
    core.load_counts(cells);
  }
  m.upload_table(core.table().data(), keys);
  if (m.move_ && src_units)  // the open's fill: every unit with a slot or a block (a file home stays in its file)
    for (uint32_t k = 0; k < keys; ++k) {
      if (core.slot_of(k) < 0 && core.block_of(k) < 0) continue;
      uint8_t* dst = core.slot_of(k) >= 0 ? m.slot_ptr(core.slot_of(k)) : m.block_ptr(core.block_of(k));
      std::memcpy(dst, src_units + size_t(k) * m.unit_, m.unit_);
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
  for (uint32_t t = 0; t < c->tokens; ++t) {
    std::vector<uint8_t> run(c->n_gated, 1);  // a held layer is not exported
    for (uint32_t g = 0; g < c->n_gated; ++g) run[g] = held[g] ? 0 : 1;
    core.begin_token(t + 1, &run);
    for (uint32_t g = 0; g < c->n_gated; ++g) {
      if (!run[g]) continue;
      uint32_t nx = g + 1;
      while (nx < c->n_gated && !run[nx]) ++nx;
      const int32_t* r = ids + (size_t(t) * c->n_gated + g) * c->n_ids;
      uint64_t mask = 0;
      for (uint32_t i = 0; i < c->n_ids; ++i) {  // the export kernel's rule on the device table
        row[i] = uint32_t(r[i]);
        if (row[i] < c->n_units[g] && m.table_[core.key(g, row[i])] < 0) mask |= 1ull << i;
      }
      core.serve_demand(g, row.data(), c->n_ids, mask);
      if (read_sum && m.move_)
        for (uint32_t i = 0; i < c->n_ids; ++i) {
          const int32_t s = m.table_[core.key(g, row[i])];
          read_sum[(size_t(t) * c->n_gated + g) * c->n_ids + i] = s < 0 ? 0 : checksum(m.slot_ptr(s), m.unit_);
        }
      core.serve_use(g, row.data(), c->n_ids, mask);
      if (preds && c->n_pred && g + 1 < c->n_gated && run[g + 1]) {
        const int32_t* p = preds + (size_t(t) * c->n_gated + g) * c->n_pred;
        for (uint32_t i = 0; i < c->n_pred; ++i) pred[i] = uint32_t(p[i]);
        core.serve_prediction(g + 1, pred.data(), c->n_pred, false);
      }
      if (core.deferred() && nx < c->n_gated) core.issue_writebacks(g, [] { return false; });
      if (core.scored()) core.score_layer(g);  // (the service closes a layer for scoring only)
    }
    core.end_token(kept_all(), c->rows ? c->rows : 1);
    if (c->reset_at && t + 1 == c->reset_at) {  // every keep and hold dropped
      core.reset_open();
      for (auto& h : held_keys) h.clear();
      std::fill(held.begin(), held.end(), uint8_t(0));
    }
    if (c->round_every && (t + 1) % c->round_every == 0) {
      RoundIn in;
      in.budget_bytes = c->round_budget;
      in.max_units = c->round_max_units;
      in.hysteresis = double(c->round_hysteresis);
      in.decay = double(c->round_decay);
      const RoundOut r = core.round(in, kept_all());
      rsum[0] += 1;
      rsum[1] += r.promoted_to_device;
      rsum[2] += r.promoted_to_pinned;
      rsum[3] += r.demoted_from_device;
      rsum[4] += r.dropped_to_file;
      rsum[5] += r.bytes_read + r.bytes_h2d + r.bytes_written_back;
    }
    for (uint32_t i = 0, at = 0; i < c->mr_n; at += c->mr_count[i], ++i) {  // kept-resident events
      if (c->mr_token[i] != t) continue;
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
    core.set_range_uploads(std::any_of(held.begin(), held.end(), [](auto h) { return h != 0; }));
    if (c->rstats) std::memcpy(c->rstats + size_t(t) * 6, rsum, sizeof rsum);
    if (c->mstats) {
      const auto& q = core.stats();
      const uint64_t mv[4] = {q.resident_units, q.resident_evicted, q.mkres_file_reads, q.mkres_wb_bytes};
      std::memcpy(c->mstats + size_t(t) * 4, mv, sizeof mv);
    }
    if (c->sstats) {
      const CacheStats& q = core.stats();
      const uint64_t sv[5] = {q.score_fallbacks, q.scored_victims, q.score_layers, q.score_candidates,
                              q.score_saturated};
      std::memcpy(c->sstats + size_t(t) * 5, sv, sizeof sv);
    }
    if (c->qstats) {
      const CacheStats& q = core.stats();
      const uint64_t qv[4] = {q.disk_overlapped, q.disk_max_in_flight, q.disk_carried, q.disk_carried_bytes};
      std::memcpy(c->qstats + size_t(t) * 4, qv, sizeof qv);
    }
    if (c->pstats) {
      const CacheStats& q = core.stats();
      const uint64_t pv[5] = {q.clean_drops, q.clean_drop_bytes, q.pf_reverted, q.pf_revert_bytes, q.pf_strict_refused};
      std::memcpy(c->pstats + size_t(t) * 5, pv, sizeof pv);
    }
    if (c->kstats) {  // the pinned homes' order as FNV-1a 64 over each key's 4 little-endian bytes
      const CacheStats& q = core.stats();
      uint64_t h = 0xcbf29ce484222325ull;
      for (uint32_t k : core.host_order())
        for (int b = 0; b < 4; ++b) h = (h ^ ((k >> (8 * b)) & 0xffu)) * 0x100000001b3ull;
      const uint64_t kv[4] = {q.bank_kept, q.bank_keep_drops, q.bank_keep_rereads, h};
      std::memcpy(c->kstats + size_t(t) * 4, kv, sizeof kv);
    }
    if (c->lstats) {
      const CacheStats& q = core.stats();
      const uint64_t lv[9] = {q.landing_issued,  q.landing_promoted,    q.landing_late,
                              q.landing_expired, q.landing_dropped_full, q.landing_read_bytes,
                              q.landing_expired_layer, q.landing_skipped_passed, core.landing_units()};
      std::memcpy(c->lstats + size_t(t) * 9, lv, sizeof lv);
    }
    std::memcpy(tables + size_t(t) * keys, m.table_.data(), size_t(keys) * 4);
    const CacheStats& s = core.stats();
    const uint64_t v[16] = {s.tokens,        s.lookups,     s.misses,          s.covered,     s.fetched,
                            s.prefetched,    s.prefetch_used, s.resurrected,   s.bank_serves, s.collected_mid,
                            s.evicted,       s.evict_short, s.writebacks_done, s.wb_deferred, s.wb_cancelled,
                            s.wb_forced};
    std::memcpy(stats + size_t(t) * 16, v, sizeof v);
    if (c->xstats) {
      const uint64_t xv[6] = {s.disk_reads, s.disk_read_bytes, s.disk_stage_waits, s.disk_drops, s.disk_discards,
                              core.file_units()};
      std::memcpy(c->xstats + size_t(t) * 6, xv, sizeof xv);
    }
    core.check();
  }
}

}  // namespace tsb
