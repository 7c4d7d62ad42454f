// Reference harness for the host forward mode (TEST INFRASTRUCTURE): drives the reference library's own ss_* calls on
// its CPU backend through a forward per routes row, and reads which slot each unit's table entry points at from the
// reference context's internals (its layer pools and stream ring), so the product's tables can be compared unit for
// unit. The product library never links this file.
#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <deque>
#include <exception>
#include <list>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "backend.hpp"
#include "desc.hpp"
#include "errors.hpp"
#include "json.hpp"
#include "dg_layout.hpp"
#include "dg_ctx.hpp"
#include "plan.hpp"
#include "resident_set.hpp"
#include "source_file.hpp"
#include "strix_stream/ss.h"
#define private public
#include "stream_ctx.hpp"
#undef private
#include "oref.h"

// The reference's C ABI context (capi.cpp): a host-mode context or a device-gated one.
struct ss_ctx {
  std::unique_ptr<ts::Ctx> c;
  std::unique_ptr<ts::DgCtx> dg;
};

extern "C" __attribute__((visibility("default"))) int oref_host_replay(
    const char* desc_json, size_t len, const uint8_t* tiers, size_t n_tiers, const ss_budget* budget,
    const ss_options* opt_in, uint32_t forwards, const int32_t* routes, uint32_t n_ids, const uint8_t* all_layers,
    int32_t* locs, uint64_t* stats, uint64_t* xstats, const int32_t* pf_ids, uint32_t n_pf, int pf_mode, char* err,
    size_t errlen) {
  ss_desc* d = nullptr;
  ss_plan* p = nullptr;
  ss_ctx* c = nullptr;
  auto bad = [&](const char* what) {
    if (err && errlen) std::snprintf(err, errlen, "%s: %s", what, ss_last_error());
    if (c) ss_close(c);
    if (p) ss_plan_free(p);
    if (d) ss_desc_free(d);
    return -1;
  };
  if (ss_desc_from_json(desc_json, len, &d) != SS_OK) return bad("ss_desc_from_json");
  if (ss_plan_from_tiers(d, budget, tiers, n_tiers, &p) != SS_OK) return bad("ss_plan_from_tiers");
  ss_options o = *opt_in;
  o.struct_size = sizeof o;
  o.backend = SS_BACKEND_CPU;
  o.forward_mode = SS_FORWARD_HOST;
  if (ss_open(d, budget, p, &o, &c) != SS_OK) return bad("ss_open");
  const int L_n = ss_desc_n_layers(d);
  const int64_t total = ss_desc_total_units(d);
  std::vector<ss_layer_stats> before(static_cast<size_t>(L_n)), after(static_cast<size_t>(L_n));
  for (uint32_t f = 0; f < forwards; ++f) {
    for (int L = 0; L < L_n; ++L) ss_stats_layer(c, L, &before[size_t(L)]);
    // prefetch schedule (pf_mode 1 certain ids, 2 speculative ids, 3 whole layer): layer 0 before ss_begin, layer
    // L + 1 before the routes of layer L
    auto prefetch = [&](int L) -> bool {
      if (!pf_mode || L >= L_n || ss_desc_layer_units(d, L) <= 0) return true;
      if (pf_mode == 3) return ss_prefetch_layer(c, L) == SS_OK;
      const int32_t* p = pf_ids + (size_t(f) * size_t(L_n) + size_t(L)) * n_pf;
      return ss_prefetch(c, L, p, int(n_pf), pf_mode == 2 ? SS_PREFETCH_SPECULATIVE : SS_PREFETCH_CERTAIN) == SS_OK;
    };
    if (!prefetch(0)) return bad("ss_prefetch");
    if (ss_begin(c, nullptr, 0) != SS_OK) return bad("ss_begin");
    int32_t* out = locs + size_t(f) * size_t(total) * 2;
    for (int64_t k = 0; k < total * 2; ++k) out[k] = k % 2 ? -1 : 0;
    for (int L = 0; L < L_n; ++L) {
      const int units = ss_desc_layer_units(d, L);
      if (units <= 0) continue;
      if (!prefetch(L + 1)) return bad("ss_prefetch");
      const int32_t* r = routes + (size_t(f) * size_t(L_n) + size_t(L)) * n_ids;
      const ss_status st = all_layers[L] ? ss_layer_all(c, L) : ss_layer_routes(c, L, r, int(n_ids));
      if (st != SS_OK) return bad("routes");
      ss_layer_view v;
      if (ss_acquire(c, L, nullptr, &v) != SS_OK) return bad("ss_acquire");
      const auto& s = c->c->L_[size_t(L)];
      const int64_t base = ss_desc_unit_index(d, L, 0);
      for (int u = 0; u < units; ++u) {
        if (!v.table_host[u]) continue;
        const bool ring = s.loc[size_t(u)] == ts::Ctx::Ring;
        out[2 * (base + u)] = ring ? 2 : 1;
        out[2 * (base + u) + 1] = ring ? s.slot[size_t(u)] : s.rs->slot(u);
      }
      if (ss_release(c, L, nullptr) != SS_OK) return bad("ss_release");
    }
    if (ss_end(c) != SS_OK) return bad("ss_end");
    for (int L = 0; L < L_n; ++L) {
      ss_stats_layer(c, L, &after[size_t(L)]);
      uint64_t* o5 = stats + (size_t(f) * size_t(L_n) + size_t(L)) * 9;
      o5[0] = after[size_t(L)].routed - before[size_t(L)].routed;
      o5[1] = after[size_t(L)].hits - before[size_t(L)].hits;
      o5[2] = after[size_t(L)].admitted - before[size_t(L)].admitted;
      o5[3] = after[size_t(L)].transient - before[size_t(L)].transient;
      o5[4] = after[size_t(L)].evicted - before[size_t(L)].evicted;
      o5[5] = after[size_t(L)].prefetched - before[size_t(L)].prefetched;
      o5[6] = after[size_t(L)].spec_issued - before[size_t(L)].spec_issued;
      o5[7] = after[size_t(L)].spec_used - before[size_t(L)].spec_used;
      o5[8] = after[size_t(L)].spec_dropped - before[size_t(L)].spec_dropped;
    }
    if (xstats) {  // the exclusive counters after the forward (cumulative): writebacks .. discards
      ss_exclusive_stats x;
      if (ss_stats_exclusive_sized(c, &x, sizeof x) != SS_OK) return bad("ss_stats_exclusive");
      uint64_t* o8 = xstats + size_t(f) * 8;
      o8[0] = x.writebacks;
      o8[1] = x.writeback_bytes;
      o8[2] = x.deferred;
      o8[3] = x.promoted;
      o8[4] = x.free_blocks;
      o8[5] = x.min_free_blocks;
      o8[6] = x.rereads;
      o8[7] = x.discards;
    }
  }
  ss_close(c);
  ss_plan_free(p);
  ss_desc_free(d);
  return 0;
}

// The reference's own ResidentSet (resident_set.cpp) driven the way its host forward mode's ingest drives it
// (stream_ctx.cpp:1303-1354), for the resident-set parity test.
namespace {
void req(bool ok, const char* what) {
  if (!ok) throw std::runtime_error(what);
}
}  // namespace
extern "C" __attribute__((visibility("default"))) int oref_resident_replay(
    int32_t n_units, int32_t capacity, int32_t policy, uint32_t window, const int32_t* place_units,
    const uint8_t* place_pin, uint32_t n_place, uint32_t steps, const int32_t* routed, uint32_t k,
    const uint8_t* flags, const int32_t* max_ev, const uint8_t* admit_misses, int32_t* slots_out, int32_t* counts_out,
    char* err, size_t errlen) {
  using RS = ts::ResidentSet;

  try {
    req(n_units > 0 && capacity >= 0 && (policy == 0 || policy == 1) && (place_units || !n_place) &&
             (routed || !steps || !k) && flags && max_ev && admit_misses && slots_out && counts_out,
         "resident replay: bad argument");
    RS rs(n_units, capacity, policy == 1 ? SS_POLICY_SCORED : SS_POLICY_LRU, window);
    for (uint32_t i = 0; i < n_place; ++i) rs.place(place_units[i], place_pin && place_pin[i]);
    for (uint32_t t = 0; t < steps; ++t) {
      std::vector<char> count(size_t(n_units), 0), busy(size_t(n_units), 0);
      for (uint32_t i = 0; i < k; ++i) {
        const int32_t u = routed[size_t(t) * k + i];
        req(u < n_units, "resident replay: unit out of range");
        if (u >= 0) count[size_t(u)] = 1;
      }
      const uint8_t* f = flags + size_t(t) * size_t(n_units);
      std::vector<int32_t> routed_now, misses, to_admit;
      int hits = 0;
      for (int32_t u = 0; u < n_units; ++u) {  // the host forward mode's ingest order
        if (f[u] & 1) busy[size_t(u)] = 1;
        if (!count[size_t(u)]) continue;
        busy[size_t(u)] = 1;
        routed_now.push_back(u);
        if (f[u] & 2) {
          misses.push_back(u);
        } else if (rs.slot(u) >= 0) {
          ++hits;
        } else {
          to_admit.push_back(u);
          misses.push_back(u);
        }
      }
      const auto a = rs.admit(to_admit, busy, admit_misses[t] != 0, max_ev[t]);
      rs.observe(routed_now, misses);
      for (int32_t u = 0; u < n_units; ++u) slots_out[size_t(t) * size_t(n_units) + size_t(u)] = rs.slot(u);
      int32_t* c = counts_out + size_t(t) * 5;
      c[0] = hits;
      c[1] = int32_t(a.admitted.size());
      c[2] = int32_t(a.evicted.size());
      c[3] = int32_t(a.transient.size());
      c[4] = a.deferred;
    }
    return 0;
  } catch (const std::exception& e) {
    if (err && errlen) std::snprintf(err, errlen, "%s", e.what());
    return -1;
  }
}

// The reference's own device-gated layout (dg_layout.cpp) of a descriptor, tiers, budget and options: the same numbers
// as this library's layout hook, or its refusal (status and message).
extern "C" __attribute__((visibility("default"))) int oref_dg_layout(const char* desc_json, size_t len,
                                                                      const uint8_t* tiers, size_t n_tiers,
                                                                      const ss_budget* budget, const ss_options* opt,
                                                                      uint64_t* out, uint32_t n_out,
                                                                      uint32_t* residents, uint32_t cap, char* err,
                                                                      size_t errlen) {
  try {
    const ts::Desc d = ts::desc_from_json(ts::json_parse(std::string(desc_json, len)));
    const ts::Plan p = ts::plan_from_tiers(d, *budget, std::vector<uint8_t>(tiers, tiers + n_tiers));
    const ts::DgLayout x = ts::dg_layout(d, p, *opt);
    const uint64_t v[27] = {x.keys, x.R, x.D, x.B, x.P, x.Q, x.I, x.F, x.S, x.disk_queue, x.blocks,
                            x.persistent_slots, x.slots, x.guard_slot, x.unit_bytes, x.host_stride, x.disk_tier,
                            x.disk_prefetch, x.scored, x.w_trans, x.w_freq, x.w_rec, x.residents.size(),
                            x.L, x.landing_queued, x.landing_ttl, x.landing_chunk};
    for (uint32_t i = 0; i < n_out && i < 27; ++i) out[i] = v[i];
    for (uint32_t i = 0; i < cap && i < x.residents.size(); ++i) residents[i] = x.residents[i];
    return 0;
  } catch (const ts::Error& e) {
    if (err && errlen) std::snprintf(err, errlen, "%s", e.what());
    return int(e.status());
  } catch (const std::exception& e) {
    if (err && errlen) std::snprintf(err, errlen, "%s", e.what());
    return -1;
  }
}

// The reference's own descriptor parser and planner through its C ABI (capi.cpp): the descriptor (status, its JSON, every
// layer's units and unit bytes), then a plan made from a budget and benefits (mode 0, ss_plan_make), given tiers (mode
// 1, ss_plan_from_tiers) or a plan JSON passed as the tiers' bytes (mode 2, ss_plan_from_json): every unit's tier, the
// totals and the plan's JSON. Returns the plan's status (or the
// descriptor's when that failed, with *desc_status set).
extern "C" __attribute__((visibility("default"))) int oref_plan(
    const char* desc_json, size_t len, const ss_budget* budget, const double* benefit, size_t n_benefit,
    const uint8_t* tiers, size_t n_tiers, int mode, uint8_t* tiers_out, size_t cap, ss_plan_totals* totals,
    char* json_out, size_t json_cap, char* desc_out, size_t desc_cap, uint64_t* layer_out, size_t layer_cap,
    int* desc_status, char* err, size_t errlen) {
  ss_desc* d = nullptr;
  *desc_status = ss_desc_from_json(desc_json, len, &d);
  if (*desc_status != SS_OK) {
    if (err && errlen) std::snprintf(err, errlen, "%s", ss_last_error());
    return *desc_status;
  }
  void* text = nullptr;
  size_t n = 0;
  if (ss_desc_to_json(d, reinterpret_cast<char**>(&text), &n) == SS_OK) {
    std::snprintf(desc_out, desc_cap, "%.*s", int(n), static_cast<const char*>(text));
    ss_free(text);
  }
  const int L = ss_desc_n_layers(d);
  for (int l = 0; l < L && size_t(2 * l + 1) < layer_cap; ++l) {
    layer_out[2 * l] = uint64_t(ss_desc_layer_units(d, l));
    layer_out[2 * l + 1] = ss_desc_unit_bytes(d, l);
  }
  ss_plan* p = nullptr;
  const ss_status st =
      mode == 0   ? ss_plan_make(d, budget, benefit, n_benefit, &p)
      : mode == 1 ? ss_plan_from_tiers(d, budget, tiers, n_tiers, &p)
                  : ss_plan_from_json(d, budget, reinterpret_cast<const char*>(tiers), n_tiers, &p);  // (tiers: JSON)
  if (st != SS_OK) {
    if (err && errlen) std::snprintf(err, errlen, "%s", ss_last_error());
    ss_desc_free(d);
    return st;
  }
  size_t at = 0;
  for (int l = 0; l < L; ++l)
    for (int u = 0; u < ss_desc_layer_units(d, l) && at < cap; ++u) tiers_out[at++] = uint8_t(ss_plan_unit_tier(p, l, u));
  ss_plan_get_totals(p, totals);
  if (ss_plan_to_json(p, reinterpret_cast<char**>(&text), &n) == SS_OK) {
    std::snprintf(json_out, json_cap, "%.*s", int(n), static_cast<const char*>(text));
    ss_free(text);
  }
  ss_plan_free(p);
  ss_desc_free(d);
  return SS_OK;
}

// The reference's defaults for the versioned structs (capi.cpp): ss_options_defaults_sized and
// ss_budget_defaults_sized into caller buffers of the given sizes.
extern "C" __attribute__((visibility("default"))) void oref_defaults(void* options, uint32_t options_size, void* budget,
                                                                     uint32_t budget_size) {
  ss_options_defaults_sized(static_cast<ss_options*>(options), options_size);
  ss_budget_defaults_sized(static_cast<ss_budget*>(budget), budget_size);
}
