// The C ABI (include/strix_stream/ss.h): every entry point catches, maps to ss_status and keeps the message per
// thread; a device or allocation failure inside a context call poisons the context (the reference's rules,
// capi.cpp:52-66 and 482-510 there). Functions outside this build's scope return SS_E_UNSUPPORTED.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <new>
#include <sstream>

#include "ctx.hpp"
#include "desc.hpp"
#include "errors.hpp"
#include "json.hpp"
#include "peer.hpp"
#include "plan.hpp"
#include "read_depth.hpp"

namespace tsb {
void check_read_pool();  // read_pool_check.cpp
}
#include "resident_set.hpp"
#include "score_profile.hpp"
#include "strix_stream/ss.h"
#include "strix_stream/ss_test.h"
#include "tierstream/tsb.h"

struct ss_desc {
  tsb::Desc d;
};
struct ss_plan {
  tsb::Plan p;
  const ss_desc* desc;
};
struct ss_ctx {
  std::unique_ptr<tsb::HostContext> host;
  std::unique_ptr<tsb::DgContext> dg;
};

namespace {

thread_local std::string g_err;

// Records `text` as this thread's last error and returns `st`.
ss_status refuse(ss_status st, std::string text) {
  g_err = std::move(text);
  return st;
}

// Inside a catch block: the status the exception in flight maps to (a library error keeps its own; running out of
// host memory is SS_E_NOMEM; anything else is an internal failure, SS_E_BACKEND), with its text kept as the last
// error. `harmful` is set when a context that was running the call can no longer be trusted: every failure except a
// library error other than SS_E_BACKEND / SS_E_NOMEM (bad arguments, IO, hash, capacity leave it consistent).
ss_status caught(bool* harmful, const char* oom_text = "out of host memory") {
  ss_status st = SS_E_BACKEND;
  try {
    throw;
  } catch (const tsb::Error& e) {
    g_err = e.what();
    st = e.status();
    *harmful = st == SS_E_BACKEND || st == SS_E_NOMEM;
    return st;
  } catch (const std::bad_alloc&) {
    g_err = oom_text;
    st = SS_E_NOMEM;
  } catch (const std::exception& e) {
    g_err = e.what();
  } catch (...) {
    g_err = "internal failure";
  }
  *harmful = true;
  return st;
}

// A call outside any context: every exception becomes its status.
template <class F>
ss_status guard(F&& f) {
  try {
    f();
  } catch (...) {
    bool harmful = false;
    return caught(&harmful);
  }
  return SS_OK;
}

// Hands `s` to the caller as a malloc'd, NUL-terminated copy (freed with ss_free), its length in *len.
ss_status give_text(const std::string& s, char** out, size_t* len) {
  if (!out) return refuse(SS_E_INVALID, "null output pointer");
  char* copy = static_cast<char*>(std::malloc(s.size() + 1));
  if (!copy) return refuse(SS_E_NOMEM, "out of host memory");
  std::memcpy(copy, s.c_str(), s.size() + 1);  // with the terminator
  *out = copy;
  if (len) *len = s.size();
  return SS_OK;
}

void need(bool ok, const char* what) { tsb::require(ok, SS_E_INVALID, what); }

ss_status unsupported(const char* fn) {
  g_err = std::string(fn) + ": not in this build (the tierstream B200 runtime implements the weight-streaming hot "
                            "path only)";
  return SS_E_UNSUPPORTED;
}

void budget_defaults(ss_budget* b) {
  std::memset(b, 0, sizeof *b);
  b->struct_size = uint32_t(sizeof *b);
  b->margin_gib = 2.0;
  b->margin_fraction = 0.03;
}

void options_defaults(ss_options* o) {
  std::memset(o, 0, sizeof *o);
  o->struct_size = uint32_t(sizeof *o);
  o->backend = SS_BACKEND_CUDA;  // the only backend of this build (the reference defaults to its CPU backend)
  o->policy = SS_POLICY_LRU;
  o->lookahead_budget = 2;
  o->reader_threads = 2;
  o->staging_buffers = 4;
  o->staging_bytes = uint64_t(256) << 20;
  o->copy_piece_bytes = uint64_t(64) << 20;
  o->fill_residents = 1;
  o->score_window = 16;
  o->pin_planned = 1;
  o->direct_io = 1;
  o->forward_mode = SS_FORWARD_HOST;
  o->dg_prefetch_reserve = 0xFFFFFFFFu;
  o->dg_prefetch_per_layer = 4;
  o->dg_prefetch_per_token = 48;
  o->dg_wait_timeout_ms = 10000;
  o->dg_spare_target = 0xFFFFFFFFu;
  o->dg_wb_defer = 1;
  o->dg_wb_stream = 1;
  o->dg_score_w_trans = 700;
  o->dg_score_w_freq = 200;
  o->dg_score_w_recency = 100;
  o->drive_readers = 4;
}

// Fills the first `size` bytes of *out with the defaults (struct_size = size).
template <class T, class F>
void sized_defaults(T* out, uint32_t size, F defaults) {
  if (!out || size < sizeof(uint32_t)) return;
  T full;
  defaults(&full);
  const size_t n = size < sizeof full ? size : sizeof full;
  std::memcpy(out, &full, n);
  out->struct_size = size;
}

// A versioned input struct: min(struct_size, own) bytes from the caller, the defaults for the rest.
template <class T, class F>
T versioned(const T* in, F defaults, const char* what) {
  T v;
  defaults(&v);
  if (!in) return v;
  tsb::require(in->struct_size >= sizeof(uint32_t), SS_E_INVALID, std::string(what) + ": struct_size not set");
  const size_t n = in->struct_size < sizeof v ? in->struct_size : sizeof v;
  std::memcpy(&v, in, n);
  v.struct_size = uint32_t(sizeof v);
  return v;
}

// A versioned output: the caller's size, at most ours.
template <class T>
void give_sized(T* out, uint32_t size, const T& full) {
  const size_t n = size < sizeof full ? size : sizeof full;
  std::memcpy(out, &full, n);
  out->struct_size = uint32_t(n);
}

std::string read_text(const char* path) {
  std::ifstream f(path, std::ios::binary);
  tsb::require(bool(f), SS_E_IO, std::string("cannot open ") + path);
  std::stringstream s;
  s << f.rdbuf();
  return s.str();
}

bool ctx_poisoned(const ss_ctx* c) { return c->dg ? c->dg->poisoned() : c->host->poisoned(); }
void ctx_poison(ss_ctx* c) {
  if (c->dg) c->dg->poison();
  else c->host->poison();
}
tsb::HostContext& host_of(const ss_ctx* c, const char* fn) {
  if (c->dg) tsb::fail(SS_E_INVALID, std::string(fn) + ": refused in device-gated mode");
  return *c->host;
}
tsb::DgContext& dg_of(const ss_ctx* c, const char* fn) {
  if (!c->dg) tsb::fail(SS_E_INVALID, std::string(fn) + ": the context is not device-gated");
  return *c->dg;
}

// A context call: a poisoned context refuses it; a failure that leaves the context untrustworthy (`caught`) poisons
// the context, so every later call is refused until it is closed. The calls run with the context's device current.
template <class F>
ss_status ctx_guard(ss_ctx* c, F&& f) {
  if (!c) return refuse(SS_E_INVALID, "null context");
  if (ctx_poisoned(c))
    return refuse(SS_E_BACKEND, "context poisoned by an earlier device, out-of-memory or internal failure: close it");
  try {
    tsb::DeviceScope on(c->dg ? c->dg->device() : c->host->device());
    f();
  } catch (...) {
    bool harmful = false;
    const ss_status st = caught(&harmful, "out of host memory (context poisoned)");
    if (harmful) ctx_poison(c);
    return st;
  }
  return SS_OK;
}

}  // namespace

namespace tsb {
const char* set_error(const std::string& msg) {
  g_err = msg;
  return g_err.c_str();
}
}  // namespace tsb

extern "C" {

const char* ss_last_error(void) { return g_err.c_str(); }
int ss_abi_version(void) { return SS_ABI_VERSION; }

// ---- descriptor ----
ss_status ss_desc_from_json(const char* json_text, size_t len, ss_desc** out) {
  return guard([&] {
    need(json_text && out, "ss_desc_from_json: null argument");
    *out = new ss_desc{tsb::desc_from_json(tsb::json_parse(std::string(json_text, len)))};
  });
}
ss_status ss_desc_from_file(const char* path, ss_desc** out) {
  return guard([&] {
    need(path && out, "ss_desc_from_file: null argument");
    *out = new ss_desc{tsb::desc_from_json(tsb::json_parse(read_text(path)))};
  });
}
ss_status ss_desc_from_model(const char* manifest_path, ss_desc** out) { return ss_desc_from_file(manifest_path, out); }
void ss_desc_free(ss_desc* d) { delete d; }
int ss_desc_n_layers(const ss_desc* d) { return d ? int(d->d.layers.size()) : -1; }
int ss_desc_layer_units(const ss_desc* d, int layer) {
  if (!d || layer < 0 || size_t(layer) >= d->d.layers.size()) return -1;
  return d->d.layers[size_t(layer)].n_units;
}
uint64_t ss_desc_unit_bytes(const ss_desc* d, int layer) {
  if (!d || layer < 0 || size_t(layer) >= d->d.layers.size()) return 0;
  return d->d.layers[size_t(layer)].unit_bytes;
}
ss_status ss_desc_to_json(const ss_desc* d, char** out_json, size_t* out_len) {
  std::string s;
  const ss_status st = guard([&] {
    need(d != nullptr, "ss_desc_to_json: null descriptor");
    s = tsb::json_write(tsb::desc_to_json(d->d));
  });
  return st != SS_OK ? st : give_text(s, out_json, out_len);
}
void ss_free(void* p) { std::free(p); }
int64_t ss_desc_unit_index(const ss_desc* d, int layer, int unit) {
  if (!d || layer < 0 || size_t(layer) >= d->d.layers.size()) return -1;
  if (unit < 0 || unit >= d->d.layers[size_t(layer)].n_units) return -1;
  return d->d.unit_base[size_t(layer)] + unit;
}
int64_t ss_desc_total_units(const ss_desc* d) { return d ? d->d.total_units : -1; }

// ---- planner ----
void ss_budget_defaults_sized(ss_budget* b, uint32_t size) { sized_defaults(b, size, budget_defaults); }
ss_status ss_plan_make(const ss_desc* d, const ss_budget* b, const double* benefit, size_t n_benefit, ss_plan** out) {
  return guard([&] {
    need(d && b && out, "ss_plan_make: null argument");
    need(!n_benefit || benefit, "ss_plan_make: null benefit");
    ss_budget bb = versioned(b, budget_defaults, "ss_plan_make budget");
    bb.reserved0 = 0;
    std::vector<double> ben(benefit, benefit + n_benefit);
    *out = new ss_plan{tsb::plan_make(d->d, bb, ben), d};
  });
}
ss_status ss_plan_from_tiers(const ss_desc* d, const ss_budget* b, const uint8_t* tiers, size_t n, ss_plan** out) {
  return guard([&] {
    need(d && b && out && (tiers || !n), "ss_plan_from_tiers: null argument");
    ss_budget bb = versioned(b, budget_defaults, "ss_plan_from_tiers budget");
    bb.reserved0 = 0;
    *out = new ss_plan{tsb::plan_from_tiers(d->d, bb, std::vector<uint8_t>(tiers, tiers + n)), d};
  });
}
ss_status ss_plan_from_json(const ss_desc* d, const ss_budget* b, const char* plan_json, size_t len, ss_plan** out) {
  return guard([&] {
    need(d && b && plan_json && out, "ss_plan_from_json: null argument");
    ss_budget bb = versioned(b, budget_defaults, "ss_plan_from_json budget");
    bb.reserved0 = 0;
    const tsb::Json j = tsb::json_parse(std::string(plan_json, len));
    *out = new ss_plan{tsb::plan_from_tiers(d->d, bb, tsb::tiers_from_json(d->d, j)), d};
  });
}
void ss_plan_free(ss_plan* p) { delete p; }
ss_tier ss_plan_unit_tier(const ss_plan* p, int layer, int unit) {
  const int64_t g = p ? ss_desc_unit_index(p->desc, layer, unit) : -1;
  return g < 0 ? SS_TIER_DISK : ss_tier(p->p.tier[size_t(g)]);
}
void ss_plan_get_totals(const ss_plan* p, ss_plan_totals* out) {
  if (!p || !out) return;
  out->fixed_bytes = p->p.fixed;
  out->margin_bytes = p->p.margin;
  out->resident_bytes = p->p.resident;
  out->dynamic_bytes = p->p.dynamic;
  out->ring_bytes = p->p.ring;
  out->peak_device_bytes = p->p.peak;
  out->pinned_bytes = p->p.pinned;
  out->disk_bytes = p->p.disk;
  out->n_resident = p->p.n_resident;
  out->n_pinned = p->p.n_pinned;
  out->n_disk = p->p.n_disk;
}
ss_status ss_plan_to_json(const ss_plan* p, char** out_json, size_t* out_len) {
  std::string s;
  const ss_status st = guard([&] {
    need(p != nullptr, "ss_plan_to_json: null plan");
    s = tsb::json_write(tsb::plan_to_json(p->desc->d, p->p));
  });
  return st != SS_OK ? st : give_text(s, out_json, out_len);
}

// ---- context ----
void ss_options_defaults_sized(ss_options* o, uint32_t size) { sized_defaults(o, size, options_defaults); }

namespace {
ss_status open_impl(const ss_desc* d, const ss_budget* budget, const ss_plan* plan, const ss_options* opt,
                    const tsb::PeerTier* peer, ss_ctx** out) {
  return guard([&] {
    need(d && budget && out, "ss_open: null argument");
    need(!plan || plan->desc == d, "ss_open: plan was made from another descriptor");
    ss_options o = versioned(opt, options_defaults, "ss_open options");
    for (uint32_t* r : {&o.reserved0, &o.reserved1, &o.reserved2, &o.reserved3, &o.reserved4, &o.reserved5,
                        &o.reserved6, &o.reserved7, &o.reserved8, &o.reserved9, &o.reserved10, &o.reserved11,
                        &o.reserved12, &o.reserved13})
      *r = 0;
    tsb::require(o.backend == SS_BACKEND_CUDA, SS_E_UNSUPPORTED,
                 "ss_open: this build has only the CUDA backend (ss_options.backend = SS_BACKEND_CUDA); the CPU and "
                 "HIP backends are not built");
    need(!o.weight_dirs || !o.weight_dirs[0], "ss_open: weight_dirs (multi-location files) is not in this build");
    need(!o.budget, "ss_open: whole-device budget ledgers are not in this build");
    need(!o.source_identity_n, "ss_open: source identities are not in this build");
    ss_budget bb = versioned(budget, budget_defaults, "ss_open budget");
    bb.reserved0 = 0;
    need(!plan || tsb::same_budget(plan->p.budget, bb), "ss_open: the plan was made with another budget");
    const tsb::Plan p = plan ? plan->p : tsb::plan_make(d->d, bb, {});
    need(o.forward_mode == SS_FORWARD_HOST || o.forward_mode == SS_FORWARD_DEVICE_GATED, "ss_open: unknown forward_mode");
    tsb::DeviceScope on(o.device);  // the open runs on the context's device; the caller's comes back after
    if (o.forward_mode == SS_FORWARD_DEVICE_GATED) {
      auto dg = tsb::open_dg_context(d->d, p, o, peer);
      *out = new ss_ctx{nullptr, std::move(dg)};
    } else {
      need(!peer, "tsb_open_peer: the peer tier serves device-gated decode only (forward_mode DEVICE_GATED)");
      need(o.policy != SS_POLICY_SCORED_AUTO, "ss_open: SCORED_AUTO needs device-gated mode");
      need(o.policy == SS_POLICY_LRU || o.policy == SS_POLICY_SCORED, "ss_open: policy must be LRU or SCORED");
      auto h = tsb::open_host_context(d->d, bb, p, o);
      *out = new ss_ctx{std::move(h), nullptr};
    }
  });
}
}  // namespace

ss_status ss_open(const ss_desc* d, const ss_budget* budget, const ss_plan* plan, const ss_options* opt, ss_ctx** out) {
  return open_impl(d, budget, plan, opt, nullptr, out);
}
void ss_close(ss_ctx* c) {
  if (!c) return;
  tsb::DeviceScope on(c->dg ? c->dg->device() : c->host->device());
  delete c;
}
int ss_source_direct(const ss_ctx* c, int source) {
  if (!c) return -1;
  if (c->dg) return source < 0 || source >= c->dg->n_sources() ? -1 : c->dg->source_direct(source) ? 1 : 0;
  return source < 0 || source >= c->host->n_sources() ? -1 : c->host->source_direct(source) ? 1 : 0;
}

ss_status ss_seed(ss_ctx* c, int layer, const int32_t* units, int n) {
  return ctx_guard(c, [&] {
    if (c->dg) c->dg->seed(layer, units, n);
    else c->host->seed(layer, units, n);
  });
}
ss_status ss_begin(ss_ctx* c, const uint32_t* rows, int n_layers) {
  return ctx_guard(c, [&] {
    if (c->dg) c->dg->begin(rows, n_layers);
    else c->host->begin(rows, n_layers);
  });
}
ss_status ss_layer_routes(ss_ctx* c, int layer, const int32_t* ids, int n) {
  return ctx_guard(c, [&] { host_of(c, "ss_layer_routes").routes(layer, ids, n); });
}
ss_status ss_layer_routes_dev(ss_ctx* c, int layer, const int32_t* ids_dev, int n, void* s) {
  return ctx_guard(c, [&] { host_of(c, "ss_layer_routes_dev").routes_dev(layer, ids_dev, n, s); });
}
ss_status ss_layer_all(ss_ctx* c, int layer) {
  return ctx_guard(c, [&] { host_of(c, "ss_layer_all").routes_all(layer); });
}
ss_status ss_prefetch(ss_ctx* c, int layer, const int32_t* ids, int n, ss_prefetch_kind kind) {
  return ctx_guard(c, [&] {
    need(n >= 0 && (ids || n == 0), "ss_prefetch: bad ids");
    need(kind == SS_PREFETCH_CERTAIN || kind == SS_PREFETCH_SPECULATIVE, "ss_prefetch: unknown kind");
    host_of(c, "ss_prefetch").prefetch(layer, ids, n, kind == SS_PREFETCH_SPECULATIVE);
  });
}
ss_status ss_prefetch_layer(ss_ctx* c, int layer) {
  return ctx_guard(c, [&] {
    tsb::HostContext& h = host_of(c, "ss_prefetch_layer");
    h.prefetch(layer, nullptr, -1, false);  // n < 0: every unit of the layer
  });
}
// Host read-ahead requests (stream_ctx.cpp:1441-1449): a no-op for a context without read-ahead buffers.
ss_status ss_host_prefetch(ss_ctx* c, int layer, const int32_t* ids, int n) {
  return ctx_guard(c, [&] {
    need(n >= 0 && (ids || n == 0), "ss_host_prefetch: bad ids");
    host_of(c, "ss_host_prefetch").host_prefetch(layer, ids, n);
  });
}
ss_status ss_host_prefetch_layer(ss_ctx* c, int layer) {
  return ctx_guard(c, [&] { host_of(c, "ss_host_prefetch_layer").host_prefetch(layer, nullptr, -1); });
}
ss_status ss_acquire(ss_ctx* c, int layer, void* s, ss_layer_view* out) {
  return ctx_guard(c, [&] {
    need(out != nullptr, "ss_acquire: null view");
    host_of(c, "ss_acquire").acquire(layer, s, true, out);
  });
}
ss_status ss_acquire_groups(ss_ctx* c, int layer, void* s, ss_layer_view* out) {
  return ctx_guard(c, [&] {
    need(out != nullptr, "ss_acquire_groups: null view");
    host_of(c, "ss_acquire_groups").acquire(layer, s, false, out);
  });
}
ss_status ss_group_wait(ss_ctx* c, int layer, int group, void* s) {
  return ctx_guard(c, [&] { host_of(c, "ss_group_wait").group_wait(layer, group, s); });
}
ss_status ss_release(ss_ctx* c, int layer, void* s) {
  return ctx_guard(c, [&] { host_of(c, "ss_release").release(layer, s); });
}
ss_status ss_end(ss_ctx* c) {
  return ctx_guard(c, [&] {
    if (c->dg) c->dg->end(1);
    else c->host->end();
  });
}
ss_status ss_check_unit(ss_ctx* c, int layer, int unit) {
  return ctx_guard(c, [&] {
    if (c->dg) c->dg->check_unit(layer, unit);
    else c->host->check_unit(layer, unit);
  });
}

ss_status ss_lookahead_select(const float* scores, int rows, int n_experts, int top_k, int32_t* out, int max_out,
                              int* n_out) {
  return guard([&] {
    need(scores && out && n_out && rows >= 0 && n_experts > 0 && top_k > 0 && top_k <= n_experts && max_out >= 0,
         "ss_lookahead_select: bad argument");
    // per row its top_k by (score desc, id asc); the union ordered by (best rank, best score, id)
    std::vector<int> rank(size_t(n_experts), top_k);
    std::vector<float> best(size_t(n_experts), 0.0f);
    std::vector<int> idx(static_cast<size_t>(n_experts), 0);
    for (int r = 0; r < rows; ++r) {
      const float* s = scores + size_t(r) * size_t(n_experts);
      for (int e = 0; e < n_experts; ++e) idx[size_t(e)] = e;
      std::partial_sort(idx.begin(), idx.begin() + top_k, idx.end(),
                        [&](int a, int b) { return s[a] != s[b] ? s[a] > s[b] : a < b; });
      for (int k = 0; k < top_k; ++k) {
        const int e = idx[size_t(k)];
        if (k < rank[size_t(e)] || (k == rank[size_t(e)] && s[e] > best[size_t(e)])) {
          rank[size_t(e)] = k;
          best[size_t(e)] = s[e];
        }
      }
    }
    std::vector<int> u;
    for (int e = 0; e < n_experts; ++e)
      if (rank[size_t(e)] < top_k) u.push_back(e);
    std::sort(u.begin(), u.end(), [&](int a, int b) {
      if (rank[size_t(a)] != rank[size_t(b)]) return rank[size_t(a)] < rank[size_t(b)];
      if (best[size_t(a)] != best[size_t(b)]) return best[size_t(a)] > best[size_t(b)];
      return a < b;
    });
    const int n = std::min(int(u.size()), max_out);
    for (int i = 0; i < n; ++i) out[i] = u[size_t(i)];
    *n_out = n;
  });
}

// ---- stats ----
ss_status ss_stats_layer(const ss_ctx* c, int layer, ss_layer_stats* out) {
  return guard([&] {
    need(c && out, "ss_stats_layer: bad argument");
    if (c->dg) c->dg->layer_stats(layer, out);
    else c->host->layer_stats(layer, out);
  });
}
ss_status ss_stats_total(const ss_ctx* c, ss_layer_stats* out) {
  return guard([&] {
    need(c && out, "ss_stats_total: bad argument");
    if (c->dg) c->dg->total_stats(out);
    else c->host->total_stats(out);
  });
}
void ss_stats_reset(ss_ctx* c) {
  if (!c) return;
  (void)guard([&] {
    if (c->dg) c->dg->reset_stats();
    else c->host->reset_stats();
  });
}
void ss_set_stats_hook(ss_ctx* c, ss_stats_hook hook, void* user) {
  if (c && c->host) c->host->set_hook(hook, user);
}
ss_status ss_stats_to_json(const ss_ctx* c, char** out_json, size_t* out_len) {
  std::string s;
  const ss_status st = guard([&] {
    need(c != nullptr, "ss_stats_to_json: null context");
    s = c->dg ? c->dg->stats_json() : c->host->stats_json();
  });
  return st != SS_OK ? st : give_text(s, out_json, out_len);
}
ss_status ss_stats_exclusive_sized(const ss_ctx* c, ss_exclusive_stats* out, uint32_t size) {
  return guard([&] {
    need(c && out && size >= 4, "ss_stats_exclusive: bad argument");
    ss_exclusive_stats s{};
    if (c->dg) c->dg->exclusive_stats(&s);
    else c->host->exclusive_stats(&s);
    give_sized(out, size, s);
  });
}
ss_status ss_stats_snapshot_sized(const ss_ctx*, ss_layer_stats*, ss_snapshot_info*, uint32_t) {
  return unsupported("ss_stats_snapshot");
}
ss_status ss_stats_snapshot_json(const ss_ctx*, char**, size_t*) { return unsupported("ss_stats_snapshot_json"); }

// ---- device-gated ----
ss_status ss_dg_get_device_view_sized(const ss_ctx* c, ss_dg_device_view* out, uint32_t size) {
  return guard([&] {
    need(c && out && size >= 4, "ss_dg_get_device_view: bad argument");
    ss_dg_device_view v;
    dg_of(c, "ss_dg_get_device_view").device_view(&v);
    const size_t n = size < sizeof v ? size : sizeof v;
    std::memcpy(out, &v, n);
    out->struct_size = uint32_t(n);
  });
}
int ss_dg_gated_index(const ss_ctx* c, int layer) { return c && c->dg ? c->dg->gated_index(layer) : -1; }
ss_status ss_dg_enqueue_begin(ss_ctx* c, void* stream) {
  return ctx_guard(c, [&] { dg_of(c, "ss_dg_enqueue_begin").enqueue_begin(stream); });
}
ss_status ss_dg_enqueue_export(ss_ctx* c, int g, const int32_t* ids_dev, int n, int n_pred, void* stream) {
  return ctx_guard(c, [&] { dg_of(c, "ss_dg_enqueue_export").enqueue_export(g, ids_dev, n, n_pred, stream); });
}
ss_status ss_dg_enqueue_predict(ss_ctx* c, int g, const int32_t* ids_dev, int n, void* stream) {
  return ctx_guard(c, [&] { dg_of(c, "ss_dg_enqueue_predict").enqueue_predict(g, ids_dev, n, stream); });
}
ss_status ss_dg_enqueue_wait(ss_ctx* c, int g, void* stream) {
  return ctx_guard(c, [&] { dg_of(c, "ss_dg_enqueue_wait").enqueue_wait(g, stream); });
}
ss_status ss_dg_enqueue_end(ss_ctx* c, void* stream) {
  return ctx_guard(c, [&] { dg_of(c, "ss_dg_enqueue_end").enqueue_end(stream); });
}
ss_status ss_dg_keep(ss_ctx* c, int g, const int32_t* ids, int n) {
  return ctx_guard(c, [&] { dg_of(c, "ss_dg_keep").keep(g, ids, n); });
}
ss_status ss_dg_residency(ss_ctx* c, ss_dg_unit* out, uint32_t cap, uint32_t* total) {
  return ctx_guard(c, [&] {
    need((out || !cap) && total, "ss_dg_residency: bad argument");
    *total = dg_of(c, "ss_dg_residency").residency(out, cap);
  });
}
ss_status ss_dg_set_sched(ss_ctx* c, uint32_t wb_defer, uint32_t flush_ready) {
  return ctx_guard(c, [&] { dg_of(c, "ss_dg_set_sched").set_sched(wb_defer, flush_ready); });
}
ss_status ss_dg_set_budgets(ss_ctx* c, uint32_t spare_target, uint32_t per_layer, uint32_t per_token) {
  return ctx_guard(c, [&] { dg_of(c, "ss_dg_set_budgets").set_budgets(spare_target, per_layer, per_token); });
}
ss_status ss_dg_timeline_sized(const ss_ctx* c, int g, ss_dg_layer_timeline* out, uint32_t size) {
  return guard([&] {
    need(c && out && size >= 4, "ss_dg_timeline: bad argument");
    ss_dg_layer_timeline t;
    dg_of(c, "ss_dg_timeline").timeline(g, &t);
    give_sized(out, size, t);
  });
}
ss_status ss_dg_boundary_timeline_sized(const ss_ctx* c, ss_dg_boundary_timeline* out, uint32_t size) {
  return guard([&] {
    need(c && out && size >= 4, "ss_dg_boundary_timeline: bad argument");
    ss_dg_boundary_timeline t;
    dg_of(c, "ss_dg_boundary_timeline").boundary_timeline(&t);
    give_sized(out, size, t);
  });
}
ss_status ss_stats_dg_sized(const ss_ctx* c, ss_dg_stats* out, uint32_t size) {
  return guard([&] {
    need(c && out && size >= 4, "ss_stats_dg: bad argument");
    ss_dg_stats s;
    dg_of(c, "ss_stats_dg").stats(&s);
    give_sized(out, size, s);
  });
}
ss_status ss_dg_reset_open(ss_ctx* c) {
  return ctx_guard(c, [&] { dg_of(c, "ss_dg_reset_open").reset_open(); });
}
ss_status ss_dg_end_rows(ss_ctx* c, uint32_t rows) {
  return ctx_guard(c, [&] {
    need(rows > 0, "ss_dg_end_rows: rows must be positive");
    dg_of(c, "ss_dg_end_rows").end(rows);
  });
}
ss_status ss_dg_set_policy(ss_ctx* c, ss_policy policy) {
  return ctx_guard(c, [&] {
    dg_of(c, "ss_dg_set_policy").set_policy(uint32_t(policy));
  });
}

// ---- test hooks ----
ss_status ss_test_dg_mutate(ss_ctx* c, int m) { return ctx_guard(c, [&] { dg_of(c, "ss_test_dg_mutate").test_mutate(m); }); }
ss_status ss_test_dg_pressure(ss_ctx* c, uint32_t f, uint32_t r) {
  return ctx_guard(c, [&] { dg_of(c, "ss_test_dg_pressure").test_pressure(f, r); });
}
ss_status ss_test_dg_check(ss_ctx* c) {
  if (!c) return SS_E_INVALID;
  return guard([&] { dg_of(c, "ss_test_dg_check").test_check(); });
}
ss_status ss_test_dg_gate(ss_ctx* c, int stream, void* event) {
  return ctx_guard(c, [&] { dg_of(c, "ss_test_dg_gate").test_gate(stream, event); });
}
ss_status ss_test_dg_flags(ss_ctx* c, uint32_t flags) {
  return ctx_guard(c, [&] { dg_of(c, "ss_test_dg_flags").test_flags(flags); });
}
ss_status ss_test_dg_coming(ss_ctx* c, uint32_t* out) {
  return ctx_guard(c, [&] {
    need(out != nullptr, "ss_test_dg_coming: null output");
    *out = dg_of(c, "ss_test_dg_coming").test_coming();
  });
}
ss_status ss_test_dg_stop_service(ss_ctx* c) {
  return ctx_guard(c, [&] { dg_of(c, "ss_test_dg_stop_service").test_stop_service(); });
}

ss_status tsb_test_dg_table(ss_ctx* c, int32_t* out, uint32_t cap) {
  if (!c) return SS_E_INVALID;
  return guard([&] { dg_of(c, "tsb_test_dg_table").test_table(out, cap); });
}

ss_status tsb_test_dg_corrupt(ss_ctx* c, int layer, int unit, uint64_t offset) {
  if (!c) return SS_E_INVALID;
  return guard([&] { dg_of(c, "tsb_test_dg_corrupt").test_corrupt(layer, unit, offset); });
}

ss_status tsb_test_host_locs(ss_ctx* c, int layer, int32_t* out, int n) {
  if (!c || !out) return SS_E_INVALID;
  return guard([&] { host_of(c, "tsb_test_host_locs").test_locs(layer, out, n); });
}

ss_status tsb_test_host_unit(ss_ctx* c, int layer, int unit, void** pinned, void** device) {
  if (!c || !pinned || !device) return SS_E_INVALID;
  return guard([&] { host_of(c, "tsb_test_host_unit").test_unit(layer, unit, pinned, device); });
}

// ---- peer tier (tsb.h) ----
struct tsb_peer_store {
  std::unique_ptr<tsb::PeerStore> s;
};

ss_status tsb_peer_plan(const uint64_t* counts, uint32_t keys, uint32_t world, const uint64_t* cap_units,
                        int32_t* owner) {
  return guard([&] {
    need(owner || !keys, "tsb_peer_plan: null owner output");
    const std::vector<int32_t> o = tsb::plan_owners(counts, keys, world, cap_units);
    std::copy(o.begin(), o.end(), owner);
  });
}

ss_status tsb_peer_index(const int32_t* owner, uint32_t keys, uint32_t world, int64_t* index,
                         uint64_t* units_per_rank) {
  return guard([&] {
    need(owner || !keys, "tsb_peer_index: null owner");
    need(world >= 1, "tsb_peer_index: world must be >= 1");
    std::vector<uint64_t> per;
    const std::vector<int64_t> ix = tsb::store_index(std::vector<int32_t>(owner, owner + keys), world, &per);
    if (index) std::copy(ix.begin(), ix.end(), index);
    if (units_per_rank) std::copy(per.begin(), per.end(), units_per_rank);
  });
}

ss_status tsb_test_resident_replay(int32_t n_units, int32_t capacity, int32_t policy, uint32_t window,
                                  const int32_t* place_units, const uint8_t* place_pin, uint32_t n_place, uint32_t steps,
                                  const int32_t* routed, uint32_t k, const uint8_t* flags, const int32_t* max_ev,
                                  const uint8_t* admit_misses, int32_t* slots_out, int32_t* counts_out) {
  using RS = tsb::ResidentSet;
  return guard([&] {
    need(n_units > 0 && capacity >= 0 && (policy == 0 || policy == 1) && (place_units || !n_place) &&
             (routed || !steps || !k) && flags && max_ev && admit_misses && slots_out && counts_out,
         "resident replay: bad argument");
    RS rs(n_units, capacity, policy == 1, window);
    for (uint32_t i = 0; i < n_place; ++i) rs.place(place_units[i], place_pin && place_pin[i]);
    for (uint32_t t = 0; t < steps; ++t) {
      std::vector<char> count(size_t(n_units), 0), busy(size_t(n_units), 0);
      for (uint32_t i = 0; i < k; ++i) {
        const int32_t u = routed[size_t(t) * k + i];
        need(u < n_units, "resident replay: unit out of range");
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
  });
}

ss_status tsb_test_dg_layout(const ss_desc* d, const ss_plan* p, const ss_options* o, uint64_t* out, uint32_t n_out,
                             uint32_t* residents, uint32_t cap) {
  return guard([&] {
    need(d && p && o && (out || !n_out) && (residents || !cap), "tsb_test_dg_layout: null argument");
    const ss_options oo = versioned(o, options_defaults, "tsb_test_dg_layout options");
    std::vector<uint32_t> res;
    const std::vector<uint64_t> v = tsb::dg_layout_summary(d->d, p->p, oo, &res);
    for (uint32_t i = 0; i < n_out && i < v.size(); ++i) out[i] = v[i];
    for (uint32_t i = 0; i < cap && i < res.size(); ++i) residents[i] = res[i];
  });
}

ss_status tsb_test_sha256(const void* data, uint64_t len, uint8_t* out) {
  return guard([&] {
    need((data || !len) && out, "tsb_test_sha256: null argument");
    const std::string h = tsb::sha256(data, size_t(len));
    std::memcpy(out, h.data(), 32);
  });
}

ss_status tsb_test_read_pool(void) {
  return guard([] { tsb::check_read_pool(); });
}

ss_status tsb_test_read_depth(uint32_t bound, const double* params, uint32_t n, const uint64_t* reads,
                              const uint64_t* bytes, const uint64_t* ns, uint32_t* depth, uint64_t* counters,
                              double* verdicts, uint32_t* n_verdicts) {
  return guard([&] {
    need((reads && bytes && ns && depth) || !n, "tsb_test_read_depth: null argument");
    tsb::ReadDepth::Params p;
    if (params) {
      p.min_reads = uint64_t(params[0]);
      p.recheck_u = uint64_t(params[1]);
      p.backoff_1 = uint64_t(params[2]);
      p.backoff_max = uint64_t(params[3]);
      p.bar = params[4];
      p.drift = params[5];
    }
    tsb::ReadDepth c(bound, p);
    for (uint32_t i = 0; i < n; ++i) depth[i] = c.on_busy(reads[i], bytes[i], ns[i]);
    if (counters) {
      const uint64_t v[11] = {c.changes, c.calibrations, c.windows, c.reads_1, c.bytes_1, c.ns_1,
                              c.reads_u, c.bytes_u, c.ns_u, c.verdicts(), c.calibrating() ? 1u : 0u};
      std::memcpy(counters, v, sizeof v);
    }
    uint32_t at = 0;
    for (const tsb::ReadDepth::Verdict& v : c.recent()) {
      if (verdicts) {
        const double row[7] = {double(v.seq), double(v.reads), double(v.from), double(v.to), v.rate_u, v.rate_1,
                               double(v.why)};
        std::memcpy(verdicts + size_t(at) * 7, row, sizeof row);
      }
      ++at;
    }
    if (n_verdicts) *n_verdicts = at;
  });
}

ss_status tsb_test_score_profile(const ss_desc* d, const void* profile, uint64_t len, uint8_t* identity,
                                 uint32_t* cells, uint64_t cells_cap) {
  return guard([&] {
    need(d && identity, "tsb_test_score_profile: null argument");
    std::vector<int> gated;
    std::vector<uint32_t> units;
    for (size_t L = 0; L < d->d.layers.size(); ++L)
      if (d->d.layers[L].n_units > 0) {
        gated.push_back(int(L));
        units.push_back(uint32_t(d->d.layers[L].n_units));
      }
    const std::string id = tsb::score_identity(d->d, gated);
    std::memcpy(identity, id.data(), 32);
    if (!profile && !len) return;
    const tsb::ScoreProfile p = tsb::check_score_profile(profile, len, units, id);
    uint64_t at = 0;
    for (const auto& layer : p.cells)
      for (uint32_t v : layer) {
        if (cells && at < cells_cap) cells[at] = v;
        ++at;
      }
  });
}

ss_status tsb_peer_store_create(const ss_desc* d, const int32_t* owner, uint32_t keys, int32_t rank, int device,
                                int verify, tsb_peer_store** out) {
  return guard([&] {
    need(d && owner && out, "tsb_peer_store_create: null argument");
    *out = nullptr;
    auto s = std::make_unique<tsb_peer_store>();
    s->s = std::make_unique<tsb::PeerStore>(d->d, std::vector<int32_t>(owner, owner + keys), rank, device, verify != 0);
    *out = s.release();
  });
}
ss_status tsb_peer_store_alloc(const ss_desc* d, const int32_t* owner, uint32_t keys, int32_t rank, int device,
                               tsb_peer_store** out) {
  return guard([&] {
    need(d && owner && out, "tsb_peer_store_alloc: null argument");
    *out = nullptr;
    auto s = std::make_unique<tsb_peer_store>();
    s->s = std::make_unique<tsb::PeerStore>(d->d, std::vector<int32_t>(owner, owner + keys), rank, device, false,
                                            false);
    *out = s.release();
  });
}
void tsb_peer_store_free(tsb_peer_store* s) { delete s; }
void* tsb_peer_store_base(const tsb_peer_store* s) { return s && s->s ? s->s->base() : nullptr; }
uint64_t tsb_peer_store_bytes(const tsb_peer_store* s) { return s && s->s ? s->s->bytes() : 0; }
ss_status tsb_peer_store_export(const tsb_peer_store* s, void* handle) {
  return guard([&] {
    need(s && s->s, "tsb_peer_store_export: null store");
    tsb::ipc_export(s->s->base(), handle);
  });
}
ss_status tsb_peer_map(const void* handle, int device, void** base) {
  return guard([&] {
    need(handle && base, "tsb_peer_map: null argument");
    *base = tsb::ipc_map(handle, device);
  });
}
ss_status tsb_peer_unmap(void* base) {
  return guard([&] { tsb::ipc_unmap(base); });
}

ss_status tsb_test_peer_pieces(const uint64_t* part_bytes, uint32_t n_parts, uint32_t world, int32_t rank,
                               uint64_t* copies, uint32_t cap, uint32_t* n) {
  return guard([&] {
    need(part_bytes && n_parts && n && (copies || !cap), "tsb_test_peer_pieces: null argument");
    need(world >= 1 && rank >= 0 && uint32_t(rank) < world, "tsb_test_peer_pieces: rank outside [0, world)");
    const std::vector<uint64_t> bytes_of(part_bytes, part_bytes + n_parts);
    std::vector<uint64_t> offset(n_parts);
    uint64_t unit = 0;
    for (uint32_t p = 0; p < n_parts; ++p) {
      offset[p] = unit;
      unit += part_bytes[p];
    }
    tsb::PeerTier t;  // one owned key at position 0 of every store, stores at fake addresses r << 40
    t.world = world;
    t.rank = rank;
    t.layout = tsb::kStriped;
    t.stripe = tsb::stripe_bytes(unit, world);
    t.owner = {0};
    t.index = {0};
    for (uint32_t r = 0; r < world; ++r) t.base.push_back(reinterpret_cast<char*>(uintptr_t(r + 1) << 40));
    uint32_t at = 0;
    t.pieces(0, unit, [&](const char* src, uint64_t off, uint64_t bytes, int32_t from) {
      const uint64_t in_stripe = uint64_t(reinterpret_cast<uintptr_t>(src) - (uintptr_t(from + 1) << 40));
      tsb::split_parts(offset, bytes_of, off, bytes, [&](uint32_t p, uint64_t a, uint64_t len) {  // the mover's split
        if (at < cap) {
          const uint64_t row[5] = {uint64_t(from), in_stripe + (a - off), p, a - offset[p], len};
          std::memcpy(copies + size_t(at) * 5, row, sizeof row);
        }
        ++at;
      });
    });
    *n = at;
  });
}

uint64_t tsb_peer_stripe_bytes(uint64_t unit_bytes, uint32_t world) {
  return world ? tsb::stripe_bytes(unit_bytes, world) : 0;
}

ss_status tsb_peer_store_create_striped(const ss_desc* d, const int32_t* owner, uint32_t keys, int32_t rank,
                                        uint32_t world, int device, int fill, tsb_peer_store** out) {
  return guard([&] {
    need(d && owner && out, "tsb_peer_store_create_striped: null argument");
    *out = nullptr;
    auto s = std::make_unique<tsb_peer_store>();
    s->s = std::make_unique<tsb::PeerStore>(d->d, std::vector<int32_t>(owner, owner + keys), rank, device, false,
                                            fill != 0, tsb::kStriped, world);
    *out = s.release();
  });
}

namespace {
// A tsb_peer_tier checked and turned into the library's form (keys: the gated units of the descriptor; unit_bytes:
// theirs, for the stripe size, or 0 where the context already knows it).
tsb::PeerTier tier_from(const tsb_peer_tier* peer, uint32_t keys, uint64_t unit_bytes) {
  tsb::PeerTier t;
  need(peer->struct_size >= sizeof(tsb_peer_tier), "tsb_peer_tier: struct_size is smaller than this build's");
  need(peer->world >= 1, "tsb_peer_tier: world must be >= 1");
  need(peer->rank >= 0 && uint32_t(peer->rank) < peer->world, "tsb_peer_tier: rank outside [0, world)");
  need(peer->copy <= 1, "tsb_peer_tier: copy must be 0 (land kernel) or 1 (copy engines)");
  need(peer->owner && peer->store_base, "tsb_peer_tier: null owner or store_base");
  tsb::require(peer->keys == keys, SS_E_INVALID,
               "tsb_peer_tier: keys " + std::to_string(peer->keys) + " where the descriptor has " +
                   std::to_string(keys) + " gated units");
  need(peer->layout <= 1, "tsb_peer_tier: layout must be 0 (whole units) or 1 (striped)");
  t.world = peer->world;
  t.rank = peer->rank;
  t.copy = int(peer->copy);
  t.layout = peer->layout;
  t.owner.assign(peer->owner, peer->owner + peer->keys);
  std::vector<uint64_t> per;
  t.index = tsb::store_index(t.owner, t.world, &per);  // (checks every owner is a rank below world)
  for (uint32_t r = 0; r < peer->world; ++r) t.base.push_back(static_cast<char*>(peer->store_base[r]));
  if (t.layout == tsb::kStriped) {
    uint64_t owned = 0;
    t.index = tsb::striped_index(t.owner, &owned);
    t.stripe = unit_bytes ? tsb::stripe_bytes(unit_bytes, t.world) : 0;
    for (uint32_t r = 0; r < t.world && unit_bytes; ++r)
      tsb::require(!owned || !tsb::stripe_len(unit_bytes, t.stripe, r) || t.base[r], SS_E_INVALID,
                   "tsb_peer_tier: rank " + std::to_string(r) + " holds a stripe of " + std::to_string(owned) +
                       " units but its store_base is null");
  } else {
    for (uint32_t r = 0; r < t.world; ++r)
      tsb::require(!per[r] || t.base[r], SS_E_INVALID,
                   "tsb_peer_tier: rank " + std::to_string(r) + " owns " + std::to_string(per[r]) +
                       " units but its store_base is null");
  }
  t.all_owned = std::all_of(t.owner.begin(), t.owner.end(), [](int32_t o) { return o >= 0; });
  return t;
}
}  // namespace

ss_status tsb_dg_peer_retier(ss_ctx* c, const tsb_peer_tier* peer) {
  return ctx_guard(c, [&] {
    need(peer != nullptr, "tsb_dg_peer_retier: null tier");
    auto& dg = dg_of(c, "tsb_dg_peer_retier");
    dg.set_peer(tier_from(peer, peer->keys, 0));
  });
}

ss_status tsb_peer_store_migrate(tsb_peer_store* dst, const int32_t* old_owner, void* const* old_base, uint32_t keys,
                                 uint32_t world, void* stream, uint64_t* moved_units, uint64_t* moved_peer_units,
                                 uint64_t* moved_bytes) {
  return guard([&] {
    need(dst && dst->s && old_owner && old_base, "tsb_peer_store_migrate: null argument");
    need(world >= 1, "tsb_peer_store_migrate: world must be >= 1");
    std::vector<char*> bases;
    for (uint32_t r = 0; r < world; ++r) bases.push_back(static_cast<char*>(old_base[r]));
    const tsb::Migration m =
        tsb::migrate_store(*dst->s, std::vector<int32_t>(old_owner, old_owner + keys), bases, stream);
    if (moved_units) *moved_units = m.units;
    if (moved_peer_units) *moved_peer_units = m.peer_units;
    if (moved_bytes) *moved_bytes = m.bytes;
  });
}

ss_status tsb_open_peer(const ss_desc* d, const ss_budget* budget, const ss_plan* plan, const ss_options* opt,
                        const tsb_peer_tier* peer, ss_ctx** out) {
  tsb::PeerTier t;
  const ss_status st = guard([&] {
    need(d && peer, "tsb_open_peer: null argument");
    const tsb::GatedKeys gk = tsb::gated_keys(d->d);
    t = tier_from(peer, gk.keys(), gk.unit_bytes);
  });
  if (st != SS_OK) return st;
  return open_impl(d, budget, plan, opt, &t, out);
}

ss_status tsb_peer_tier_verify(const ss_desc* d, const tsb_peer_tier* peer, int device, uint64_t* checked_units) {
  return guard([&] {
    need(d && peer, "tsb_peer_tier_verify: null argument");
    const tsb::GatedKeys gk = tsb::gated_keys(d->d);
    const uint64_t n = tsb::verify_tier(d->d, tier_from(peer, gk.keys(), gk.unit_bytes), device);
    if (checked_units) *checked_units = n;
  });
}

// ---- not in this build ----
void ss_dg_winpf_defaults_sized(ss_dg_winpf_params*, uint32_t) {}
ss_status ss_dg_winpf_set(ss_ctx*, const ss_dg_winpf_params*) { return unsupported("ss_dg_winpf_set"); }
ss_status ss_dg_window_hint(ss_ctx*, const int32_t*, const float*, uint32_t) { return unsupported("ss_dg_window_hint"); }
ss_status ss_recipe_from_text(const char*, size_t, const char*, ss_recipe**) { return unsupported("ss_recipe_from_text"); }
ss_status ss_recipe_from_file(const char*, ss_recipe**) { return unsupported("ss_recipe_from_file"); }
void ss_recipe_free(ss_recipe*) {}
ss_status ss_recipe_add_profile(ss_recipe*, const char*, size_t, const char*, const char*, size_t) {
  return unsupported("ss_recipe_add_profile");
}
ss_status ss_recipe_add_overrides(ss_recipe*, const char*, size_t, const char*) {
  return unsupported("ss_recipe_add_overrides");
}
ss_status ss_recipe_set(ss_recipe*, const char*, const char*, const char*) { return unsupported("ss_recipe_set"); }
ss_status ss_recipe_to_json(const ss_recipe*, char**, size_t*) { return unsupported("ss_recipe_to_json"); }
ss_status ss_recipe_explain(const ss_recipe*, char**, size_t*) { return unsupported("ss_recipe_explain"); }
ss_status ss_recipe_match(const ss_recipe*, const char*, size_t, char**, size_t*) { return unsupported("ss_recipe_match"); }
ss_status ss_recipe_select(const ss_recipe*, const char*, size_t, char**, size_t*) {
  return unsupported("ss_recipe_select");
}
ss_status ss_recipe_plan(const ss_recipe*, const char*, const char*, int, const char*, const ss_desc*, const double*,
                         size_t, const ss_desc* const*, const double* const*, const size_t*, size_t, ss_budget*,
                         ss_options*, ss_plan**, char**, size_t*) {
  return unsupported("ss_recipe_plan");
}
void ss_mfile_options_defaults_sized(ss_mfile_options*, uint32_t) {}
ss_status ss_mfile_open(const char*, const char*, const ss_mfile_options*, ss_mfile**) { return unsupported("ss_mfile_open"); }
void ss_mfile_close(ss_mfile*) {}
uint64_t ss_mfile_size(const ss_mfile*) { return 0; }
uint32_t ss_mfile_alignment(const ss_mfile*) { return 0; }
int ss_mfile_multi(const ss_mfile*) { return 0; }
ss_status ss_mfile_pread(ss_mfile*, void*, uint64_t, uint64_t, uint64_t*) { return unsupported("ss_mfile_pread"); }
ss_status ss_mfile_preadv(ss_mfile*, const ss_mfile_io*, uint32_t) { return unsupported("ss_mfile_preadv"); }
ss_status ss_mfile_get_counters(const ss_mfile*, ss_mfile_counters*) { return unsupported("ss_mfile_get_counters"); }
const char* ss_mfile_location_path(const ss_mfile*, int) { return nullptr; }
const char* ss_mfile_open_report(const ss_mfile*) { return nullptr; }
ss_status ss_mfile_location_info(const ss_mfile*, uint32_t, ss_mfile_location*) {
  return unsupported("ss_mfile_location_info");
}
void ss_budget_in_defaults_sized(ss_budget_in*, uint32_t) {}
ss_status ss_budget_plan(const ss_budget_in*, ss_budget_out*) { return unsupported("ss_budget_plan"); }
size_t ss_budget_plan_json(const ss_budget_in*, const ss_budget_out*, char*, size_t) { return 0; }
ss_status ss_budget_ledger_create(uint64_t, uint64_t, ss_budget_ledger**) { return unsupported("ss_budget_ledger_create"); }
void ss_budget_ledger_free(ss_budget_ledger*) {}
ss_status ss_budget_ledger_add(ss_budget_ledger*, ss_budget_kind, const char*, uint64_t) {
  return unsupported("ss_budget_ledger_add");
}
ss_status ss_budget_ledger_sub(ss_budget_ledger*, ss_budget_kind, const char*, uint64_t) {
  return unsupported("ss_budget_ledger_sub");
}
ss_status ss_budget_ledger_observe_device(ss_budget_ledger*, uint64_t) {
  return unsupported("ss_budget_ledger_observe_device");
}
ss_status ss_budget_ledger_stats(const ss_budget_ledger*, ss_budget_stats*) { return unsupported("ss_budget_ledger_stats"); }
ss_status ss_budget_ledger_observe(ss_budget_ledger*, const char*, uint64_t, uint64_t) {
  return unsupported("ss_budget_ledger_observe");
}
int ss_budget_ledger_within_caps(const ss_budget_ledger*) { return 0; }
ss_status ss_budget_in_dg_library(ss_budget_in*, const ss_desc*, const ss_options*) {
  return unsupported("ss_budget_in_dg_library");
}
ss_status ss_dg_make_resident(ss_ctx* c, int g, const int32_t* ids, int n) {
  return ctx_guard(c, [&] { dg_of(c, "ss_dg_make_resident").make_resident(g, ids, n); });
}
namespace {
void round_defaults(ss_dg_round_params* p) {
  *p = ss_dg_round_params{};
  p->struct_size = uint32_t(sizeof *p);
  p->budget_bytes = 0;
  p->max_units = 96;
  p->hysteresis = 1.25f;
  p->decay = 0.85f;
}
ss_dg_round_result round_result(const tsb::RoundOut& r) {
  ss_dg_round_result x{};
  x.promoted_to_device = r.promoted_to_device;
  x.promoted_to_pinned = r.promoted_to_pinned;
  x.demoted_from_device = r.demoted_from_device;
  x.dropped_to_file = r.dropped_to_file;
  x.cancelled = r.cancelled;
  x.bytes_read = r.bytes_read;
  x.bytes_h2d = r.bytes_h2d;
  x.bytes_written_back = r.bytes_written_back;
  x.ns = r.ns;
  return x;
}
}  // namespace
void ss_dg_round_defaults_sized(ss_dg_round_params* p, uint32_t size) { sized_defaults(p, size, round_defaults); }
ss_status ss_dg_round_sized(ss_ctx* c, const ss_dg_round_params* p, ss_dg_round_result* out, uint32_t size) {
  return ctx_guard(c, [&] {
    need(!out || size >= sizeof(uint32_t), "ss_dg_round: bad result size");
    const ss_dg_round_params v = versioned(p, round_defaults, "ss_dg_round");
    tsb::RoundIn in;
    in.flags = v.flags;
    in.budget_bytes = v.budget_bytes;
    in.max_units = v.max_units;
    in.hysteresis = double(v.hysteresis);
    in.decay = double(v.decay);
    tsb::DgContext& dg = dg_of(c, "ss_dg_round");
    // the result is written however the round ends: a failure after the round began still reports the moves it made
    struct ReportOnExit {
      const tsb::DgContext& dg;
      ss_dg_round_result* out;
      uint32_t size;
      ~ReportOnExit() {
        if (out) give_sized(out, size, round_result(dg.last_round()));
      }
    } report{dg, out, size};
    dg.round(in);
  });
}
// Any thread: one atomic store, no context state read (a poisoned or busy context is the engine's to report).
ss_status ss_dg_round_cancel(ss_ctx* c) {
  if (!c || !c->dg) return refuse(SS_E_INVALID, "ss_dg_round_cancel: not a device-gated context");
  c->dg->round_cancel();
  return SS_OK;
}
ss_status ss_dg_round_seed_counts(ss_ctx* c, const ss_dg_unit* units, const float* counts, uint32_t n) {
  return ctx_guard(c, [&] {
    need(n == 0 || (units && counts), "ss_dg_round_seed_counts: bad arguments");
    dg_of(c, "ss_dg_round_seed_counts").round_seed_counts(units, counts, n);
  });
}
void ss_devprof_detect_opts_defaults_sized(ss_devprof_detect_opts*, uint32_t) {}
ss_status ss_devprof_detect(const ss_devprof_detect_opts*, ss_devprof**) { return unsupported("ss_devprof_detect"); }
ss_status ss_devprof_from_json(const char*, size_t, ss_devprof**) { return unsupported("ss_devprof_from_json"); }
ss_status ss_devprof_merge_json(ss_devprof*, const char*, size_t, const char*) { return unsupported("ss_devprof_merge_json"); }
void ss_devprof_free(ss_devprof*) {}
ss_status ss_devprof_to_json(const ss_devprof*, char**, size_t*) { return unsupported("ss_devprof_to_json"); }
ss_status ss_devprof_hash(const ss_devprof*, char[17]) { return unsupported("ss_devprof_hash"); }
ss_status ss_devprof_probe_report(const ss_devprof*, const char*, char**, size_t*) {
  return unsupported("ss_devprof_probe_report");
}
ss_status ss_devprof_get(const ss_devprof*, ss_devprof_info*) { return unsupported("ss_devprof_get"); }
ss_status ss_devprof_limit(const ss_devprof*, const char*, uint64_t*) { return unsupported("ss_devprof_limit"); }
ss_status ss_devprof_get_device(const ss_devprof*, uint32_t, ss_devprof_device*) { return unsupported("ss_devprof_get_device"); }
ss_status ss_devprof_budget(const ss_devprof*, uint32_t, ss_budget_in*) { return unsupported("ss_devprof_budget"); }
void ss_devprof_topology_in_defaults_sized(ss_devprof_topology_in*, uint32_t) {}
ss_status ss_devprof_topology(const ss_devprof* const*, uint32_t, const ss_devprof_topology_in*, ss_devprof_topology_out*) {
  return unsupported("ss_devprof_topology");
}
void ss_devprof_piece_in_defaults_sized(ss_devprof_piece_in*, uint32_t) {}
ss_status ss_devprof_piece_rows(const ss_devprof*, const ss_devprof_piece_in*, uint32_t*) {
  return unsupported("ss_devprof_piece_rows");
}
void ss_pack_options_defaults_sized(ss_pack_options*, uint32_t) {}
ss_status ss_pack_open(const char*, const ss_pack_options*, ss_pack**) { return unsupported("ss_pack_open"); }
void ss_pack_close(ss_pack*) {}
uint64_t ss_pack_records(const ss_pack*) { return 0; }
ss_status ss_pack_entry_at_sized(const ss_pack*, uint64_t, ss_pack_entry*, uint32_t) { return unsupported("ss_pack_entry_at"); }
ss_status ss_pack_find_sized(const ss_pack*, int, int, const char*, ss_pack_entry*, uint32_t) {
  return unsupported("ss_pack_find");
}
ss_status ss_pack_segment_at(const ss_pack*, uint64_t, uint32_t, ss_pack_segment*) { return unsupported("ss_pack_segment_at"); }
ss_status ss_pack_unit_find(const ss_pack*, int, int, ss_pack_unit*) { return unsupported("ss_pack_unit_find"); }
ss_status ss_pack_read(ss_pack*, uint64_t, uint32_t, uint32_t, void*) { return unsupported("ss_pack_read"); }
ss_status ss_pack_readv(ss_pack*, const ss_pack_read_req*, uint32_t) { return unsupported("ss_pack_readv"); }
ss_status ss_pack_read_unit(ss_pack*, int, int, void*) { return unsupported("ss_pack_read_unit"); }
ss_status ss_pack_dg_descriptor(ss_pack*, const char*, size_t, char**, size_t*) { return unsupported("ss_pack_dg_descriptor"); }
uint32_t ss_pack_files(const ss_pack*) { return 0; }
int ss_pack_has_layout(const ss_pack*, const char*) { return 0; }
ss_status ss_pack_file_identity(const ss_pack*, uint32_t, ss_file_identity*) { return unsupported("ss_pack_file_identity"); }
ss_status ss_pack_info_json(const ss_pack*, char**, size_t*) { return unsupported("ss_pack_info_json"); }
ss_status ss_pack_verify_full(ss_pack*, char**, size_t*) { return unsupported("ss_pack_verify_full"); }
ss_status ss_pack_writer_begin(const char*, const char*, size_t, ss_pack_writer**) { return unsupported("ss_pack_writer_begin"); }
ss_status ss_pack_writer_record_begin(ss_pack_writer*, const ss_pack_record_spec*) {
  return unsupported("ss_pack_writer_record_begin");
}
ss_status ss_pack_writer_record_write(ss_pack_writer*, const void*, uint64_t) {
  return unsupported("ss_pack_writer_record_write");
}
ss_status ss_pack_writer_record_end(ss_pack_writer*) { return unsupported("ss_pack_writer_record_end"); }
ss_status ss_pack_writer_add(ss_pack_writer*, const ss_pack_record_spec*, const void*) { return unsupported("ss_pack_writer_add"); }
ss_status ss_pack_writer_finish(ss_pack_writer*, char*) { return unsupported("ss_pack_writer_finish"); }
void ss_pack_writer_abort(ss_pack_writer*) {}
ss_status ss_dg_set_clean_evict(ss_ctx* c, uint32_t on) {
  return ctx_guard(c, [&] { dg_of(c, "ss_dg_set_clean_evict").set_clean_evict(on); });
}
ss_status ss_dg_begin_layer(ss_ctx*, int, int) { return unsupported("ss_dg_begin_layer"); }
ss_status ss_dg_enqueue_export_part(ss_ctx*, int, int, const int32_t*, int, void*) {
  return unsupported("ss_dg_enqueue_export_part");
}
ss_status ss_dg_enqueue_wait_part(ss_ctx*, int, int, void*) { return unsupported("ss_dg_enqueue_wait_part"); }
ss_status ss_dg_enqueue_end_layer(ss_ctx*, void*) { return unsupported("ss_dg_enqueue_end_layer"); }
ss_status ss_dg_set_pf_revert_unused(ss_ctx* c, uint32_t on) {
  return ctx_guard(c, [&] { dg_of(c, "ss_dg_set_pf_revert_unused").set_pf_revert_unused(on); });
}

}  // extern "C"
