// The two context kinds behind ss_ctx: host forward mode (host_ctx.cpp) and device-gated decode (dg_ctx.cu). capi.cpp
// dispatches the ss_* calls to them and maps their exceptions to ss_status.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "desc.hpp"
#include "plan.hpp"
#include "dg_core.hpp"
#include "strix_stream/ss.h"

namespace tsb {

// Makes `device` the calling thread's current CUDA device for the scope and puts the caller's back on exit, so no
// ss_* call leaves the engine thread on another device than it had (a failed switch shows in the calls that follow).
class DeviceScope {
 public:
  explicit DeviceScope(int device);
  ~DeviceScope();
  DeviceScope(const DeviceScope&) = delete;
  DeviceScope& operator=(const DeviceScope&) = delete;

 private:
  int prev_ = -1;
};

struct PeerTier;

class DgContext {
 public:
  virtual ~DgContext() = default;
  virtual bool poisoned() const = 0;
  virtual int device() const = 0;  // the CUDA device the context lives on
  virtual void poison() = 0;
  virtual int n_sources() const = 0;
  virtual bool source_direct(int i) const = 0;
  virtual int gated_index(int layer) const = 0;
  virtual void begin(const uint32_t* rows, int n_layers) = 0;
  // rows: the token's rows (scored eviction's SCORED_AUTO takes scored victims only above 1)
  virtual void end(uint32_t rows) = 0;
  // Between tokens: LRU, SCORED or SCORED_AUTO (scoring must have been set up at the open)
  virtual void set_policy(uint32_t policy) = 0;
  // Placement rounds: one round between tokens (its result kept for last_round, also after a failure once it began);
  // a cancellation from any thread; counts set from a shipped profile
  virtual void round(const RoundIn& in) = 0;
  virtual const RoundOut& last_round() const = 0;
  virtual void round_cancel() = 0;
  virtual void round_seed_counts(const ss_dg_unit* units, const float* counts, uint32_t n) = 0;
  // Between tokens: the opt-in policies dg_clean_evict and dg_pf_revert_unused switched at run time
  virtual void set_clean_evict(uint32_t on) = 0;
  virtual void set_pf_revert_unused(uint32_t on) = 0;
  virtual void seed(int layer, const int32_t* units, int n) = 0;
  virtual void check_unit(int layer, int unit) = 0;
  virtual void device_view(ss_dg_device_view* v) const = 0;
  virtual void enqueue_begin(void* s) = 0;
  virtual void enqueue_export(int g, const int32_t* ids, int n, int n_pred, void* s) = 0;
  virtual void enqueue_predict(int g, const int32_t* ids, int n, void* s) = 0;
  virtual void enqueue_wait(int g, void* s) = 0;
  virtual void enqueue_end(void* s) = 0;
  virtual void keep(int g, const int32_t* ids, int n) = 0;
  virtual void make_resident(int g, const int32_t* ids, int n) = 0;
  virtual uint32_t residency(ss_dg_unit* out, uint32_t cap) = 0;
  virtual void set_sched(uint32_t wb_defer, uint32_t flush_ready) = 0;
  virtual void set_budgets(uint32_t spare_target, uint32_t per_layer, uint32_t per_token) = 0;
  virtual void timeline(int g, ss_dg_layer_timeline* out) const = 0;
  virtual void boundary_timeline(ss_dg_boundary_timeline* out) const = 0;
  virtual void stats(ss_dg_stats* out) const = 0;
  virtual void layer_stats(int layer, ss_layer_stats* out) const = 0;
  virtual void total_stats(ss_layer_stats* out) const = 0;
  virtual void reset_stats() = 0;
  virtual void exclusive_stats(ss_exclusive_stats* out) const = 0;
  virtual std::string stats_json() const = 0;
  virtual void reset_open() = 0;
  // The peer tier's owners and store addresses replaced between tokens (a re-plan): the same ranks, the same set of
  // owned keys; every copy that read the old stores has finished when it returns.
  virtual void set_peer(const PeerTier& t) = 0;
  // test hooks (ss_test.h), refused unless opened with dg_test_hooks
  virtual void test_mutate(int m) = 0;
  virtual void test_pressure(uint32_t free_per_token, uint32_t evict_recent) = 0;
  virtual void test_check() = 0;
  virtual void test_gate(int stream, void* event) = 0;
  virtual void test_flags(uint32_t flags) = 0;
  virtual uint32_t test_coming() = 0;
  virtual void test_stop_service() = 0;
  virtual uint32_t test_table(int32_t* out, uint32_t cap) = 0;  // the device's slot table; returns the key count
  // flips the byte at `offset` of the unit's pinned block (a Host home with a block), between tokens
  virtual void test_corrupt(int layer, int unit, uint64_t offset) = 0;
};

struct PeerTier;
// peer: the peer tier (peer.hpp), or null for pinned RAM only.
// The device-gated layout of an open (no device work): the numbers of the layout test hook, the residents' keys.
std::vector<uint64_t> dg_layout_summary(const Desc& d, const Plan& p, const ss_options& o,
                                        std::vector<uint32_t>* residents);
std::unique_ptr<DgContext> open_dg_context(const Desc& d, const Plan& p, const ss_options& o,
                                           const PeerTier* peer = nullptr);

class HostContext {
 public:
  virtual ~HostContext() = default;
  virtual bool poisoned() const = 0;
  virtual int device() const = 0;  // the CUDA device the context lives on
  virtual void poison() = 0;
  virtual int n_sources() const = 0;
  virtual bool source_direct(int i) const = 0;
  virtual void seed(int layer, const int32_t* units, int n) = 0;
  virtual void begin(const uint32_t* rows, int n_layers) = 0;
  virtual void routes(int layer, const int32_t* ids, int n) = 0;
  virtual void routes_dev(int layer, const int32_t* ids_dev, int n, void* stream) = 0;
  virtual void routes_all(int layer) = 0;
  // ss_prefetch / ss_prefetch_layer: issue the copies of a layer's units ahead of its routes (certain: admitted as a
  // demand; speculative: the stream ring only, budgeted); allowed between forwards (they belong to the next one)
  virtual void prefetch(int layer, const int32_t* ids, int n, bool speculative) = 0;
  // ss_host_prefetch / ss_host_prefetch_layer (n < 0): read-ahead requests (a no-op without read-ahead buffers)
  virtual void host_prefetch(int layer, const int32_t* ids, int n) = 0;
  virtual void acquire(int layer, void* stream, bool wait_all, ss_layer_view* out) = 0;
  virtual void group_wait(int layer, int group, void* stream) = 0;
  virtual void release(int layer, void* stream) = 0;
  virtual void end() = 0;
  virtual void check_unit(int layer, int unit) = 0;
  virtual void layer_stats(int layer, ss_layer_stats* out) const = 0;
  virtual void total_stats(ss_layer_stats* out) const = 0;
  virtual void reset_stats() = 0;
  virtual void set_hook(ss_stats_hook hook, void* user) = 0;
  virtual void exclusive_stats(ss_exclusive_stats* out) const = 0;
  virtual std::string stats_json() const = 0;
  // between ss_acquire and ss_release of `layer`: per unit (loc, slot) of its table entry: (1, persistent slot),
  // (2, ring slot) or (0, -1) for no entry
  virtual void test_locs(int layer, int32_t* out, int n) const = 0;
  // between forwards: where unit (layer, unit)'s bytes are kept - its pinned block (a mapped host address, usable by
  // kernels) and its persistent device slot when resident; nullptr for either it does not have
  virtual void test_unit(int layer, int unit, void** pinned, void** device) const = 0;
};

std::unique_ptr<HostContext> open_host_context(const Desc& d, const ss_budget& b, const Plan& p, const ss_options& o);

}  // namespace tsb
