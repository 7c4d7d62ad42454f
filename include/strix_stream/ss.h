/*
 * strix-stream C ABI, version 1, as implemented by the tierstream B200 runtime.
 *
 * This header declares the same functions, enums and versioned structs as the reference tierstream library's
 * include/strix_stream/ss.h, with identical field order, types and therefore offsets, so an engine compiled against
 * either header links and runs against this library. The comments here are this build's own.
 *
 * What is implemented (everything else is exported and returns SS_E_UNSUPPORTED with a message):
 *   - descriptor (desc-v1 JSON), planner (plan_make / plan_from_tiers / plan JSON), budgets and options;
 *   - host forward mode on CUDA: ss_begin / ss_layer_routes / ss_layer_all / ss_acquire / ss_acquire_groups /
 *     ss_group_wait / ss_release / ss_end with LRU admission and pinned or file sources;
 *   - device-gated decode on CUDA (exclusive tiers, LRU): the device view, the enqueue_* kernels (graph capturable),
 *     the service thread, boundaries with write-backs, ss_dg_keep / residency / budgets / sched / timeline /
 *     reset_open and the stats.
 * There is no CPU or HIP backend in this build: ss_open refuses them with SS_E_UNSUPPORTED.
 *
 * Rules shared with the reference ABI:
 *   - one engine thread drives a context; the library runs its own threads;
 *   - versioned structs start with struct_size; the library reads min(struct_size, its own size) bytes and defaults
 *     the rest; fields are only ever appended;
 *   - SS_E_INVALID / DESC / IO / CAPACITY / HASH leave a context usable; SS_E_BACKEND / SS_E_NOMEM inside a context
 *     call poison it (every later call but ss_close and the stats calls fails);
 *   - bytes are never changed: a unit's device bytes equal its source bytes wherever it came from.
 */
#ifndef STRIX_STREAM_SS_H
#define STRIX_STREAM_SS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define SS_API __attribute__((visibility("default")))
#else
#define SS_API
#endif

#define SS_ABI_VERSION 1

typedef enum ss_status {
  SS_OK = 0,
  SS_E_INVALID = 1,     /* bad argument or call order */
  SS_E_DESC = 2,        /* descriptor parse or validation error */
  SS_E_IO = 3,          /* file open or read error */
  SS_E_NOMEM = 4,       /* host or device allocation failed */
  SS_E_BACKEND = 5,     /* CUDA error or internal failure */
  SS_E_CAPACITY = 6,    /* the plan or a ring cannot hold what is needed */
  SS_E_HASH = 7,        /* landed bytes differ from the descriptor's xxh64 */
  SS_E_UNSUPPORTED = 8, /* not in this build */
  SS_E_RECIPE = 9       /* recipe errors (recipes are not in this build) */
} ss_status;

/* Message of the calling thread's last failure (valid until its next failing call). */
SS_API const char* ss_last_error(void);
SS_API int ss_abi_version(void);

/* ---- Descriptor (strix-stream/desc-v1) ---- */
typedef struct ss_desc ss_desc;

SS_API ss_status ss_desc_from_json(const char* json_text, size_t len, ss_desc** out);
SS_API ss_status ss_desc_from_file(const char* path, ss_desc** out);
SS_API ss_status ss_desc_from_model(const char* manifest_path, ss_desc** out);
SS_API void ss_desc_free(ss_desc* d);
SS_API int ss_desc_n_layers(const ss_desc* d);
SS_API int ss_desc_layer_units(const ss_desc* d, int layer);
SS_API uint64_t ss_desc_unit_bytes(const ss_desc* d, int layer);
SS_API ss_status ss_desc_to_json(const ss_desc* d, char** out_json, size_t* out_len);
SS_API void ss_free(void* p);

/* ---- Planner ---- */
typedef enum ss_tier {
  SS_TIER_RESIDENT = 0,        /* on the device from open */
  SS_TIER_PINNED = 1,          /* copied from the pinned host tier when needed */
  SS_TIER_DISK = 2,            /* read from its file when needed */
  SS_TIER_PAIR = 3,            /* computed by another device, never fetched */
  SS_TIER_RESIDENT_BACKED = 4  /* resident, plus a pinned host copy */
} ss_tier;

typedef enum ss_tier_mode {
  SS_TIER_MODE_INCLUSIVE = 0, /* a promoted unit keeps its pinned copy */
  SS_TIER_MODE_EXCLUSIVE = 1  /* one home per unit at a boundary: a slot, a pinned block, or its file */
} ss_tier_mode;

typedef struct ss_budget {
  uint32_t struct_size;
  uint64_t device_bytes;       /* device cap for the library and the engine's fixed bytes */
  uint64_t host_pinned_bytes;  /* pinned host bytes the library may lock */
  uint64_t workspace_bytes;    /* engine workspaces already sized */
  double margin_gib;           /* default 2.0 */
  double margin_fraction;      /* default 0.03 */
  uint32_t dynamic_slots_per_layer;
  uint32_t ring_slots;
  int pinned_backing;
  uint32_t reserved0;          /* never read */
  int tier_mode;               /* ss_tier_mode */
  uint32_t host_spare_units;   /* exclusive: free pinned blocks wanted per unit size (0 = min(64, units)) */
} ss_budget;

typedef struct ss_plan ss_plan;

SS_API void ss_budget_defaults_sized(ss_budget* b, uint32_t size);
static inline void ss_budget_defaults(ss_budget* b) { ss_budget_defaults_sized(b, (uint32_t)sizeof *b); }
SS_API ss_status ss_plan_make(const ss_desc* d, const ss_budget* b, const double* benefit, size_t n_benefit,
                              ss_plan** out);
SS_API ss_status ss_plan_from_tiers(const ss_desc* d, const ss_budget* b, const uint8_t* tiers, size_t n,
                                    ss_plan** out);
SS_API ss_status ss_plan_from_json(const ss_desc* d, const ss_budget* b, const char* plan_json, size_t len,
                                   ss_plan** out);
SS_API void ss_plan_free(ss_plan* p);
SS_API ss_tier ss_plan_unit_tier(const ss_plan* p, int layer, int unit);
typedef struct ss_plan_totals {
  uint64_t fixed_bytes, margin_bytes, resident_bytes, dynamic_bytes, ring_bytes, peak_device_bytes;
  uint64_t pinned_bytes, disk_bytes;
  uint64_t n_resident, n_pinned, n_disk;
} ss_plan_totals;
SS_API void ss_plan_get_totals(const ss_plan* p, ss_plan_totals* out);
SS_API ss_status ss_plan_to_json(const ss_plan* p, char** out_json, size_t* out_len);
SS_API int64_t ss_desc_unit_index(const ss_desc* d, int layer, int unit);
SS_API int64_t ss_desc_total_units(const ss_desc* d);

/* ---- Context ---- */
typedef enum ss_backend_kind {
  SS_BACKEND_CPU = 0,   /* not in this build */
  SS_BACKEND_CUDA = 1,  /* discrete GPU (the only backend of this build) */
  SS_BACKEND_HIP = 2    /* not in this build */
} ss_backend_kind;

typedef enum ss_policy {
  SS_POLICY_LRU = 0,
  SS_POLICY_SCORED = 1,     /* not in this build */
  SS_POLICY_SCORED_AUTO = 2 /* not in this build */
} ss_policy;

struct ss_dg_unit;
struct ss_budget_ledger;

typedef struct ss_file_identity {
  uint64_t volume;
  uint64_t index;
  uint64_t size;
} ss_file_identity;

typedef struct ss_options {
  uint32_t struct_size;
  ss_backend_kind backend;          /* default SS_BACKEND_CUDA in this build */
  int device;                       /* CUDA device ordinal */
  ss_policy policy;                 /* LRU */
  uint32_t lookahead_budget;
  uint32_t reader_threads;          /* file reader threads (host mode, default 2) */
  uint32_t staging_buffers;         /* default 4 */
  uint64_t staging_bytes;           /* default 256 MiB */
  uint64_t copy_piece_bytes;        /* default 64 MiB */
  int verify_hash;                  /* 1 = check every landed unit's xxh64 (on the device in this build) */
  int fill_residents;               /* default 1 */
  uint32_t score_window;
  int pin_planned;                  /* host mode: 1 = planned residents are never evicted */
  int direct_io;                    /* default 1 */
  uint32_t group_units;
  int spec_persistent;
  uint32_t reserved0;
  uint32_t readahead_units;
  uint32_t reserved1;
  int forward_mode;                 /* ss_forward_mode */
  uint32_t dg_max_ids;              /* routed ids per gated layer per token, 1..64 */
  uint32_t dg_prefetch_reserve;     /* 0xFFFFFFFF = min(24, spare_target / 4) */
  uint32_t dg_prefetch_per_layer;   /* default 4 */
  uint32_t dg_prefetch_per_token;   /* default 48 */
  uint32_t dg_wait_timeout_ms;      /* default 10000 */
  uint32_t dg_service_boost;
  uint32_t dg_diag;                 /* 1 = per-layer timeline of the last token */
  uint32_t dg_test_hooks;           /* 1 = the ss_test_dg_* hooks act on this context */
  uint32_t dg_spare_target;         /* 0xFFFFFFFF = every billed spare slot */
  uint32_t dg_seed_n;
  const struct ss_dg_unit* dg_seed; /* read during ss_open only */
  uint32_t dg_spare_slots;
  uint32_t dg_flush_ready;
  uint32_t dg_wb_defer;             /* default 1 */
  uint32_t dg_wb_stream;            /* default 1 */
  uint32_t dg_wb_layer_bytes;
  uint32_t dg_wb_max_outstanding;
  uint64_t dg_prior_len;
  const void* dg_prior;
  uint32_t exclusive_discard;
  uint32_t reserved2;
  uint32_t dg_score_w_trans, dg_score_w_freq, dg_score_w_recency;
  uint32_t reserved3;
  uint64_t dg_score_profile_len;
  const void* dg_score_profile;
  const char* weight_dirs;
  uint32_t drive_readers;
  int weight_verify;
  uint32_t dg_disk_tier;
  uint32_t dg_disk_prefetch;
  uint32_t dg_disk_staging;
  uint32_t dg_inclusive_blocks;
  uint32_t dg_disk_queue;
  uint32_t reserved4;
  uint32_t source_identity_n;
  uint32_t reserved5;
  const ss_file_identity* source_identities;
  struct ss_budget_ledger* budget;
  uint32_t dg_no_admit;
  uint32_t reserved6;
  uint32_t dg_clean_evict;
  uint32_t reserved7;
  uint32_t dg_pf_revert_unused;
  uint32_t reserved8;
  uint32_t dg_pf_strict_admit;
  uint32_t reserved9;
  uint32_t dg_landing_blocks;
  uint32_t dg_landing_max_queued;
  uint32_t dg_landing_ttl;
  uint32_t reserved10;
  uint32_t dg_landing_chunk;
  uint32_t reserved11;
  uint32_t dg_bank_keep;
  uint32_t reserved12;
  uint32_t dg_disk_queue_adapt;
  uint32_t reserved13;
} ss_options;

typedef enum ss_forward_mode { SS_FORWARD_HOST = 0, SS_FORWARD_DEVICE_GATED = 1 } ss_forward_mode;

typedef struct ss_ctx ss_ctx;

SS_API void ss_options_defaults_sized(ss_options* o, uint32_t size);
static inline void ss_options_defaults(ss_options* o) { ss_options_defaults_sized(o, (uint32_t)sizeof *o); }
SS_API ss_status ss_open(const ss_desc* d, const ss_budget* budget, const ss_plan* plan, const ss_options* opt,
                         ss_ctx** out);
SS_API void ss_close(ss_ctx* c);
SS_API int ss_source_direct(const ss_ctx* c, int source);
SS_API ss_status ss_seed(ss_ctx* c, int layer, const int32_t* units, int n);

/* ---- One forward ---- */
SS_API ss_status ss_begin(ss_ctx* c, const uint32_t* rows_per_layer, int n_layers);
SS_API ss_status ss_layer_routes(ss_ctx* c, int layer, const int32_t* ids, int n);
SS_API ss_status ss_layer_routes_dev(ss_ctx* c, int layer, const int32_t* ids_dev, int n, void* engine_stream);
SS_API ss_status ss_layer_all(ss_ctx* c, int layer);

typedef enum ss_prefetch_kind { SS_PREFETCH_CERTAIN = 0, SS_PREFETCH_SPECULATIVE = 1 } ss_prefetch_kind;
SS_API ss_status ss_prefetch(ss_ctx* c, int layer, const int32_t* ids, int n, ss_prefetch_kind kind);
SS_API ss_status ss_prefetch_layer(ss_ctx* c, int layer);
SS_API ss_status ss_host_prefetch(ss_ctx* c, int layer, const int32_t* ids, int n);
SS_API ss_status ss_host_prefetch_layer(ss_ctx* c, int layer);
SS_API ss_status ss_lookahead_select(const float* scores, int rows, int n_experts, int top_k, int32_t* out,
                                     int max_out, int* n_out);

typedef struct ss_group {
  const int32_t* units; /* ascending unit ids */
  int n_units;
} ss_group;
typedef struct ss_layer_view {
  const uint64_t* table_dev;  /* device array: n_units device addresses (0 = not available this forward) */
  const uint64_t* table_host; /* the same table in host memory */
  int n_units;
  const ss_group* groups;
  int n_groups;
} ss_layer_view;

SS_API ss_status ss_acquire(ss_ctx* c, int layer, void* engine_stream, ss_layer_view* out);
SS_API ss_status ss_acquire_groups(ss_ctx* c, int layer, void* engine_stream, ss_layer_view* out);
SS_API ss_status ss_group_wait(ss_ctx* c, int layer, int group, void* engine_stream);
SS_API ss_status ss_release(ss_ctx* c, int layer, void* engine_stream);
SS_API ss_status ss_end(ss_ctx* c);
SS_API ss_status ss_check_unit(ss_ctx* c, int layer, int unit);

/* ---- Stats ---- */
typedef struct ss_layer_stats {
  uint64_t routed, hits, admitted, transient, evicted, prefetched;
  uint64_t spec_issued, spec_used, spec_dropped;
  uint64_t bytes_pinned, bytes_disk, wait_ns;
} ss_layer_stats;

SS_API ss_status ss_stats_layer(const ss_ctx* c, int layer, ss_layer_stats* out);
SS_API ss_status ss_stats_total(const ss_ctx* c, ss_layer_stats* out);
SS_API void ss_stats_reset(ss_ctx* c);
typedef void (*ss_stats_hook)(void* user, const ss_layer_stats* forward_total, const ss_layer_stats* per_layer,
                              int n_layers);
SS_API void ss_set_stats_hook(ss_ctx* c, ss_stats_hook hook, void* user);
SS_API ss_status ss_stats_to_json(const ss_ctx* c, char** out_json, size_t* out_len);

typedef struct ss_exclusive_stats {
  uint32_t struct_size;
  uint64_t writebacks, writeback_bytes, deferred, promoted, free_blocks, min_free_blocks, rereads;
  uint64_t discards;
} ss_exclusive_stats;
SS_API ss_status ss_stats_exclusive_sized(const ss_ctx* c, ss_exclusive_stats* out, uint32_t size);
static inline ss_status ss_stats_exclusive(const ss_ctx* c, ss_exclusive_stats* out) {
  return ss_stats_exclusive_sized(c, out, (uint32_t)sizeof *out);
}

#define SS_HAVE_STATS_SNAPSHOT 1
#define SS_SNAPSHOT_READAHEAD 1u
#define SS_SNAPSHOT_EXCLUSIVE 2u
typedef struct ss_snapshot_info {
  uint32_t struct_size;
  uint32_t flags;
  uint64_t sequence;
  uint64_t forwards;
  uint64_t readahead_buffers, readahead_buffer_bytes, readahead_requested, readahead_read, readahead_landed;
  uint64_t readahead_unused, readahead_failed, readahead_fallback, readahead_bytes;
  uint64_t exclusive_writebacks, exclusive_writeback_bytes, exclusive_deferred, exclusive_promoted;
  uint64_t exclusive_free_blocks, exclusive_min_free_blocks, exclusive_rereads, exclusive_blocks;
  uint64_t exclusive_discards;
} ss_snapshot_info;
SS_API ss_status ss_stats_snapshot_sized(const ss_ctx* c, ss_layer_stats* total_out, ss_snapshot_info* info_out,
                                         uint32_t info_size);
static inline ss_status ss_stats_snapshot(const ss_ctx* c, ss_layer_stats* total_out, ss_snapshot_info* info_out) {
  return ss_stats_snapshot_sized(c, total_out, info_out, (uint32_t)sizeof *info_out);
}
SS_API ss_status ss_stats_snapshot_json(const ss_ctx* c, char** out_json, size_t* out_len);

/* ---- Device-gated decode ----
 * Per token, captured in the engine's graph: ss_dg_enqueue_begin; for each gated layer g in order:
 * ss_dg_enqueue_export(g, ids), work that does not read g's slots, ss_dg_enqueue_wait(g), then readers that resolve
 * every id through ss_dg_slot; optionally ss_dg_enqueue_predict(g, ids of g + 1); ss_dg_enqueue_end after every
 * reader. On the host: ss_begin before launching the step, ss_end after it. Unit (g, u) lives at
 * parts[p].base + slot * parts[p].stride with slot = slot_of[unit_base[g] + u]. */
#define SS_DG_MAX_PARTS 4
#define SS_DG_MAX_IDS 64
#define SS_DG_PROTOCOL 1
typedef struct ss_dg_part {
  void* base;       /* device array of this part, `slots` entries */
  uint64_t stride;  /* bytes between slots (== bytes) */
  uint64_t bytes;
} ss_dg_part;
typedef struct ss_dg_device_view { /* passed by value to engine kernels; pointers fixed for the context's life */
  uint32_t struct_size, protocol;
  uint32_t n_gated, n_parts, guard_slot, slots;
  const int32_t* slot_of;    /* device: unit_base[n_gated] entries */
  const uint32_t* unit_base; /* device: n_gated + 1 entries */
  const uint32_t* abort;     /* device word, sticky per token */
  ss_dg_part parts[SS_DG_MAX_PARTS];
  uint32_t* absent_err;      /* device word set by a lookup that met an absent entry */
} ss_dg_device_view;
typedef struct ss_dg_unit {
  int32_t gated, unit;
} ss_dg_unit;
SS_API ss_status ss_dg_get_device_view_sized(const ss_ctx* c, ss_dg_device_view* out, uint32_t size);
static inline ss_status ss_dg_get_device_view(const ss_ctx* c, ss_dg_device_view* out) {
  return ss_dg_get_device_view_sized(c, out, (uint32_t)sizeof *out);
}
SS_API int ss_dg_gated_index(const ss_ctx* c, int layer);
SS_API ss_status ss_dg_enqueue_begin(ss_ctx* c, void* stream);
SS_API ss_status ss_dg_enqueue_export(ss_ctx* c, int g, const int32_t* ids_dev, int n, int n_pred, void* stream);
SS_API ss_status ss_dg_enqueue_predict(ss_ctx* c, int g, const int32_t* ids_dev, int n, void* stream);
SS_API ss_status ss_dg_enqueue_wait(ss_ctx* c, int g, void* stream);
SS_API ss_status ss_dg_enqueue_end(ss_ctx* c, void* stream);
SS_API ss_status ss_dg_keep(ss_ctx* c, int g, const int32_t* ids, int n);
#define SS_DG_SET_SCHED 1
#define SS_DG_RESIDENCY 1
SS_API ss_status ss_dg_residency(ss_ctx* c, ss_dg_unit* out, uint32_t cap, uint32_t* total);
SS_API ss_status ss_dg_set_sched(ss_ctx* c, uint32_t wb_defer, uint32_t flush_ready);
SS_API ss_status ss_dg_set_budgets(ss_ctx* c, uint32_t spare_target, uint32_t prefetch_per_layer,
                                   uint32_t prefetch_per_token);
typedef struct ss_dg_layer_timeline {
  uint32_t struct_size, layer;
  double seen_us, demand_us, pred_wait_us, prefetch_us, serve_us;
  uint32_t ids, misses, covered, fetched, prefetched, reserved0;
  double dma_ms;
  uint32_t predicted_true, covered_waits;
  double gpu_wait_us, gpu_export_ready_us, wb_left_ms, dma_first_ms;
} ss_dg_layer_timeline;
SS_API ss_status ss_dg_timeline_sized(const ss_ctx* c, int g, ss_dg_layer_timeline* out, uint32_t size);
typedef struct ss_dg_boundary_timeline {
  uint32_t struct_size, writebacks;
  double sync_us, select_us, upload_us, issue_us;
} ss_dg_boundary_timeline;
SS_API ss_status ss_dg_boundary_timeline_sized(const ss_ctx* c, ss_dg_boundary_timeline* out, uint32_t size);
#define SS_DG_SCORED 1
typedef struct ss_dg_stats {
  uint32_t struct_size, reserved0;
  uint64_t tokens, lookups, misses, covered, fetched, prefetched, prefetch_used, pred_invalid;
  uint64_t resurrected, bank_serves, collected_mid, evicted, evict_short, writebacks_done, stalled;
  uint64_t free_slots, blocks, slots;
  uint64_t predicted, predicted_true, miss_layers, device_timeouts, covered_waits;
  uint64_t wb_deferred, wb_cancelled, wb_forced, wb_boundary_flushed;
  uint64_t wb_issued_bytes, wb_completed_bytes, wb_cancelled_bytes, wb_boundary_flushed_bytes, wb_outstanding_bytes;
  uint64_t wb_forced_wait_ns;
  uint64_t winpf_hints, winpf_hint_rows, prior_issued, prior_used, prior_late, prior_reverted;
  uint64_t l1_candidates, l1_issued, l1_used, l1_late, l1_reverted, l1_priced_out, l1_skipped_ahead;
  uint64_t prior_budget_stops;
  uint64_t score_fallbacks, scored_victims, score_layers, score_candidates, score_saturated, score_ns;
  uint64_t score_deferred, score_last_ns;
  uint64_t disk_reads, disk_read_bytes, disk_read_ns, disk_stage_waits, disk_drops, disk_discards;
  uint64_t inclusive_kept, inclusive_drops, disk_units, backed_units;
  uint64_t disk_wait_ns;
  uint64_t disk_overlapped, disk_max_in_flight, disk_carried, disk_carried_bytes;
  uint64_t resident_units, resident_evicted, resident_bytes, resident_ns;
  uint64_t round_count, round_units, round_bytes, round_ns, round_cancelled;
  uint32_t cuda_module_loading;
  uint32_t reserved1;
  uint64_t clean_drops, clean_drop_bytes;
  uint64_t mkres_file_reads, mkres_file_bytes, mkres_read_ns, mkres_h2d_bytes, mkres_wb_bytes;
  uint64_t lm_tokens, lm_parts, lm_mid_evictions, lm_early_admits;
  uint64_t pf_reverted, pf_revert_bytes;
  uint64_t pred_skipped_ahead, pf_strict_refused;
  uint64_t pred_shadow_file_predicted, pred_shadow_file_demanded, pred_shadow_file_hit;
  uint64_t pred_shadow_file_predicted_bytes, pred_shadow_file_demanded_bytes, pred_shadow_file_hit_bytes;
  uint32_t disk_queue_resolved, disk_locations;
  uint64_t landing_issued, landing_promoted, landing_late, landing_wait_ns, landing_expired, landing_dropped_full;
  uint64_t landing_read_bytes;
  uint64_t landing_cancelled;
  uint64_t landing_expired_layer, landing_skipped_passed;
  uint64_t landing_yields, landing_aborted_bytes;
  uint64_t bank_kept;
  uint32_t disk_depth_active, disk_depth_adapt;
  uint64_t disk_depth_changes, disk_depth_calibrations;
} ss_dg_stats;
SS_API ss_status ss_stats_dg_sized(const ss_ctx* c, ss_dg_stats* out, uint32_t size);
static inline ss_status ss_stats_dg(const ss_ctx* c, ss_dg_stats* out) {
  return ss_stats_dg_sized(c, out, (uint32_t)sizeof *out);
}

/* Window prefetch: not in this build (the functions return SS_E_UNSUPPORTED). */
typedef struct ss_dg_winpf_params ss_dg_winpf_params;
SS_API void ss_dg_winpf_defaults_sized(ss_dg_winpf_params* p, uint32_t size);
SS_API ss_status ss_dg_winpf_set(ss_ctx* c, const ss_dg_winpf_params* p);
SS_API ss_status ss_dg_window_hint(ss_ctx* c, const int32_t* symbols, const float* weights, uint32_t rows);

#if defined(__CUDACC__)
/* The slot engine kernels read exported unit `id` of gated layer g from, after ss_dg_enqueue_wait(g). An aborted
 * token or an id outside the layer gives the zeroed guard slot; an absent entry is reported through absent_err and
 * also gives the guard slot, so every read stays in bounds. */
static __device__ __forceinline__ int32_t ss_dg_slot(const ss_dg_device_view* v, uint32_t g, int32_t id) {
  if (*(volatile const uint32_t*)v->abort) return (int32_t)v->guard_slot;
  const uint32_t first = v->unit_base[g];
  if ((uint32_t)id >= v->unit_base[g + 1] - first) return (int32_t)v->guard_slot;
  const int32_t slot = ((volatile const int32_t*)v->slot_of)[first + (uint32_t)id];
  if (slot >= 0) return slot;
  const uint32_t need = (uint32_t)((const char*)&v->absent_err - (const char*)v) + (uint32_t)sizeof(void*);
  if (need <= v->struct_size && v->absent_err) atomicOr(v->absent_err, 1u);
  return (int32_t)v->guard_slot;
}
/* Before ss_dg_enqueue_wait(g): the slot if its bytes are complete, else -1 (acquire load at system scope). */
static __device__ __forceinline__ int32_t ss_dg_slot_if_ready(const ss_dg_device_view* v, uint32_t g, int32_t id) {
  if (*(volatile const uint32_t*)v->abort) return (int32_t)v->guard_slot;
  const uint32_t first = v->unit_base[g];
  if ((uint32_t)id >= v->unit_base[g + 1] - first) return (int32_t)v->guard_slot;
  int32_t slot;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(slot) : "l"(v->slot_of + first + (uint32_t)id) : "memory");
  return slot >= 0 ? slot : -1;
}
#endif

/* ---- Recipes: not in this build ---- */
typedef struct ss_recipe ss_recipe;
SS_API ss_status ss_recipe_from_text(const char* text, size_t len, const char* origin, ss_recipe** out);
SS_API ss_status ss_recipe_from_file(const char* path, ss_recipe** out);
SS_API void ss_recipe_free(ss_recipe* r);
SS_API ss_status ss_recipe_add_profile(ss_recipe* r, const char* text, size_t len, const char* origin,
                                       const char* identity_json, size_t identity_len);
SS_API ss_status ss_recipe_add_overrides(ss_recipe* r, const char* text, size_t len, const char* origin);
SS_API ss_status ss_recipe_set(ss_recipe* r, const char* path, const char* value, const char* origin);
SS_API ss_status ss_recipe_to_json(const ss_recipe* r, char** out, size_t* len);
SS_API ss_status ss_recipe_explain(const ss_recipe* r, char** out, size_t* len);
SS_API ss_status ss_recipe_match(const ss_recipe* r, const char* probe_json, size_t len, char** out, size_t* olen);
SS_API ss_status ss_recipe_select(const ss_recipe* r, const char* state_json, size_t len, char** out, size_t* olen);
SS_API ss_status ss_recipe_plan(const ss_recipe* r, const char* route, const char* set, int member,
                                const char* device_id, const ss_desc* desc, const double* benefit, size_t n_benefit,
                                const ss_desc* const* ref_descs, const double* const* ref_benefits,
                                const size_t* ref_n_benefits, size_t n_refs, ss_budget* budget, ss_options* options,
                                ss_plan** plan, char** out, size_t* olen);

/* ---- Device-gated between-token calls ---- */
#define SS_DG_RESET_OPEN 1
/* Restores the open placement by moving only misplaced units (slot to slot on the device, block to block on the
 * host); captured device addresses stay valid. Engine thread, between tokens. */
SS_API ss_status ss_dg_reset_open(ss_ctx* c);
#define SS_DG_AUTO_EVICT 1
SS_API ss_status ss_dg_end_rows(ss_ctx* c, uint32_t rows);
#define SS_DG_SET_POLICY 1
SS_API ss_status ss_dg_set_policy(ss_ctx* c, ss_policy policy);

/* ---- Multi-location files, whole-device budgets, device profiles, packs, rounds, layer tokens: not in this
 * build. The types are opaque here; every function returns SS_E_UNSUPPORTED (or does nothing). ---- */
typedef struct ss_mfile ss_mfile;
typedef struct ss_mfile_options ss_mfile_options;
typedef struct ss_mfile_io ss_mfile_io;
typedef struct ss_mfile_counters ss_mfile_counters;
typedef struct ss_mfile_location ss_mfile_location;
SS_API void ss_mfile_options_defaults_sized(ss_mfile_options* o, uint32_t size);
SS_API ss_status ss_mfile_open(const char* primary, const char* weight_dirs, const ss_mfile_options* opt,
                               ss_mfile** out);
SS_API void ss_mfile_close(ss_mfile* f);
SS_API uint64_t ss_mfile_size(const ss_mfile* f);
SS_API uint32_t ss_mfile_alignment(const ss_mfile* f);
SS_API int ss_mfile_multi(const ss_mfile* f);
SS_API ss_status ss_mfile_pread(ss_mfile* f, void* dst, uint64_t bytes, uint64_t offset, uint64_t* got);
SS_API ss_status ss_mfile_preadv(ss_mfile* f, const ss_mfile_io* ios, uint32_t n);
SS_API ss_status ss_mfile_get_counters(const ss_mfile* f, ss_mfile_counters* out);
SS_API const char* ss_mfile_location_path(const ss_mfile* f, int loc);
SS_API const char* ss_mfile_open_report(const ss_mfile* f);
SS_API ss_status ss_mfile_location_info(const ss_mfile* f, uint32_t loc, ss_mfile_location* out);

typedef struct ss_budget_in ss_budget_in;
typedef struct ss_budget_out ss_budget_out;
typedef struct ss_budget_ledger ss_budget_ledger;
typedef struct ss_budget_stats ss_budget_stats;
typedef int ss_budget_kind;
SS_API void ss_budget_in_defaults_sized(ss_budget_in* in, uint32_t size);
SS_API ss_status ss_budget_plan(const ss_budget_in* in, ss_budget_out* out);
SS_API size_t ss_budget_plan_json(const ss_budget_in* in, const ss_budget_out* out, char* buf, size_t len);
SS_API ss_status ss_budget_ledger_create(uint64_t vram_total_bytes, uint64_t ram_total_bytes, ss_budget_ledger** out);
SS_API void ss_budget_ledger_free(ss_budget_ledger* l);
SS_API ss_status ss_budget_ledger_add(ss_budget_ledger* l, ss_budget_kind kind, const char* name, uint64_t bytes);
SS_API ss_status ss_budget_ledger_sub(ss_budget_ledger* l, ss_budget_kind kind, const char* name, uint64_t bytes);
SS_API ss_status ss_budget_ledger_observe_device(ss_budget_ledger* l, uint64_t measured_used_bytes);
SS_API ss_status ss_budget_ledger_stats(const ss_budget_ledger* l, ss_budget_stats* out);
SS_API ss_status ss_budget_ledger_observe(ss_budget_ledger* l, const char* stage, uint64_t device_used_bytes,
                                          uint64_t host_used_bytes);
SS_API int ss_budget_ledger_within_caps(const ss_budget_ledger* l);
SS_API ss_status ss_budget_in_dg_library(ss_budget_in* in, const ss_desc* d, const ss_options* o);

/* Placement rounds (device-gated, between tokens on the engine thread): every gated unit keeps a decayed count of the
 * steps that routed it (s = decay x s + hits since the last round); a round moves units toward the placement that
 * count ranks (the hottest on the device, the next pinned, the rest in their files), at most max_units promotions and
 * budget_bytes bytes (0 = no limit), a unit replacing another only when its count is above hysteresis x the other's.
 * Kept units and units with a write-back in flight never move. ss_dg_round_cancel (any thread) stops a running round
 * at its next unit; ss_dg_round_seed_counts sets counts (finite, >= 0). */
typedef struct ss_dg_round_params {
  uint32_t struct_size;  /* sizeof, set by ss_dg_round_defaults */
  uint32_t flags;        /* 0 */
  uint64_t budget_bytes; /* 0 = no limit */
  uint32_t max_units;    /* promotions per round (default 96) */
  float hysteresis;      /* >= 1 (default 1.25) */
  float decay;           /* 0..1 (default 0.85) */
  uint32_t reserved0;
} ss_dg_round_params;
typedef struct ss_dg_round_result {
  uint32_t struct_size;
  uint32_t promoted_to_device, promoted_to_pinned, demoted_from_device, dropped_to_file;
  uint32_t cancelled;    /* 1: stopped by ss_dg_round_cancel at a unit boundary */
  uint64_t bytes_read, bytes_h2d, bytes_written_back, ns;
} ss_dg_round_result;
SS_API ss_status ss_dg_make_resident(ss_ctx* c, int g, const int32_t* ids, int n);
SS_API void ss_dg_round_defaults_sized(ss_dg_round_params* p, uint32_t size);
SS_API ss_status ss_dg_round_sized(ss_ctx* c, const ss_dg_round_params* p, ss_dg_round_result* out, uint32_t size);
SS_API ss_status ss_dg_round_cancel(ss_ctx* c);
SS_API ss_status ss_dg_round_seed_counts(ss_ctx* c, const ss_dg_unit* units, const float* counts, uint32_t n);

typedef struct ss_devprof ss_devprof;
typedef struct ss_devprof_detect_opts ss_devprof_detect_opts;
typedef struct ss_devprof_info ss_devprof_info;
typedef struct ss_devprof_device ss_devprof_device;
typedef struct ss_devprof_topology_in ss_devprof_topology_in;
typedef struct ss_devprof_topology_out ss_devprof_topology_out;
typedef struct ss_devprof_piece_in ss_devprof_piece_in;
SS_API void ss_devprof_detect_opts_defaults_sized(ss_devprof_detect_opts* o, uint32_t size);
SS_API ss_status ss_devprof_detect(const ss_devprof_detect_opts* o, ss_devprof** out);
SS_API ss_status ss_devprof_from_json(const char* text, size_t len, ss_devprof** out);
SS_API ss_status ss_devprof_merge_json(ss_devprof* p, const char* text, size_t len, const char* origin);
SS_API void ss_devprof_free(ss_devprof* p);
SS_API ss_status ss_devprof_to_json(const ss_devprof* p, char** out, size_t* len);
SS_API ss_status ss_devprof_hash(const ss_devprof* p, char out[17]);
SS_API ss_status ss_devprof_probe_report(const ss_devprof* p, const char* host, char** out, size_t* len);
SS_API ss_status ss_devprof_get(const ss_devprof* p, ss_devprof_info* out);
SS_API ss_status ss_devprof_limit(const ss_devprof* p, const char* key, uint64_t* value);
SS_API ss_status ss_devprof_get_device(const ss_devprof* p, uint32_t i, ss_devprof_device* out);
SS_API ss_status ss_devprof_budget(const ss_devprof* p, uint32_t device, ss_budget_in* in);
SS_API void ss_devprof_topology_in_defaults_sized(ss_devprof_topology_in* in, uint32_t size);
SS_API ss_status ss_devprof_topology(const ss_devprof* const* profiles, uint32_t n_profiles,
                                     const ss_devprof_topology_in* in, ss_devprof_topology_out* out);
SS_API void ss_devprof_piece_in_defaults_sized(ss_devprof_piece_in* in, uint32_t size);
SS_API ss_status ss_devprof_piece_rows(const ss_devprof* p, const ss_devprof_piece_in* in, uint32_t* rows);

typedef struct ss_pack ss_pack;
typedef struct ss_pack_options ss_pack_options;
typedef struct ss_pack_entry ss_pack_entry;
typedef struct ss_pack_segment ss_pack_segment;
typedef struct ss_pack_unit ss_pack_unit;
typedef struct ss_pack_read_req ss_pack_read_req;
typedef struct ss_pack_writer ss_pack_writer;
typedef struct ss_pack_record_spec ss_pack_record_spec;
SS_API void ss_pack_options_defaults_sized(ss_pack_options* o, uint32_t size);
SS_API ss_status ss_pack_open(const char* dir, const ss_pack_options* opt, ss_pack** out);
SS_API void ss_pack_close(ss_pack* p);
SS_API uint64_t ss_pack_records(const ss_pack* p);
SS_API ss_status ss_pack_entry_at_sized(const ss_pack* p, uint64_t index, ss_pack_entry* out, uint32_t size);
SS_API ss_status ss_pack_find_sized(const ss_pack* p, int layer, int expert, const char* name, ss_pack_entry* out,
                                    uint32_t size);
SS_API ss_status ss_pack_segment_at(const ss_pack* p, uint64_t record, uint32_t k, ss_pack_segment* out);
SS_API ss_status ss_pack_unit_find(const ss_pack* p, int layer, int expert, ss_pack_unit* out);
SS_API ss_status ss_pack_read(ss_pack* p, uint64_t record, uint32_t row0, uint32_t row1, void* dst);
SS_API ss_status ss_pack_readv(ss_pack* p, const ss_pack_read_req* reads, uint32_t n);
SS_API ss_status ss_pack_read_unit(ss_pack* p, int layer, int expert, void* dst);
SS_API ss_status ss_pack_dg_descriptor(ss_pack* p, const char* base_json, size_t len, char** out_json,
                                       size_t* out_len);
SS_API uint32_t ss_pack_files(const ss_pack* p);
SS_API int ss_pack_has_layout(const ss_pack* p, const char* layout);
SS_API ss_status ss_pack_file_identity(const ss_pack* p, uint32_t file, ss_file_identity* out);
SS_API ss_status ss_pack_info_json(const ss_pack* p, char** out_json, size_t* out_len);
SS_API ss_status ss_pack_verify_full(ss_pack* p, char** out_json, size_t* out_len);
SS_API ss_status ss_pack_writer_begin(const char* dir, const char* meta_json, size_t len, ss_pack_writer** out);
SS_API ss_status ss_pack_writer_record_begin(ss_pack_writer* w, const ss_pack_record_spec* r);
SS_API ss_status ss_pack_writer_record_write(ss_pack_writer* w, const void* data, uint64_t n);
SS_API ss_status ss_pack_writer_record_end(ss_pack_writer* w);
SS_API ss_status ss_pack_writer_add(ss_pack_writer* w, const ss_pack_record_spec* r, const void* data);
SS_API ss_status ss_pack_writer_finish(ss_pack_writer* w, char* manifest_sha256);
SS_API void ss_pack_writer_abort(ss_pack_writer* w);

SS_API ss_status ss_dg_set_clean_evict(ss_ctx* c, uint32_t on);
SS_API ss_status ss_dg_begin_layer(ss_ctx* c, int g, int parts);
SS_API ss_status ss_dg_enqueue_export_part(ss_ctx* c, int g, int part, const int32_t* ids_dev, int n, void* stream);
SS_API ss_status ss_dg_enqueue_wait_part(ss_ctx* c, int g, int part, void* stream);
SS_API ss_status ss_dg_enqueue_end_layer(ss_ctx* c, void* stream);
SS_API ss_status ss_dg_set_pf_revert_unused(ss_ctx* c, uint32_t on);

#ifdef __cplusplus
}
#endif

#endif /* STRIX_STREAM_SS_H */
