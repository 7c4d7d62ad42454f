"""ctypes view of the C ABI (include/strix_stream/ss.h, include/tierstream/tsb.h) of libtierstream.so.

The structs mirror the header's versioned structs field for field; `load()` opens the in-tree library and declares
every function's argument and result types. The library is the product: when it is missing, `load()` raises
(there is no Python fallback for any of it).
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtierstream.so")
ENGINE_PATH = os.path.join(HERE, "libtsb_engine.so")

SS_OK, SS_E_INVALID, SS_E_DESC, SS_E_IO, SS_E_NOMEM, SS_E_BACKEND, SS_E_CAPACITY, SS_E_HASH, SS_E_UNSUPPORTED = range(9)
STATUS_NAMES = ["SS_OK", "SS_E_INVALID", "SS_E_DESC", "SS_E_IO", "SS_E_NOMEM", "SS_E_BACKEND", "SS_E_CAPACITY",
                "SS_E_HASH", "SS_E_UNSUPPORTED", "SS_E_RECIPE"]
SS_TIER_RESIDENT, SS_TIER_PINNED, SS_TIER_DISK, SS_TIER_PAIR, SS_TIER_RESIDENT_BACKED = range(5)
SS_POLICY_LRU, SS_POLICY_SCORED, SS_POLICY_SCORED_AUTO = range(3)
SS_TIER_MODE_INCLUSIVE, SS_TIER_MODE_EXCLUSIVE = 0, 1
SS_BACKEND_CPU, SS_BACKEND_CUDA, SS_BACKEND_HIP = 0, 1, 2
SS_FORWARD_HOST, SS_FORWARD_DEVICE_GATED = 0, 1
SS_DG_MAX_PARTS = 4

u32, u64, i32, i64, dbl = C.c_uint32, C.c_uint64, C.c_int32, C.c_int64, C.c_double
vp = C.c_void_p


class ss_budget(C.Structure):
    _fields_ = [("struct_size", u32), ("device_bytes", u64), ("host_pinned_bytes", u64), ("workspace_bytes", u64),
                ("margin_gib", dbl), ("margin_fraction", dbl), ("dynamic_slots_per_layer", u32), ("ring_slots", u32),
                ("pinned_backing", C.c_int), ("reserved0", u32), ("tier_mode", C.c_int), ("host_spare_units", u32)]


_OPT = [("struct_size", u32), ("backend", C.c_int), ("device", C.c_int), ("policy", C.c_int),
        ("lookahead_budget", u32), ("reader_threads", u32), ("staging_buffers", u32), ("staging_bytes", u64),
        ("copy_piece_bytes", u64), ("verify_hash", C.c_int), ("fill_residents", C.c_int), ("score_window", u32),
        ("pin_planned", C.c_int), ("direct_io", C.c_int), ("group_units", u32), ("spec_persistent", C.c_int),
        ("reserved0", u32), ("readahead_units", u32), ("reserved1", u32), ("forward_mode", C.c_int),
        ("dg_max_ids", u32), ("dg_prefetch_reserve", u32), ("dg_prefetch_per_layer", u32),
        ("dg_prefetch_per_token", u32), ("dg_wait_timeout_ms", u32), ("dg_service_boost", u32), ("dg_diag", u32),
        ("dg_test_hooks", u32), ("dg_spare_target", u32), ("dg_seed_n", u32), ("dg_seed", vp),
        ("dg_spare_slots", u32), ("dg_flush_ready", u32), ("dg_wb_defer", u32), ("dg_wb_stream", u32),
        ("dg_wb_layer_bytes", u32), ("dg_wb_max_outstanding", u32), ("dg_prior_len", u64), ("dg_prior", vp),
        ("exclusive_discard", u32), ("reserved2", u32), ("dg_score_w_trans", u32), ("dg_score_w_freq", u32),
        ("dg_score_w_recency", u32), ("reserved3", u32), ("dg_score_profile_len", u64), ("dg_score_profile", vp),
        ("weight_dirs", C.c_char_p), ("drive_readers", u32), ("weight_verify", C.c_int), ("dg_disk_tier", u32),
        ("dg_disk_prefetch", u32), ("dg_disk_staging", u32), ("dg_inclusive_blocks", u32), ("dg_disk_queue", u32),
        ("reserved4", u32), ("source_identity_n", u32), ("reserved5", u32), ("source_identities", vp),
        ("budget", vp), ("dg_no_admit", u32), ("reserved6", u32), ("dg_clean_evict", u32), ("reserved7", u32),
        ("dg_pf_revert_unused", u32), ("reserved8", u32), ("dg_pf_strict_admit", u32), ("reserved9", u32),
        ("dg_landing_blocks", u32), ("dg_landing_max_queued", u32), ("dg_landing_ttl", u32), ("reserved10", u32),
        ("dg_landing_chunk", u32), ("reserved11", u32), ("dg_bank_keep", u32), ("reserved12", u32),
        ("dg_disk_queue_adapt", u32), ("reserved13", u32)]


class ss_options(C.Structure):
    _fields_ = _OPT


class ss_plan_totals(C.Structure):
    _fields_ = [(n, u64) for n in ("fixed_bytes", "margin_bytes", "resident_bytes", "dynamic_bytes", "ring_bytes",
                                   "peak_device_bytes", "pinned_bytes", "disk_bytes", "n_resident", "n_pinned",
                                   "n_disk")]


class ss_layer_stats(C.Structure):
    _fields_ = [(n, u64) for n in ("routed", "hits", "admitted", "transient", "evicted", "prefetched", "spec_issued",
                                   "spec_used", "spec_dropped", "bytes_pinned", "bytes_disk", "wait_ns")]


class ss_group(C.Structure):
    _fields_ = [("units", C.POINTER(i32)), ("n_units", C.c_int)]


class ss_layer_view(C.Structure):
    _fields_ = [("table_dev", C.POINTER(u64)), ("table_host", C.POINTER(u64)), ("n_units", C.c_int),
                ("groups", C.POINTER(ss_group)), ("n_groups", C.c_int)]


class ss_exclusive_stats(C.Structure):
    _fields_ = [("struct_size", u32)] + [(n, u64) for n in (
        "writebacks", "writeback_bytes", "deferred", "promoted", "free_blocks", "min_free_blocks", "rereads",
        "discards")]


class ss_dg_part(C.Structure):
    _fields_ = [("base", vp), ("stride", u64), ("bytes", u64)]


class ss_dg_device_view(C.Structure):
    _fields_ = [("struct_size", u32), ("protocol", u32), ("n_gated", u32), ("n_parts", u32), ("guard_slot", u32),
                ("slots", u32), ("slot_of", vp), ("unit_base", vp), ("abort", vp),
                ("parts", ss_dg_part * SS_DG_MAX_PARTS), ("absent_err", vp)]


class ss_dg_unit(C.Structure):
    _fields_ = [("gated", i32), ("unit", i32)]


class ss_dg_layer_timeline(C.Structure):
    _fields_ = [("struct_size", u32), ("layer", u32), ("seen_us", dbl), ("demand_us", dbl), ("pred_wait_us", dbl),
                ("prefetch_us", dbl), ("serve_us", dbl), ("ids", u32), ("misses", u32), ("covered", u32),
                ("fetched", u32), ("prefetched", u32), ("reserved0", u32), ("dma_ms", dbl), ("predicted_true", u32),
                ("covered_waits", u32), ("gpu_wait_us", dbl), ("gpu_export_ready_us", dbl), ("wb_left_ms", dbl),
                ("dma_first_ms", dbl)]


class ss_dg_boundary_timeline(C.Structure):
    _fields_ = [("struct_size", u32), ("writebacks", u32), ("sync_us", dbl), ("select_us", dbl), ("upload_us", dbl),
                ("issue_us", dbl)]


_DG_STATS_U64_1 = ["tokens", "lookups", "misses", "covered", "fetched", "prefetched", "prefetch_used", "pred_invalid",
                   "resurrected", "bank_serves", "collected_mid", "evicted", "evict_short", "writebacks_done",
                   "stalled", "free_slots", "blocks", "slots", "predicted", "predicted_true", "miss_layers",
                   "device_timeouts", "covered_waits", "wb_deferred", "wb_cancelled", "wb_forced",
                   "wb_boundary_flushed", "wb_issued_bytes", "wb_completed_bytes", "wb_cancelled_bytes",
                   "wb_boundary_flushed_bytes", "wb_outstanding_bytes", "wb_forced_wait_ns",
                   "winpf_hints", "winpf_hint_rows", "prior_issued", "prior_used", "prior_late", "prior_reverted",
                   "l1_candidates", "l1_issued", "l1_used", "l1_late", "l1_reverted", "l1_priced_out",
                   "l1_skipped_ahead", "prior_budget_stops", "score_fallbacks", "scored_victims", "score_layers",
                   "score_candidates", "score_saturated", "score_ns", "score_deferred", "score_last_ns",
                   "disk_reads", "disk_read_bytes", "disk_read_ns", "disk_stage_waits", "disk_drops", "disk_discards",
                   "inclusive_kept", "inclusive_drops", "disk_units", "backed_units", "disk_wait_ns",
                   "disk_overlapped", "disk_max_in_flight", "disk_carried", "disk_carried_bytes",
                   "resident_units", "resident_evicted", "resident_bytes", "resident_ns", "round_count",
                   "round_units", "round_bytes", "round_ns", "round_cancelled"]


class ss_dg_stats(C.Structure):
    """The leading fields of ss_dg_stats (a versioned struct: the library writes min(size, its own) bytes)."""
    _fields_ = [("struct_size", u32), ("reserved0", u32)] + [(n, u64) for n in _DG_STATS_U64_1]


class dg_replay_config(C.Structure):
    """tsb_dg_replay_config and the reference harness's oref_dg_config (the same layout)."""
    _fields_ = [("n_gated", u32), ("n_units", C.POINTER(u32)), ("n_parts", u32), ("part_bytes", C.POINTER(u64)),
                ("persistent_slots", u32), ("bank_slots", u32), ("blocks", u32), ("spare_target", u32),
                ("prefetch_reserve", u32), ("prefetch_per_layer", u32), ("prefetch_per_token", u32),
                ("wb_defer", u32), ("wb_on_d2h", u32), ("wb_layer_bytes", u64), ("wb_max_outstanding", u64),
                ("n_order", u32), ("order", C.POINTER(u32)), ("tokens", u32), ("n_ids", u32), ("n_pred", u32),
                ("move_bytes", u32), ("inclusive", u32), ("disk_tier", u32), ("disk_prefetch", u32),
                ("home_blocks", u32), ("disk_staging", u32), ("disk", C.POINTER(C.c_uint8)),
                ("xstats", C.POINTER(u64)), ("reset_at", u32), ("bank_keep", u32), ("policy", u32), ("rows", u32),
                ("w_trans", u32), ("w_freq", u32), ("w_rec", u32), ("reserved2", u32),
                ("profile", C.POINTER(u32)), ("round_every", u32), ("round_max_units", u32),
                ("round_hysteresis", C.c_float), ("round_decay", C.c_float), ("round_budget", u64),
                ("rstats", C.POINTER(u64)), ("no_admit", u32), ("clean_evict", u32), ("pf_revert", u32),
                ("pf_strict", u32), ("pstats", C.POINTER(u64)), ("disk_queue", u32), ("reserved3", u32),
                ("qstats", C.POINTER(u64)), ("mr_n", u32), ("reserved4", u32), ("mr_token", C.POINTER(u32)),
                ("mr_layer", C.POINTER(u32)), ("mr_count", C.POINTER(u32)), ("mr_ids", C.POINTER(u32)),
                ("mstats", C.POINTER(u64)), ("sstats", C.POINTER(u64)), ("kstats", C.POINTER(u64)),
                ("landing_blocks", u32), ("landing_ttl", u32), ("lstats", C.POINTER(u64))]


class ss_dg_round_params(C.Structure):
    _fields_ = [("struct_size", u32), ("flags", u32), ("budget_bytes", u64), ("max_units", u32),
                ("hysteresis", C.c_float), ("decay", C.c_float), ("reserved0", u32)]


class ss_dg_round_result(C.Structure):
    _fields_ = [("struct_size", u32), ("promoted_to_device", u32), ("promoted_to_pinned", u32),
                ("demoted_from_device", u32), ("dropped_to_file", u32), ("cancelled", u32), ("bytes_read", u64),
                ("bytes_h2d", u64), ("bytes_written_back", u64), ("ns", u64)]


class tsb_peer_tier(C.Structure):
    """tsb_peer_tier (include/tierstream/tsb.h): the peer tier's owners and store addresses for tsb_open_peer."""
    _fields_ = [("struct_size", u32), ("world", u32), ("rank", C.c_int32), ("keys", u32),
                ("owner", C.POINTER(C.c_int32)), ("store_base", C.POINTER(vp)), ("copy", u32), ("layout", u32)]


PEER_WHOLE_UNITS, PEER_STRIPED = 0, 1


PEER_HANDLE_BYTES = 64

P = C.POINTER
_PROTOS = {
    "ss_last_error": (C.c_char_p, []),
    "ss_abi_version": (C.c_int, []),
    "ss_desc_from_json": (C.c_int, [C.c_char_p, C.c_size_t, P(vp)]),
    "ss_desc_from_file": (C.c_int, [C.c_char_p, P(vp)]),
    "ss_desc_free": (None, [vp]),
    "ss_desc_n_layers": (C.c_int, [vp]),
    "ss_desc_layer_units": (C.c_int, [vp, C.c_int]),
    "ss_desc_unit_bytes": (u64, [vp, C.c_int]),
    "ss_desc_to_json": (C.c_int, [vp, P(vp), P(C.c_size_t)]),
    "ss_desc_unit_index": (i64, [vp, C.c_int, C.c_int]),
    "ss_desc_total_units": (i64, [vp]),
    "ss_free": (None, [vp]),
    "ss_budget_defaults_sized": (None, [P(ss_budget), u32]),
    "ss_plan_make": (C.c_int, [vp, P(ss_budget), P(dbl), C.c_size_t, P(vp)]),
    "ss_plan_from_tiers": (C.c_int, [vp, P(ss_budget), P(C.c_uint8), C.c_size_t, P(vp)]),
    "ss_plan_from_json": (C.c_int, [vp, P(ss_budget), C.c_char_p, C.c_size_t, P(vp)]),
    "ss_plan_free": (None, [vp]),
    "ss_plan_unit_tier": (C.c_int, [vp, C.c_int, C.c_int]),
    "ss_plan_get_totals": (None, [vp, P(ss_plan_totals)]),
    "ss_plan_to_json": (C.c_int, [vp, P(vp), P(C.c_size_t)]),
    "ss_options_defaults_sized": (None, [P(ss_options), u32]),
    "ss_open": (C.c_int, [vp, P(ss_budget), vp, P(ss_options), P(vp)]),
    "ss_close": (None, [vp]),
    "ss_begin": (C.c_int, [vp, P(u32), C.c_int]),
    "ss_end": (C.c_int, [vp]),
    "ss_layer_routes": (C.c_int, [vp, C.c_int, P(i32), C.c_int]),
    "ss_layer_all": (C.c_int, [vp, C.c_int]),
    "ss_prefetch": (C.c_int, [vp, C.c_int, P(C.c_int32), C.c_int, C.c_int]),
    "ss_prefetch_layer": (C.c_int, [vp, C.c_int]),
    "ss_host_prefetch": (C.c_int, [vp, C.c_int, P(C.c_int32), C.c_int]),
    "ss_host_prefetch_layer": (C.c_int, [vp, C.c_int]),
    "ss_acquire": (C.c_int, [vp, C.c_int, vp, P(ss_layer_view)]),
    "ss_acquire_groups": (C.c_int, [vp, C.c_int, vp, P(ss_layer_view)]),
    "ss_group_wait": (C.c_int, [vp, C.c_int, C.c_int, vp]),
    "ss_release": (C.c_int, [vp, C.c_int, vp]),
    "ss_check_unit": (C.c_int, [vp, C.c_int, C.c_int]),
    "ss_seed": (C.c_int, [vp, C.c_int, P(i32), C.c_int]),
    "ss_stats_layer": (C.c_int, [vp, C.c_int, P(ss_layer_stats)]),
    "ss_stats_total": (C.c_int, [vp, P(ss_layer_stats)]),
    "ss_stats_reset": (None, [vp]),
    "ss_stats_to_json": (C.c_int, [vp, P(vp), P(C.c_size_t)]),
    "ss_stats_exclusive_sized": (C.c_int, [vp, P(ss_exclusive_stats), u32]),
    "ss_stats_dg_sized": (C.c_int, [vp, P(ss_dg_stats), u32]),
    "ss_dg_get_device_view_sized": (C.c_int, [vp, P(ss_dg_device_view), u32]),
    "ss_dg_gated_index": (C.c_int, [vp, C.c_int]),
    "ss_dg_enqueue_begin": (C.c_int, [vp, vp]),
    "ss_dg_enqueue_export": (C.c_int, [vp, C.c_int, vp, C.c_int, C.c_int, vp]),
    "ss_dg_enqueue_predict": (C.c_int, [vp, C.c_int, vp, C.c_int, vp]),
    "ss_dg_enqueue_wait": (C.c_int, [vp, C.c_int, vp]),
    "ss_dg_enqueue_end": (C.c_int, [vp, vp]),
    "ss_dg_keep": (C.c_int, [vp, C.c_int, P(i32), C.c_int]),
    "ss_dg_make_resident": (C.c_int, [vp, C.c_int, P(i32), C.c_int]),
    "ss_dg_residency": (C.c_int, [vp, P(ss_dg_unit), u32, P(u32)]),
    "ss_dg_set_sched": (C.c_int, [vp, u32, u32]),
    "ss_dg_set_budgets": (C.c_int, [vp, u32, u32, u32]),
    "ss_dg_timeline_sized": (C.c_int, [vp, C.c_int, P(ss_dg_layer_timeline), u32]),
    "ss_dg_boundary_timeline_sized": (C.c_int, [vp, P(ss_dg_boundary_timeline), u32]),
    "ss_dg_reset_open": (C.c_int, [vp]),
    "ss_dg_set_policy": (C.c_int, [vp, C.c_int]),
    "ss_dg_round_defaults_sized": (None, [P(ss_dg_round_params), u32]),
    "ss_dg_round_sized": (C.c_int, [vp, P(ss_dg_round_params), P(ss_dg_round_result), u32]),
    "ss_dg_round_cancel": (C.c_int, [vp]),
    "ss_dg_round_seed_counts": (C.c_int, [vp, vp, P(C.c_float), u32]),
    "ss_test_dg_check": (C.c_int, [vp]),
    "ss_test_dg_flags": (C.c_int, [vp, u32]),
    "ss_test_dg_pressure": (C.c_int, [vp, u32, u32]),
    "ss_test_dg_mutate": (C.c_int, [vp, C.c_int]),
    "ss_test_dg_stop_service": (C.c_int, [vp]),
    "tsb_land": (C.c_int, [P(vp), P(vp), P(u64), u32, vp, P(u32), P(i32), u32, vp, u32, vp, u32, vp]),
    "tsb_move": (C.c_int, [P(vp), P(vp), P(u64), u32, vp, P(u32), P(i32), u32, vp, u32, vp, u32, vp]),
    "tsb_move_timeouts": (C.c_int, []),
    "tsb_test_file_read": (C.c_int, [C.c_char_p, u64, u64, vp, u64, u32, C.c_int]),
    "tsb_test_sha256": (C.c_int, [vp, u64, vp]),
    "tsb_test_dg_layout": (C.c_int, [vp, vp, P(ss_options), P(u64), u32, vp, u32]),
    "tsb_test_async_reads": (C.c_int, [C.c_char_p, P(u64), u32, u64, vp, u32, C.c_int]),
    "tsb_test_dg_async_replay": (C.c_int, [C.c_void_p, vp, vp, vp, u32, u32, C.c_int32, P(u64), P(u64)]),
    "tsb_test_read_ahead": (C.c_int, [C.c_char_p, P(u64), u32, u64, u32, u32, u32, P(C.c_int32), u32, P(u64),
                                      P(C.c_int32), P(u64)]),
    "tsb_test_load": (C.c_int, [C.c_char_p, P(u64), P(C.c_int32), u32, u64, vp, vp, u32, u64, u32, C.c_int, u32,
                                C.c_int32, P(u64)]),
    "tsb_test_resident_replay": (C.c_int, [C.c_int32, C.c_int32, C.c_int32, u32, vp, vp, u32, u32, vp, u32, vp, vp,
                                           vp, vp, vp]),
    "tsb_test_score_profile": (C.c_int, [vp, vp, u64, vp, vp, u64]),
    "tsb_xxh64_units": (C.c_int, [P(vp), P(u64), P(u32), u32, vp, vp, vp, vp, vp]),
    "tsb_xxh64_units_static": (C.c_int, [P(vp), P(u64), P(u32), u32, vp, vp, vp, vp]),
    "tsb_peer_plan": (C.c_int, [P(u64), u32, u32, P(u64), P(C.c_int32)]),
    "tsb_peer_index": (C.c_int, [P(C.c_int32), u32, u32, P(i64), P(u64)]),
    "tsb_peer_store_create": (C.c_int, [vp, P(C.c_int32), u32, C.c_int32, C.c_int, C.c_int, P(vp)]),
    "tsb_peer_store_alloc": (C.c_int, [vp, P(C.c_int32), u32, C.c_int32, C.c_int, P(vp)]),
    "tsb_peer_stripe_bytes": (u64, [u64, u32]),
    "tsb_peer_store_create_striped": (C.c_int, [vp, P(C.c_int32), u32, C.c_int32, u32, C.c_int, C.c_int, P(vp)]),
    "tsb_peer_tier_verify": (C.c_int, [vp, P(tsb_peer_tier), C.c_int, P(u64)]),
    "tsb_peer_store_free": (None, [vp]),
    "tsb_peer_store_base": (vp, [vp]),
    "tsb_peer_store_bytes": (u64, [vp]),
    "tsb_peer_store_export": (C.c_int, [vp, vp]),
    "tsb_peer_map": (C.c_int, [vp, C.c_int, P(vp)]),
    "tsb_peer_unmap": (C.c_int, [vp]),
    "tsb_open_peer": (C.c_int, [vp, P(ss_budget), vp, P(ss_options), P(tsb_peer_tier), P(vp)]),
    "tsb_peer_store_migrate": (C.c_int, [vp, P(C.c_int32), P(vp), u32, u32, vp, P(u64), P(u64), P(u64)]),
    "tsb_dg_peer_retier": (C.c_int, [vp, P(tsb_peer_tier)]),
    "tsb_test_dg_replay": (C.c_int, [P(dg_replay_config), P(i32), P(i32), P(i32), P(u64), P(C.c_uint8), P(u64)]),
    "tsb_test_dg_table": (C.c_int, [vp, P(i32), u32]),
    "tsb_test_dg_corrupt": (C.c_int, [vp, C.c_int, C.c_int, u64]),
    "tsb_xxh64": (u64, [vp, C.c_size_t, u64]),
    "tsb_test_host_locs": (C.c_int, [vp, C.c_int, P(i32), C.c_int]),
    "tsb_test_host_unit": (C.c_int, [vp, C.c_int, C.c_int, P(vp), P(vp)]),
    "ss_layer_routes_dev": (C.c_int, [vp, C.c_int, vp, C.c_int, vp]),
    "tsb_cuda_arch": (C.c_int, []),
}

_ENGINE_PROTOS = {
    "tse_capture_token": (C.c_int, [vp, u32, vp, u32, vp, u32, vp, u32, C.c_int, C.c_int, vp, P(vp), vp]),
    "tse_launch": (C.c_int, [vp, vp]),
    "tse_destroy": (C.c_int, [vp]),
    "tse_read_units": (C.c_int, [vp, u32, vp, u32, vp, u32, C.c_int, vp]),
    "tse_fill_bytes": (None, [u64, u64, u64, vp, u32]),
    "tse_fill_units_device": (C.c_int, [u64, P(u64), u32, u64, vp, vp]),
    "tse_read_table": (C.c_int, [vp, vp, u32, u64, vp, u32, vp]),
    "tse_read_table16": (C.c_int, [vp, vp, u32, u64, vp, u32, C.c_int, vp]),
    "tse_host_forward": (C.c_int, [vp, vp, vp, u32, vp, vp, vp, u32, C.c_int, vp]),
    "tse_expect_sums": (C.c_int, [u64, vp, u32, u64, C.c_int, vp, u32, vp]),
}

_lib = None
_engine = None


class TsError(RuntimeError):
    """A failed ss_* / tsb_* call: the status and the library's message."""

    def __init__(self, status, message):
        name = STATUS_NAMES[status] if 0 <= status < len(STATUS_NAMES) else str(status)
        super().__init__("%s: %s" % (name, message))
        self.status = status


def _declare(lib, protos):
    for name, (res, args) in protos.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    return lib


def load():
    """The in-tree libtierstream.so (raises when it is not built: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError("libtierstream.so is not built (%s): run __graft_entry__.build()" % LIB_PATH)
        _lib = _declare(C.CDLL(LIB_PATH), _PROTOS)
    return _lib


def load_engine():
    """The decode-step stand-in (libtsb_engine.so) the tests and the bench drive the ABI with."""
    global _engine
    if _engine is None:
        load()
        if not os.path.exists(ENGINE_PATH):
            raise RuntimeError("libtsb_engine.so is not built (%s)" % ENGINE_PATH)
        _engine = _declare(C.CDLL(ENGINE_PATH), _ENGINE_PROTOS)
    return _engine


def check(status):
    """Raises TsError for a non-OK ss_status."""
    if status != SS_OK:
        raise TsError(status, load().ss_last_error().decode(errors="replace"))
    return status


def budget_defaults():
    b = ss_budget()
    load().ss_budget_defaults_sized(C.byref(b), C.sizeof(b))
    return b


def options_defaults():
    o = ss_options()
    load().ss_options_defaults_sized(C.byref(o), C.sizeof(o))
    return o


def take_text(ptr, n):
    """A malloc'd library string (freed with ss_free)."""
    s = C.string_at(ptr, n).decode()
    load().ss_free(ptr)
    return s
