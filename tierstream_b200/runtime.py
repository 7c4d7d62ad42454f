"""Python handles over the C ABI, in the reference's vocabulary: a descriptor, a plan, a context.

These are thin owners of the library's opaque handles (ss_desc*, ss_plan*, ss_ctx*); every operation is the C call.
"""
import ctypes as C

import numpy as np

from . import abi


class Desc:
    def __init__(self, json_text):
        lib = abi.load()
        self.h = C.c_void_p()
        raw = json_text.encode()
        abi.check(lib.ss_desc_from_json(raw, len(raw), C.byref(self.h)))

    def __del__(self):
        if getattr(self, "h", None):
            abi.load().ss_desc_free(self.h)
            self.h = None

    @property
    def n_layers(self):
        return abi.load().ss_desc_n_layers(self.h)

    def layer_units(self, layer):
        return abi.load().ss_desc_layer_units(self.h, layer)

    def total_units(self):
        return abi.load().ss_desc_total_units(self.h)

    def to_json(self):
        p, n = C.c_void_p(), C.c_size_t()
        abi.check(abi.load().ss_desc_to_json(self.h, C.byref(p), C.byref(n)))
        return abi.take_text(p, n.value)


class Plan:
    def __init__(self, desc, budget, tiers=None, benefit=None):
        lib = abi.load()
        self.desc = desc
        self.budget = budget
        self.h = C.c_void_p()
        if tiers is not None:
            t = (C.c_uint8 * len(tiers))(*tiers)
            abi.check(lib.ss_plan_from_tiers(desc.h, C.byref(budget), t, len(tiers), C.byref(self.h)))
        else:
            b = (C.c_double * len(benefit))(*benefit) if benefit is not None else None
            abi.check(lib.ss_plan_make(desc.h, C.byref(budget), b, len(benefit) if benefit is not None else 0,
                                       C.byref(self.h)))

    def __del__(self):
        if getattr(self, "h", None):
            abi.load().ss_plan_free(self.h)
            self.h = None

    def to_json(self):
        p, n = C.c_void_p(), C.c_size_t()
        abi.check(abi.load().ss_plan_to_json(self.h, C.byref(p), C.byref(n)))
        return abi.take_text(p, n.value)

    def totals(self):
        t = abi.ss_plan_totals()
        abi.load().ss_plan_get_totals(self.h, C.byref(t))
        return {n: getattr(t, n) for n, _ in t._fields_}


class DgContext:
    """A device-gated context (ss_open with forward_mode = SS_FORWARD_DEVICE_GATED; tsb_open_peer with a peer.Tier,
    whose stores stay allocated and mapped until close())."""

    def __init__(self, desc, plan, options, peer=None):
        lib = abi.load()
        self.desc, self.plan, self.peer = desc, plan, peer
        self.h = C.c_void_p()
        if peer is None:
            abi.check(lib.ss_open(desc.h, C.byref(plan.budget), plan.h, C.byref(options), C.byref(self.h)))
        else:
            t = peer.struct()
            abi.check(lib.tsb_open_peer(desc.h, C.byref(plan.budget), plan.h, C.byref(options), C.byref(t),
                                        C.byref(self.h)))

    def close(self):
        if getattr(self, "h", None):
            abi.load().ss_close(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def begin(self):
        abi.check(abi.load().ss_begin(self.h, None, 0))

    def end(self):
        abi.check(abi.load().ss_end(self.h))

    def view(self):
        v = abi.ss_dg_device_view()
        abi.check(abi.load().ss_dg_get_device_view_sized(self.h, C.byref(v), C.sizeof(v)))
        return v

    def stats(self):
        s = abi.ss_dg_stats()
        abi.check(abi.load().ss_stats_dg_sized(self.h, C.byref(s), C.sizeof(s)))
        return {n: getattr(s, n) for n, _ in s._fields_}

    def stats_json(self):
        p, n = C.c_void_p(), C.c_size_t()
        abi.check(abi.load().ss_stats_to_json(self.h, C.byref(p), C.byref(n)))
        return abi.take_text(p, n.value)

    def make_resident(self, g, ids):
        """ss_dg_make_resident: gated layer g's units `ids` on the device and kept there (not exported while held);
        no ids releases the layer."""
        a = np.ascontiguousarray(ids, dtype=np.int32)
        abi.check(abi.load().ss_dg_make_resident(self.h, g, a.ctypes.data_as(C.POINTER(C.c_int32)) if a.size else None,
                                                 a.size))

    def table(self, keys):
        out = np.empty(keys, dtype=np.int32)
        abi.check(abi.load().tsb_test_dg_table(self.h, out.ctypes.data_as(C.POINTER(C.c_int32)), keys))
        return out

    def check(self):
        abi.check(abi.load().ss_test_dg_check(self.h))

    def check_unit(self, layer, unit):
        abi.check(abi.load().ss_check_unit(self.h, layer, unit))

    def residency(self, cap):
        out = (abi.ss_dg_unit * cap)()
        total = C.c_uint32()
        abi.check(abi.load().ss_dg_residency(self.h, out, cap, C.byref(total)))
        return [(out[i].gated, out[i].unit) for i in range(min(cap, total.value))], total.value

    def reset_open(self):
        abi.check(abi.load().ss_dg_reset_open(self.h))

    def round(self, **params):
        """One placement round between tokens (ss_dg_round): params override the defaults (budget_bytes, max_units,
        hysteresis, decay); returns the result's fields."""
        p = abi.ss_dg_round_params()
        abi.load().ss_dg_round_defaults_sized(C.byref(p), C.sizeof(p))
        for k, v in params.items():
            setattr(p, k, v)
        r = abi.ss_dg_round_result()
        abi.check(abi.load().ss_dg_round_sized(self.h, C.byref(p), C.byref(r), C.sizeof(r)))
        return {n: getattr(r, n) for n, _ in r._fields_ if n != "struct_size"}

    def set_policy(self, policy):
        """Between tokens: SS_POLICY_LRU / SCORED / SCORED_AUTO (ss_dg_set_policy)."""
        abi.check(abi.load().ss_dg_set_policy(self.h, policy))

    def retier(self, tier):
        """Between tokens: the peer tier's owners and store addresses replaced (tsb_dg_peer_retier)."""
        t = tier.struct()
        abi.check(abi.load().tsb_dg_peer_retier(self.h, C.byref(t)))
        self.peer = tier

    def timeline(self, g):
        """The last token's timeline of gated layer g (ss_dg_timeline; -1 where not measured)."""
        t = abi.ss_dg_layer_timeline()
        abi.check(abi.load().ss_dg_timeline_sized(self.h, g, C.byref(t), C.sizeof(t)))
        return {n: getattr(t, n) for n, _ in t._fields_}


class HostContext:
    """A host forward mode context (ss_open with forward_mode = SS_FORWARD_HOST)."""

    def __init__(self, desc, plan, options):
        lib = abi.load()
        self.desc, self.plan = desc, plan
        self.h = C.c_void_p()
        abi.check(lib.ss_open(desc.h, C.byref(plan.budget), plan.h, C.byref(options), C.byref(self.h)))

    def close(self):
        if getattr(self, "h", None):
            abi.load().ss_close(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def begin(self):
        abi.check(abi.load().ss_begin(self.h, None, 0))

    def routes(self, layer, ids):
        a = np.ascontiguousarray(ids, dtype=np.int32)
        abi.check(abi.load().ss_layer_routes(self.h, layer, a.ctypes.data_as(C.POINTER(C.c_int32)), a.size))

    def layer_all(self, layer):
        abi.check(abi.load().ss_layer_all(self.h, layer))

    def prefetch(self, layer, ids, speculative=False):
        a = np.ascontiguousarray(ids, dtype=np.int32)
        abi.check(abi.load().ss_prefetch(self.h, layer, a.ctypes.data_as(C.POINTER(C.c_int32)), a.size,
                                         1 if speculative else 0))

    def prefetch_layer(self, layer):
        abi.check(abi.load().ss_prefetch_layer(self.h, layer))

    def host_prefetch_layer(self, layer):
        """Read-ahead requests for every unit of the layer (ss_host_prefetch_layer)."""
        abi.check(abi.load().ss_host_prefetch_layer(self.h, layer))

    def stats_json(self):
        p, n = C.c_void_p(), C.c_size_t()
        abi.check(abi.load().ss_stats_to_json(self.h, C.byref(p), C.byref(n)))
        return abi.take_text(p, n.value)

    def acquire(self, layer, stream):
        v = abi.ss_layer_view()
        abi.check(abi.load().ss_acquire(self.h, layer, stream, C.byref(v)))
        return v

    def release(self, layer, stream):
        abi.check(abi.load().ss_release(self.h, layer, stream))

    def end(self):
        abi.check(abi.load().ss_end(self.h))

    def locs(self, layer, n_units):
        out = np.empty(2 * n_units, dtype=np.int32)
        abi.check(abi.load().tsb_test_host_locs(self.h, layer, out.ctypes.data_as(C.POINTER(C.c_int32)), n_units))
        return out.reshape(n_units, 2)

    def unit_home(self, layer, unit):
        """(pinned host block address or None, resident device slot address or None) of a unit, between forwards."""
        p, d = C.c_void_p(), C.c_void_p()
        abi.check(abi.load().tsb_test_host_unit(self.h, layer, unit, C.byref(p), C.byref(d)))
        return p.value, d.value

    def layer_stats(self, layer):
        s = abi.ss_layer_stats()
        abi.check(abi.load().ss_stats_layer(self.h, layer, C.byref(s)))
        return {n: getattr(s, n) for n, _ in s._fields_}

    def check_unit(self, layer, unit):
        abi.check(abi.load().ss_check_unit(self.h, layer, unit))

    def exclusive_stats(self):
        x = abi.ss_exclusive_stats()
        abi.check(abi.load().ss_stats_exclusive_sized(self.h, C.byref(x), C.sizeof(x)))
        return [x.writebacks, x.writeback_bytes, x.deferred, x.promoted, x.free_blocks, x.min_free_blocks,
                x.rereads, x.discards]


class TokenGraph:
    """One decode step captured once (libtsb_engine.so): begin, per layer export / wait / reader, end."""

    def __init__(self, ctx, n_gated, ids_dev, n_ids, out_dev, stream, slices=64, mode=0, pred_dev=0, n_pred=0,
                 with_reader=True, held=None):
        eng = abi.load_engine()
        self.exec = C.c_void_p()
        self.stream = stream
        h = (C.c_uint8 * n_gated)(*[1 if x else 0 for x in held]) if held is not None else None
        rc = eng.tse_capture_token(ctx.h, n_gated, ids_dev, n_ids, pred_dev or None, n_pred, out_dev, slices, mode,
                                   1 if with_reader else 0, stream, C.byref(self.exec), h)
        if rc != 0:
            msg = abi.load().ss_last_error().decode(errors="replace") if rc >= 1000 else ""
            raise RuntimeError("tse_capture_token failed: %d %s" % (rc, msg))

    def launch(self):
        rc = abi.load_engine().tse_launch(self.exec, self.stream)
        if rc != 0:
            raise RuntimeError("cudaGraphLaunch failed: %d" % rc)

    def close(self):
        if self.exec:
            abi.load_engine().tse_destroy(self.exec)
            self.exec = C.c_void_p()

    def __del__(self):
        self.close()


def replay_config(n_units, part_bytes, persistent_slots, bank_slots, blocks, spare_target, order, tokens, n_ids,
                  n_pred=0, prefetch_reserve=0xFFFFFFFF, prefetch_per_layer=4, prefetch_per_token=48, wb_defer=1,
                  wb_on_d2h=1, wb_layer_bytes=0, wb_max_outstanding=0, move_bytes=0, inclusive=0, disk=None,
                  home_blocks=0, disk_staging=0, disk_prefetch=0, policy=0, rows=1, weights=None, profile=None,
                  round_every=0, round_max_units=96, round_hysteresis=1.25, round_decay=0.85, round_budget=0,
                  no_admit=0, clean_evict=0, pf_revert=0, pf_strict=0, disk_queue=0, resident_events=(), bank_keep=0,
                  landing_blocks=0, landing_ttl=0):
    """A dg_replay_config with its arrays kept alive on the returned object. disk (file tier): one flag per key for
    the plan's disk units (blocks then counts home_blocks + the spare blocks); xstats is attached by replay().
    policy (scored eviction): 0 LRU, 1 SCORED, 2 SCORED_AUTO, with each boundary's row count `rows`, weights
    (w_trans, w_freq, w_rec) out of 1000 and an optional profile: per gated layer units x units transition counts."""
    c = abi.dg_replay_config()
    keep = {}
    keep["n_units"] = (C.c_uint32 * len(n_units))(*n_units)
    keep["part_bytes"] = (C.c_uint64 * len(part_bytes))(*part_bytes)
    keep["order"] = (C.c_uint32 * max(1, len(order)))(*order)
    c.n_gated = len(n_units)
    c.n_units = keep["n_units"]
    c.n_parts = len(part_bytes)
    c.part_bytes = keep["part_bytes"]
    c.persistent_slots, c.bank_slots, c.blocks, c.spare_target = persistent_slots, bank_slots, blocks, spare_target
    c.prefetch_reserve, c.prefetch_per_layer, c.prefetch_per_token = prefetch_reserve, prefetch_per_layer, \
        prefetch_per_token
    c.wb_defer, c.wb_on_d2h, c.wb_layer_bytes, c.wb_max_outstanding = wb_defer, wb_on_d2h, wb_layer_bytes, \
        wb_max_outstanding
    c.n_order = len(order)
    c.order = keep["order"]
    c.tokens, c.n_ids, c.n_pred, c.move_bytes, c.inclusive = tokens, n_ids, n_pred, move_bytes, inclusive
    c.policy, c.rows = policy, rows
    c.no_admit, c.clean_evict, c.pf_revert, c.pf_strict = no_admit, clean_evict, pf_revert, pf_strict
    c.disk_queue, c.bank_keep = disk_queue, bank_keep
    c.landing_blocks, c.landing_ttl = landing_blocks, landing_ttl
    if resident_events:  # (token, gated layer, ids): ss_dg_make_resident after that token's boundary; ids () = release
        ev = list(resident_events)
        keep["mr_token"] = (C.c_uint32 * len(ev))(*[e[0] for e in ev])
        keep["mr_layer"] = (C.c_uint32 * len(ev))(*[e[1] for e in ev])
        keep["mr_count"] = (C.c_uint32 * len(ev))(*[len(e[2]) for e in ev])
        flat = [u for e in ev for u in e[2]]
        keep["mr_ids"] = (C.c_uint32 * max(1, len(flat)))(*flat)
        c.mr_n = len(ev)
        c.mr_token, c.mr_layer, c.mr_count, c.mr_ids = (keep["mr_token"], keep["mr_layer"], keep["mr_count"],
                                                          keep["mr_ids"])
    c.round_every, c.round_max_units, c.round_hysteresis, c.round_decay, c.round_budget = \
        round_every, round_max_units, round_hysteresis, round_decay, round_budget
    if weights:
        c.w_trans, c.w_freq, c.w_rec = weights
    if profile is not None:
        flat = np.ascontiguousarray(np.concatenate([np.asarray(x, dtype=np.uint32).reshape(-1) for x in profile]))
        keep["profile"] = flat
        c.profile = flat.ctypes.data_as(C.POINTER(C.c_uint32))
    if disk is not None:
        keep["disk"] = (C.c_uint8 * max(1, len(disk)))(*[1 if f else 0 for f in disk])
        c.disk_tier, c.disk_prefetch, c.home_blocks, c.disk_staging = 1, disk_prefetch, home_blocks, disk_staging
        c.disk = keep["disk"]
    c._keep = keep
    return c


def replay(cfg, ids, preds=None, src_units=None, want_reads=False, xstats=None, rstats=None, pstats=None,
           qstats=None, mstats=None, sstats=None, kstats=None, lstats=None):
    """This library's deterministic replay (tsb_test_dg_replay): (tables, stats[, read_sum]). xstats: an optional
    uint64 array [tokens][6] filled with the file tier's counters after each boundary."""
    keys = sum(cfg.n_units[i] for i in range(cfg.n_gated))
    cfg.xstats = xstats.ctypes.data_as(C.POINTER(C.c_uint64)) if xstats is not None else None
    cfg.rstats = rstats.ctypes.data_as(C.POINTER(C.c_uint64)) if rstats is not None else None  # [tokens][6] rounds
    cfg.pstats = pstats.ctypes.data_as(C.POINTER(C.c_uint64)) if pstats is not None else None  # [tokens][5]
    cfg.qstats = qstats.ctypes.data_as(C.POINTER(C.c_uint64)) if qstats is not None else None  # [tokens][4]
    cfg.mstats = mstats.ctypes.data_as(C.POINTER(C.c_uint64)) if mstats is not None else None  # [tokens][4]
    cfg.sstats = sstats.ctypes.data_as(C.POINTER(C.c_uint64)) if sstats is not None else None  # [tokens][5]
    cfg.kstats = kstats.ctypes.data_as(C.POINTER(C.c_uint64)) if kstats is not None else None  # [tokens][4]
    cfg.lstats = lstats.ctypes.data_as(C.POINTER(C.c_uint64)) if lstats is not None else None  # [tokens][9]
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    tables = np.empty((cfg.tokens, keys), dtype=np.int32)
    stats = np.empty((cfg.tokens, 16), dtype=np.uint64)
    reads = np.zeros((cfg.tokens, cfg.n_gated, cfg.n_ids), dtype=np.uint64) if want_reads else None
    p = np.ascontiguousarray(preds, dtype=np.int32) if preds is not None else None
    P = C.POINTER
    abi.check(abi.load().tsb_test_dg_replay(
        C.byref(cfg), ids.ctypes.data_as(P(C.c_int32)), p.ctypes.data_as(P(C.c_int32)) if p is not None else None,
        tables.ctypes.data_as(P(C.c_int32)), stats.ctypes.data_as(P(C.c_uint64)),
        src_units.ctypes.data_as(P(C.c_uint8)) if src_units is not None else None,
        reads.ctypes.data_as(P(C.c_uint64)) if reads is not None else None))
    return (tables, stats, reads) if want_reads else (tables, stats)
