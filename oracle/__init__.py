"""TEST INFRASTRUCTURE ONLY: the CPU checkers the tests, __graft_entry__.smoke() and bench.py's cpu_baseline leg compare
the product with. Nothing in tierstream_b200/ imports this package.

  oracle/_ref/liboracle.so  the C restatement (oracle.c): xxh64, the synthetic bytes, the export mask, ss_dg_slot,
                            the GPU tests' checksum; each function cites the reference file:line it restates.
  oracle/_ref/libtsref.so   the reference's own C++ sources compiled directly (oracle/Makefile), with a harness
                            (ref_harness.cpp) that replays a trace through the reference's DgCore.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
_orc = None
_ref = None


def orc():
    global _orc
    if _orc is None:
        lib = C.CDLL(os.path.join(HERE, "_ref", "liboracle.so"))
        lib.orc_xxh64.restype = C.c_uint64
        lib.orc_xxh64.argtypes = [C.c_void_p, C.c_size_t, C.c_uint64]
        lib.orc_xxh64_spans.restype = C.c_uint64
        lib.orc_xxh64_spans.argtypes = [C.POINTER(C.c_void_p), C.POINTER(C.c_uint64), C.c_uint32, C.c_uint64]
        lib.orc_fill_bytes.restype = None
        lib.orc_fill_bytes.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_void_p]
        lib.orc_checksum.restype = C.c_uint64
        lib.orc_checksum.argtypes = [C.c_void_p, C.c_uint64]
        lib.orc_export_mask.restype = C.c_uint64
        lib.orc_export_mask.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_uint32,
                                        C.POINTER(C.c_uint32)]
        lib.orc_dg_slot.restype = C.c_int32
        lib.orc_dg_slot.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.c_int32, C.c_uint32, C.c_uint32,
                                    C.POINTER(C.c_uint32)]
        _orc = lib
    return _orc


def ref_available():
    return os.path.exists(os.path.join(HERE, "_ref", "libtsref.so"))


def ref():
    """The reference harness (None when oracle/_ref/libtsref.so was not built)."""
    global _ref
    if _ref is None and ref_available():
        lib = C.CDLL(os.path.join(HERE, "_ref", "libtsref.so"))
        lib.oref_copy_threads.restype = C.c_uint
        lib.oref_copy_threads.argtypes = []
        lib.oref_xxh64.restype = C.c_uint64
        lib.oref_xxh64.argtypes = [C.c_void_p, C.c_size_t, C.c_uint64]
        lib.oref_host_replay.restype = C.c_int
        lib.oref_host_replay.argtypes = [C.c_char_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p,
                                         C.c_uint32, C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.c_void_p, C.c_void_p, C.c_uint32, C.c_int, C.c_char_p, C.c_size_t]
        lib.oref_resident_replay.restype = C.c_int
        lib.oref_resident_replay.argtypes = [C.c_int32, C.c_int32, C.c_int32, C.c_uint32, C.c_void_p, C.c_void_p,
                                             C.c_uint32, C.c_uint32, C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p,
                                             C.c_void_p, C.c_void_p, C.c_void_p, C.c_char_p, C.c_size_t]
        lib.oref_defaults.restype = None
        lib.oref_defaults.argtypes = [C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32]
        lib.oref_plan.restype = C.c_int
        lib.oref_plan.argtypes = [C.c_char_p, C.c_size_t, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t,
                                  C.c_int, C.c_void_p, C.c_size_t, C.c_void_p, C.c_char_p, C.c_size_t, C.c_char_p,
                                  C.c_size_t, C.c_void_p, C.c_size_t, C.c_void_p, C.c_char_p, C.c_size_t]
        lib.oref_dg_layout.restype = C.c_int
        lib.oref_dg_layout.argtypes = [C.c_char_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p,
                                       C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32, C.c_char_p, C.c_size_t]
        lib.oref_dg_replay.restype = C.c_int
        lib.oref_dg_replay.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                       C.c_void_p, C.c_char_p, C.c_size_t]
        _ref = lib
    return _ref


def ref_host_replay(desc_json, tiers, budget, options, routes, all_layers, want_exclusive=False, pf_ids=None,
                    pf_mode=0):
    """The reference's host forward mode (CPU backend) over routes [forwards][layers][n_ids]: (locs [forwards][units][2],
    stats [forwards][layers][9] = routed, hits, admitted, transient, evicted, prefetched, spec_issued, spec_used,
    spec_dropped[, exclusive [forwards][8] = writebacks,
    writeback_bytes, deferred, promoted, free_blocks, min_free_blocks, rereads, discards after each forward]).
    Prefetches (pf_mode 1 certain pf_ids, 2 speculative pf_ids [forwards][layers][n], 3 whole layers): layer 0's
    before ss_begin, layer L + 1's before the routes of layer L."""
    import numpy as np
    routes = np.ascontiguousarray(routes, dtype=np.int32)
    F, L, n = routes.shape
    total = len(tiers)
    t = np.ascontiguousarray(tiers, dtype=np.uint8)
    al = np.ascontiguousarray(all_layers, dtype=np.uint8)
    locs = np.empty((F, total, 2), dtype=np.int32)
    stats = np.empty((F, L, 9), dtype=np.uint64)
    err = C.create_string_buffer(512)
    raw = desc_json.encode()
    xs = np.zeros((F, 8), dtype=np.uint64) if want_exclusive else None
    pf = np.ascontiguousarray(pf_ids, dtype=np.int32) if pf_ids is not None else None
    n_pf = pf.shape[2] if pf is not None else 0
    rc = ref().oref_host_replay(raw, len(raw), t.ctypes.data, t.size, C.byref(budget), C.byref(options), F,
                                routes.ctypes.data, n, al.ctypes.data, locs.ctypes.data, stats.ctypes.data,
                                xs.ctypes.data if xs is not None else None, pf.ctypes.data if pf is not None else None,
                                n_pf, pf_mode, err, 512)
    if rc != 0:
        raise RuntimeError("reference host replay failed: " + err.value.decode())
    return (locs, stats, xs) if want_exclusive else (locs, stats)


def ref_replay(cfg, ids, preds=None, src_units=None, want_reads=False, xstats=None, rstats=None, pstats=None,
               qstats=None, mstats=None, sstats=None, kstats=None, lstats=None):
    """The reference DgCore's deterministic replay on the same config struct: (tables, stats[, read_sum]). xstats: an
    optional uint64 array [tokens][6] for the three-tier counters (disk_reads, disk_read_bytes, disk_stage_waits,
    disk_drops, disk_discards, file units) after each boundary."""
    import numpy as np
    keys = sum(cfg.n_units[i] for i in range(cfg.n_gated))
    cfg.xstats = xstats.ctypes.data_as(C.POINTER(C.c_uint64)) if xstats is not None else None
    cfg.rstats = rstats.ctypes.data_as(C.POINTER(C.c_uint64)) if rstats is not None else None
    cfg.pstats = pstats.ctypes.data_as(C.POINTER(C.c_uint64)) if pstats is not None else None
    cfg.qstats = qstats.ctypes.data_as(C.POINTER(C.c_uint64)) if qstats is not None else None
    cfg.mstats = mstats.ctypes.data_as(C.POINTER(C.c_uint64)) if mstats is not None else None
    cfg.sstats = sstats.ctypes.data_as(C.POINTER(C.c_uint64)) if sstats is not None else None
    cfg.kstats = kstats.ctypes.data_as(C.POINTER(C.c_uint64)) if kstats is not None else None
    cfg.lstats = lstats.ctypes.data_as(C.POINTER(C.c_uint64)) if lstats is not None else None
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    tables = np.empty((cfg.tokens, keys), dtype=np.int32)
    stats = np.empty((cfg.tokens, 16), dtype=np.uint64)
    reads = np.zeros((cfg.tokens, cfg.n_gated, cfg.n_ids), dtype=np.uint64) if want_reads else None
    p = np.ascontiguousarray(preds, dtype=np.int32) if preds is not None else None
    err = C.create_string_buffer(512)
    rc = ref().oref_dg_replay(C.byref(cfg), ids.ctypes.data, p.ctypes.data if p is not None else None,
                              tables.ctypes.data, stats.ctypes.data,
                              src_units.ctypes.data if src_units is not None else None,
                              reads.ctypes.data if reads is not None else None, err, 512)
    if rc != 0:
        raise RuntimeError("reference replay failed: " + err.value.decode())
    return (tables, stats, reads) if want_reads else (tables, stats)
