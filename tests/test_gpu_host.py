"""Host forward mode on the GPU through the C ABI (C1: 8 layers x 16 experts x 3 parts of
131072 bytes, seed 0; top-2 uniform routes from seed 1; 4 residents per layer, 12 pinned; a 4-slot ring; inclusive):
per forward and layer, every unit's table entry points at the same slot as the reference's own host-mode context
(its CPU backend, oracle/_ref) on the same routes, the counters match, and the bytes read through the device table
equal the source bytes."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle  # noqa: E402
from tierstream_b200 import abi, harness, runtime, synth  # noqa: E402


@pytest.fixture(scope="module")
def c1_model():
    m = synth.Model(os.path.join(harness.model_dir(), "tsb-test-c1.bin"), layers=8, units=16,
                    part_bytes=(131072, 131072, 131072), seed=0, top_k=2, with_hash=True)
    m.write()
    return m


def setup(m, dynamic, pin_planned, ring=4, residents=4):
    tiers = []
    for _ in range(m.layers):
        tiers += [abi.SS_TIER_RESIDENT] * residents + [abi.SS_TIER_PINNED] * (m.units - residents)
    b = abi.budget_defaults()
    b.device_bytes = 1 << 30
    b.margin_gib = 1.0 / 1024
    b.margin_fraction = 0.0
    b.ring_slots = ring
    b.dynamic_slots_per_layer = dynamic
    b.host_pinned_bytes = 1 << 30
    o = abi.options_defaults()
    o.forward_mode = abi.SS_FORWARD_HOST
    o.pin_planned = pin_planned
    o.verify_hash = 1
    return tiers, b, o


def expected(m, orc):
    buf = np.empty(m.unit_bytes, dtype=np.uint8)
    out = np.zeros(m.layers * m.units, dtype=np.uint64)
    for L in range(m.layers):
        for u in range(m.units):
            orc.orc_fill_bytes(m.seed, m.unit_offset(L, u), m.unit_bytes, buf.ctypes.data)
            out[L * m.units + u] = orc.orc_checksum(buf.ctypes.data, m.unit_bytes)
    return out


@pytest.mark.parametrize("dynamic,pin_planned,scored", [(0, 1, 0), (2, 0, 0), (3, 1, 0), (2, 1, 1), (0, 1, 1)])
def test_c1_tables_counters_and_bytes_match_reference(c1_model, orc, ref, dynamic, pin_planned, scored):
    """scored: the resident set's SCORED policy (src/resident_set.cpp) with its default window, on Zipf routes so the
    scores differ from recency; the reference's host mode runs the same options."""
    m = c1_model
    tiers, b, o = setup(m, dynamic, pin_planned)
    if scored:
        o.policy = abi.SS_POLICY_SCORED
        routes = synth.zipf_trace(64, m.layers, m.units, 2, s=1.0, seed=3)
    else:
        routes = synth.zipf_trace(64, m.layers, m.units, 2, seed=1, uniform=True)
    desc_json = m.desc(order="ranked")
    ref_locs, ref_stats = oracle.ref_host_replay(desc_json, tiers, b, o, routes, [0] * m.layers)
    desc = runtime.Desc(desc_json)
    plan = runtime.Plan(desc, b, tiers=tiers)
    ctx = runtime.HostContext(desc, plan, o)
    eng = abi.load_engine()
    want = expected(m, orc)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())  # after the inputs torch made on its own stream
    ids_dev = torch.zeros(m.units, dtype=torch.int32, device="cuda")
    out = torch.zeros(m.units, dtype=torch.int64, device="cuda")
    try:
        for f in range(routes.shape[0]):
            before = [ctx.layer_stats(L) for L in range(m.layers)]
            ctx.begin()
            for L in range(m.layers):
                ctx.routes(L, routes[f, L])
                v = ctx.acquire(L, s.cuda_stream)
                locs = ctx.locs(L, m.units)
                assert np.array_equal(locs, ref_locs[f, L * m.units:(L + 1) * m.units]), \
                    "forward %d layer %d: table differs from the reference" % (f, L)
                ids = np.unique(routes[f, L]).astype(np.int32)
                with torch.cuda.stream(s):
                    ids_dev[:ids.size].copy_(torch.from_numpy(ids), non_blocking=False)
                    rc = eng.tse_read_table(C_ptr(v.table_dev), ids_dev.data_ptr(), ids.size, m.unit_bytes,
                                            out.data_ptr(), 16, s.cuda_stream)
                    assert rc == 0
                s.synchronize()
                got = out[:ids.size].cpu().numpy().astype(np.uint64)
                assert np.array_equal(got, want[L * m.units + ids]), "forward %d layer %d: wrong bytes" % (f, L)
                ctx.release(L, s.cuda_stream)
            ctx.end()
            for L in range(m.layers):
                a = ctx.layer_stats(L)
                mine = [a[k] - before[L][k] for k in ("routed", "hits", "admitted", "transient", "evicted")]
                assert mine == [int(x) for x in ref_stats[f, L, :5]], "forward %d layer %d counters" % (f, L)
    finally:
        ctx.close()


def C_ptr(p):
    import ctypes
    return ctypes.cast(p, ctypes.c_void_p).value


def test_layer_all_streams_blobs_through_a_two_slot_ring(orc, ref):
    """C3-shaped, scaled: dense layer blobs, prefix order, the first layers resident, the rest streamed through a
    2-slot ring with ss_layer_all (the Llama-3-70B config at 1 MiB + 17 byte blobs)."""
    m = synth.Model(os.path.join(harness.model_dir(), "tsb-test-blobs.bin"), layers=12, units=1,
                    part_bytes=((1 << 20) + 17,), seed=5, top_k=1)
    m.write()
    import json
    d = json.loads(m.desc(order="prefix"))
    for lay in d["layers"]:
        lay["kind"] = "blob"
        lay.pop("top_k")
    desc_json = json.dumps(d)
    tiers = [abi.SS_TIER_RESIDENT] * 5 + [abi.SS_TIER_PINNED] * 7
    b = abi.budget_defaults()
    b.device_bytes = 1 << 30
    b.margin_gib = 1.0 / 1024
    b.margin_fraction = 0.0
    b.ring_slots = 2
    b.host_pinned_bytes = 1 << 30
    o = abi.options_defaults()
    o.forward_mode = abi.SS_FORWARD_HOST
    routes = np.zeros((3, m.layers, 1), dtype=np.int32)
    ref_locs, ref_stats = oracle.ref_host_replay(desc_json, tiers, b, o, routes, [1] * m.layers)
    desc = runtime.Desc(desc_json)
    plan = runtime.Plan(desc, b, tiers=tiers)
    ctx = runtime.HostContext(desc, plan, o)
    eng = abi.load_engine()
    want = expected(m, orc)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())  # after the inputs torch made on its own stream
    ids_dev = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.zeros(1, dtype=torch.int64, device="cuda")
    try:
        for f in range(3):
            ctx.begin()
            for L in range(m.layers):
                ctx.layer_all(L)
                v = ctx.acquire(L, s.cuda_stream)
                assert np.array_equal(ctx.locs(L, 1), ref_locs[f, L:L + 1])
                with torch.cuda.stream(s):
                    assert eng.tse_read_table(C_ptr(v.table_dev), ids_dev.data_ptr(), 1, m.unit_bytes, out.data_ptr(),
                                              8, s.cuda_stream) == 0
                s.synchronize()
                assert int(out[0].item()) == int(want[L])
                ctx.check_unit(L, 0)
                ctx.release(L, s.cuda_stream)
            ctx.end()
    finally:
        ctx.close()


@pytest.mark.parametrize("dynamic,spare_units,discard,zipf",
                         [(2, 4, 0, None), (0, 1, 0, None), (0, 1, 1, None), (0, 2, 0, 1.2), (1, 1, 1, 0.8)])
def test_c1_exclusive_mode_matches_reference(c1_model, orc, ref, dynamic, spare_units, discard, zipf):
    """The exclusive tier mode on C1's shape: admissions capped by the free blocks (deferred misses stay transient),
    victims written back into free blocks before their slots are refilled, promotions freeing their blocks at
    ss_end, and with exclusive_discard the victims past the free blocks discarded to their files. Per forward and
    layer the table slots and counters equal the reference's, the eight exclusive counters after every forward equal
    the reference's, and every unit read through the table has its source bytes."""
    m = c1_model
    tiers, b, o = setup(m, dynamic=dynamic, pin_planned=0)
    b.tier_mode = abi.SS_TIER_MODE_EXCLUSIVE
    b.host_spare_units = spare_units
    o.exclusive_discard = discard
    if zipf:
        routes = synth.zipf_trace(48, m.layers, m.units, 2, s=zipf, seed=3)
    else:
        routes = synth.zipf_trace(48, m.layers, m.units, 2, seed=1, uniform=True)
    desc_json = m.desc(order="ranked", tiers="pinned|disk" if discard else "pinned")
    ref_locs, ref_stats, ref_x = oracle.ref_host_replay(desc_json, tiers, b, o, routes, [0] * m.layers,
                                                        want_exclusive=True)
    assert ref_x[-1][0] > 0, "the trace must write back"
    if dynamic == 0 and not discard:
        assert ref_x[-1][2] > 0, "few free blocks must defer admissions"
    if discard:
        assert ref_x[-1][7] > 0, "victims past the free blocks must be discarded"
    desc = runtime.Desc(desc_json)
    plan = runtime.Plan(desc, b, tiers=tiers)
    ctx = runtime.HostContext(desc, plan, o)
    eng = abi.load_engine()
    want = expected(m, orc)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())  # after the inputs torch made on its own stream
    ids_dev = torch.zeros(m.units, dtype=torch.int32, device="cuda")
    out = torch.zeros(m.units, dtype=torch.int64, device="cuda")
    try:
        for f in range(routes.shape[0]):
            before = [ctx.layer_stats(L) for L in range(m.layers)]
            ctx.begin()
            for L in range(m.layers):
                ctx.routes(L, routes[f, L])
                v = ctx.acquire(L, s.cuda_stream)
                assert np.array_equal(ctx.locs(L, m.units), ref_locs[f, L * m.units:(L + 1) * m.units]), \
                    "forward %d layer %d: table differs from the reference" % (f, L)
                ids = np.unique(routes[f, L]).astype(np.int32)
                with torch.cuda.stream(s):
                    ids_dev[:ids.size].copy_(torch.from_numpy(ids), non_blocking=False)
                    assert eng.tse_read_table(C_ptr(v.table_dev), ids_dev.data_ptr(), ids.size, m.unit_bytes,
                                              out.data_ptr(), 16, s.cuda_stream) == 0
                s.synchronize()
                got = out[:ids.size].cpu().numpy().astype(np.uint64)
                assert np.array_equal(got, want[L * m.units + ids]), "forward %d layer %d: wrong bytes" % (f, L)
                ctx.release(L, s.cuda_stream)
            ctx.end()
            for L in range(m.layers):
                a = ctx.layer_stats(L)
                mine = [a[k] - before[L][k] for k in ("routed", "hits", "admitted", "transient", "evicted")]
                assert mine == [int(x) for x in ref_stats[f, L, :5]], "forward %d layer %d counters" % (f, L)
            assert ctx.exclusive_stats() == [int(x) for x in ref_x[f]], "forward %d exclusive counters" % f
    finally:
        ctx.close()


def run_with_prefetch(m, ctx, routes, pf, mode, ref_locs, ref_stats, want, all_layers=False):
    """Drives forwards the way the reference harness does (layer 0's prefetch before ss_begin, layer L + 1's before
    the routes of layer L) and checks tables, the nine counters and the bytes read through the table."""
    eng = abi.load_engine()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())  # after the inputs torch made on its own stream
    ids_dev = torch.zeros(m.units, dtype=torch.int32, device="cuda")
    out = torch.zeros(m.units, dtype=torch.int64, device="cuda")
    keys9 = ("routed", "hits", "admitted", "transient", "evicted", "prefetched", "spec_issued", "spec_used",
             "spec_dropped")

    def prefetch(f, L):
        if L >= m.layers:
            return
        if mode == 3:
            ctx.prefetch_layer(L)
        else:
            ctx.prefetch(L, pf[f, L], speculative=mode == 2)

    for f in range(routes.shape[0]):
        before = [ctx.layer_stats(L) for L in range(m.layers)]
        prefetch(f, 0)
        ctx.begin()
        for L in range(m.layers):
            prefetch(f, L + 1)
            if all_layers:
                ctx.layer_all(L)
                ids = np.arange(m.units, dtype=np.int32)
            else:
                ctx.routes(L, routes[f, L])
                ids = np.unique(routes[f, L]).astype(np.int32)
            v = ctx.acquire(L, s.cuda_stream)
            assert np.array_equal(ctx.locs(L, m.units), ref_locs[f, L * m.units:(L + 1) * m.units]), \
                "forward %d layer %d: table differs from the reference" % (f, L)
            with torch.cuda.stream(s):
                ids_dev[:ids.size].copy_(torch.from_numpy(ids), non_blocking=False)
                assert eng.tse_read_table(C_ptr(v.table_dev), ids_dev.data_ptr(), ids.size, m.unit_bytes,
                                          out.data_ptr(), 16, s.cuda_stream) == 0
            s.synchronize()
            got = out[:ids.size].cpu().numpy().astype(np.uint64)
            assert np.array_equal(got, want[L * m.units + ids]), "forward %d layer %d: wrong bytes" % (f, L)
            ctx.release(L, s.cuda_stream)
        ctx.end()
        for L in range(m.layers):
            a = ctx.layer_stats(L)
            mine = [a[k] - before[L][k] for k in keys9]
            assert mine == [int(x) for x in ref_stats[f, L]], "forward %d layer %d counters %s vs %s" % (
                f, L, mine, ref_stats[f, L].tolist())


@pytest.mark.parametrize("mode,dynamic", [(2, 2), (2, 0), (1, 2), (1, 0)])
def test_c1_prefetch_matches_reference(c1_model, orc, ref, mode, dynamic):
    """ss_prefetch ahead of the routes (speculative guesses through the stream ring within lookahead_budget, or
    certain ids admitted as demands), layer 0's issued between forwards: tables, the nine counters (prefetched and
    the speculative issued / used / dropped among them) and the bytes equal the reference's."""
    m = c1_model
    tiers, b, o = setup(m, dynamic=dynamic, pin_planned=0)
    routes = synth.zipf_trace(24, m.layers, m.units, 2, seed=1, uniform=True)
    pf = synth.zipf_trace(24, m.layers, m.units, 3, seed=9, uniform=True) if mode == 2 else routes
    desc_json = m.desc(order="ranked")
    ref_locs, ref_stats = oracle.ref_host_replay(desc_json, tiers, b, o, routes, [0] * m.layers, pf_ids=pf,
                                                 pf_mode=mode)
    assert ref_stats[:, :, 5:].sum() > 0, "the schedule must prefetch"
    desc = runtime.Desc(desc_json)
    plan = runtime.Plan(desc, b, tiers=tiers)
    ctx = runtime.HostContext(desc, plan, o)
    try:
        run_with_prefetch(m, ctx, routes, pf, mode, ref_locs, ref_stats, expected(m, orc))
    finally:
        ctx.close()


def test_layer_prefetch_overlaps_the_blob_stream(orc, ref):
    """C3-shaped, scaled: ss_prefetch_layer(L + 1) before layer L's ss_layer_all, through a 2-slot ring."""
    m = synth.Model(os.path.join(harness.model_dir(), "tsb-test-blobs.bin"), layers=12, units=1,
                    part_bytes=((1 << 20) + 17,), seed=5, top_k=1)
    m.write()
    import json
    d = json.loads(m.desc(order="prefix"))
    for lay in d["layers"]:
        lay["kind"] = "blob"
        lay.pop("top_k")
    desc_json = json.dumps(d)
    tiers = [abi.SS_TIER_RESIDENT] * 5 + [abi.SS_TIER_PINNED] * 7
    b = abi.budget_defaults()
    b.device_bytes = 1 << 30
    b.margin_gib = 1.0 / 1024
    b.margin_fraction = 0.0
    b.ring_slots = 2
    b.host_pinned_bytes = 1 << 30
    o = abi.options_defaults()
    o.forward_mode = abi.SS_FORWARD_HOST
    routes = np.zeros((3, m.layers, 1), dtype=np.int32)
    ref_locs, ref_stats = oracle.ref_host_replay(desc_json, tiers, b, o, routes, [1] * m.layers, pf_mode=3)
    assert ref_stats[:, :, 5].sum() > 0
    desc = runtime.Desc(desc_json)
    plan = runtime.Plan(desc, b, tiers=tiers)
    ctx = runtime.HostContext(desc, plan, o)
    try:
        run_with_prefetch(m, ctx, routes, None, 3, ref_locs, ref_stats, expected(m, orc), all_layers=True)
    finally:
        ctx.close()



class _NoClocks:
    def __init__(self, index):
        pass

    def stop(self):
        return {}


@pytest.mark.parametrize("name", ["c1-host", "blob-sparse"])
def test_host_bench_forwards_read_the_generator_bytes(monkeypatch, name):
    """bench.py's host-mode leg (tierstream_b200/host_bench.py) at small size: forwards of tse_host_forward (routes,
    acquire, reader through the device table, release, end - the engine loop in native code) over C1, and over a
    sparse 6-layer blob model (1 MiB + 48 byte blobs, 2 resident, 2-slot ring) whose residents' slots and pinned blocks
    are written from the generator after the open, as the Llama-3-70B-shaped workload does at full size. Every reader's
    checksum equals the generator's, in both checksum modes."""
    from tierstream_b200 import host_bench
    if name == "blob-sparse":
        monkeypatch.setitem(host_bench.WORKLOADS, name, dict(host_bench.WORKLOADS["llama3-70b-host"], layers=6,
                                                             parts=((1 << 20) + 48,), resident=2, slices=64,
                                                             file="tsb-test-blob-sparse.bin"))
    line, trace, bad = host_bench.run(name, 4, 2, torch, _NoClocks, 0)
    assert bad == 0
    assert line["verified"]["units"] > 0 and line["value"] > 0 and line["streamed_units_per_token"] > 0
    if name == "blob-sparse":
        assert line["streamed_units_per_token"] == 4  # the 4 pinned layers, every forward
