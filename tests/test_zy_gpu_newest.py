"""The newest GPU paths, kept in the last file so that a failure here does not stop the earlier files under pytest -x:
the open's pipelined fill, host read-ahead, scored eviction and placement rounds.

Scored eviction (SS_POLICY_SCORED) and placement rounds (ss_dg_round) through the device-gated context on the GPU:
under the deterministic schedule the device's slot table after every token equals the reference DgCore's replay with
the same policy (with and without a TSSCPRF1 profile of transition counts) or the same rounds, every routed unit's
bytes are the source's, ss_dg_set_policy switches between LRU and SCORED between tokens (refused for a context opened
with LRU, whose score tables do not exist), and the rounds' results sum to the reference's."""
import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle  # noqa: E402
from tierstream_b200 import abi, harness, runtime, synth  # noqa: E402

from test_gpu_dg import expected_sums, run_tokens, small_model  # noqa: E402,F401
from test_gpu_host import C_ptr, expected  # noqa: E402
from test_score_profile import identity_of, profile_bytes  # noqa: E402


@pytest.fixture(scope="module")
def model():
    m = synth.Model(os.path.join(harness.model_dir(), "tsb-test-scored.bin"), layers=6, units=16,
                    part_bytes=(2048, 2048, 4096), seed=13, top_k=2, with_hash=True, base=0)
    m.write()
    return m


@pytest.mark.parametrize("with_profile", [False, True])
def test_scored_tables_match_reference(model, orc, ref, monkeypatch, with_profile):
    monkeypatch.setenv("TSB_DG_DETERMINISTIC", "1")
    m = model
    G, U = m.layers, m.units
    ids = synth.zipf_trace(30, G, U, 2, s=0.8, seed=41, rho=0.5)
    cells = prof = None
    if with_profile:
        ident, units = identity_of(m.desc())
        rng = np.random.default_rng(3)
        cells = [rng.integers(0, 40, size=(u, u), dtype=np.uint32) for u in units]
        prof = profile_bytes(units, ident, cells)
    run = harness.DgRun(m, residents_per_layer=3, spare_per_layer=2, max_ids=2, policy=abi.SS_POLICY_SCORED,
                        profile=prof)
    try:
        res = run.resident_keys
        P = G * U - len(res)
        cfg = runtime.replay_config([U] * G, list(m.part_bytes), persistent_slots=len(res) + 2 * G, bank_slots=2,
                                    blocks=P + 2 * G, spare_target=2 * G, order=res, tokens=ids.shape[0], n_ids=2,
                                    policy=1, profile=cells)
        t_ref, s_ref = oracle.ref_replay(cfg, ids)
        want = expected_sums(m, orc)
        for t in range(ids.shape[0]):
            got = run.step(ids[t])
            keys = np.arange(G)[:, None] * U + ids[t]
            assert np.array_equal(got, want[keys]), "token %d read wrong bytes" % t
            assert np.array_equal(run.ctx.table(run.keys), t_ref[t]), "slot table differs after token %d" % t
        st = run.ctx.stats()
        assert st["evicted"] == s_ref[-1][10] and st["misses"] == s_ref[-1][2]
        assert st["scored_victims"] > 0 and st["score_fallbacks"] == 0
        # LRU, then SCORED again, between tokens: the bytes stay right
        run.ctx.set_policy(abi.SS_POLICY_LRU)
        for t in range(5):
            got = run.step(ids[t])
            assert np.array_equal(got, want[np.arange(G)[:, None] * U + ids[t]])
        v = run.ctx.stats()["scored_victims"]
        run.ctx.set_policy(abi.SS_POLICY_SCORED)
        for t in range(5, 15):
            got = run.step(ids[t])
            assert np.array_equal(got, want[np.arange(G)[:, None] * U + ids[t]])
        assert run.ctx.stats()["scored_victims"] > v
        run.ctx.check()
    finally:
        run.close()


def test_set_policy_needs_scoring_at_open(model):
    run = harness.DgRun(model, residents_per_layer=3, max_ids=2)
    try:
        st = abi.load().ss_dg_set_policy(run.ctx.h, abi.SS_POLICY_SCORED)
        assert st == abi.SS_E_INVALID and b"set up at ss_open" in abi.load().ss_last_error()
    finally:
        run.close()


@pytest.mark.parametrize("wb_defer", [0, 1])
def test_rounds_match_reference(model, orc, ref, monkeypatch, wb_defer):
    monkeypatch.setenv("TSB_DG_DETERMINISTIC", "1")
    m = model
    G, U = m.layers, m.units
    ids = synth.zipf_trace(30, G, U, 2, s=1.2, seed=51)
    run = harness.DgRun(m, residents_per_layer=3, max_ids=2, wb_defer=wb_defer)
    try:
        res = run.resident_keys
        P = G * U - len(res)
        cfg = runtime.replay_config([U] * G, list(m.part_bytes), persistent_slots=len(res) + G, bank_slots=2,
                                    blocks=P + G, spare_target=G, order=res, tokens=ids.shape[0], n_ids=2,
                                    wb_defer=wb_defer, round_every=5)
        r_ref = np.zeros((ids.shape[0], 6), dtype=np.uint64)
        t_ref, s_ref = oracle.ref_replay(cfg, ids, rstats=r_ref)
        want = expected_sums(m, orc)
        sums = np.zeros(6, dtype=np.uint64)
        for t in range(ids.shape[0]):
            got = run.step(ids[t])
            assert np.array_equal(got, want[np.arange(G)[:, None] * U + ids[t]]), "token %d read wrong bytes" % t
            if (t + 1) % 5 == 0:
                r = run.ctx.round()
                sums += np.array([1, r["promoted_to_device"], r["promoted_to_pinned"], r["demoted_from_device"],
                                  r["dropped_to_file"], r["bytes_read"] + r["bytes_h2d"] + r["bytes_written_back"]],
                                 dtype=np.uint64)
            assert np.array_equal(run.ctx.table(run.keys), t_ref[t]), "slot table differs after token %d" % t
        assert np.array_equal(sums, r_ref[-1]) and sums[1] > 0
        assert run.ctx.stats()["round_count"] == 6
        run.ctx.check()
        for L in range(G):
            for u in range(U):
                run.ctx.check_unit(L, u)
    finally:
        run.close()


@pytest.mark.parametrize("load", [{"TSB_LOAD_SERIAL": "1"},
                                  {"TSB_LOAD_BUFFERS": "1", "TSB_LOAD_BUFFER_MIB": "1", "TSB_LOAD_READERS": "3"},
                                  {"TSB_LOAD_BUFFERS": "3", "TSB_LOAD_READERS": "16"}, {}])
def test_open_fill_lands_every_unit(small_model, orc, monkeypatch, load):
    """The open's fill, phased or pipelined with rings of one buffer of a few units up to the default: every resident's
    slot and every pinned unit's block equals the source, and the tokens read the right bytes."""
    for k, v in load.items():
        monkeypatch.setenv(k, v)
    m = small_model
    run = harness.DgRun(m, residents_per_layer=5, max_ids=2, verify=True)
    try:
        for L in range(m.layers):
            for u in range(m.units):
                run.ctx.check_unit(L, u)
        o = json.loads(run.ctx.stats_json())["open"]
        assert o["load"] == ("serial" if load.get("TSB_LOAD_SERIAL") else "pipeline")
        if o["load"] == "pipeline":
            assert o["load_slot_units"] == 5 * m.layers and o["load_pinned_units"] == (m.units - 5) * m.layers
            assert 1 <= o["load_buffers"] <= int(load.get("TSB_LOAD_BUFFERS", 4))
        run_tokens(run, synth.zipf_trace(10, m.layers, m.units, 2, s=0.8, seed=21), expected_sums(m, orc))
    finally:
        run.close()


@pytest.mark.parametrize("ra", [0, 3])
def test_host_read_ahead_lands_file_blobs(orc, ra):
    """C3-shaped, scaled, with the streamed blobs in the model file only (tier DISK): ss_host_prefetch_layer for the
    next two layers ahead of each layer's ss_layer_all. With readahead_units = 3 the blobs are read into the read-ahead
    buffers and land from there; every blob read through the table has its bytes, with and without read-ahead, and
    the read-ahead counters add up (landed + unused = read <= requested)."""
    import json
    m = synth.Model(os.path.join(harness.model_dir(), "tsb-test-blobs.bin"), layers=12, units=1,
                    part_bytes=((1 << 20) + 17,), seed=5, top_k=1)
    m.write()
    d = json.loads(m.desc(order="prefix", tiers="pinned|disk"))
    for lay in d["layers"]:
        lay["kind"] = "blob"
        lay.pop("top_k")
    desc_json = json.dumps(d)
    tiers = [abi.SS_TIER_RESIDENT] * 5 + [abi.SS_TIER_DISK] * 7
    b = abi.budget_defaults()
    b.device_bytes = 1 << 30
    b.margin_gib = 1.0 / 1024
    b.margin_fraction = 0.0
    b.ring_slots = 2
    b.host_pinned_bytes = 1 << 30
    o = abi.options_defaults()
    o.forward_mode = abi.SS_FORWARD_HOST
    o.verify_hash = 1
    o.readahead_units = ra
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
                for k in (1, 2):
                    if L + k < m.layers:
                        ctx.host_prefetch_layer(L + k)
                ctx.layer_all(L)
                v = ctx.acquire(L, s.cuda_stream)
                with torch.cuda.stream(s):
                    assert eng.tse_read_table(C_ptr(v.table_dev), ids_dev.data_ptr(), 1, m.unit_bytes, out.data_ptr(),
                                              8, s.cuda_stream) == 0
                s.synchronize()
                assert int(out[0].item()) == int(want[L]), "forward %d layer %d read wrong bytes" % (f, L)
                ctx.check_unit(L, 0)
                ctx.release(L, s.cuda_stream)
            ctx.end()
        st = json.loads(ctx.stats_json())
        if ra:
            r = st["readahead"]
            assert r["buffers"] == ra and r["landed"] > 0 and r["failed"] == 0
            assert r["landed"] + r["unused"] == r["read"] <= r["requested"]
        else:
            assert "readahead" not in st
    finally:
        ctx.close()
