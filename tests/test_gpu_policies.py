"""Scored eviction (SS_POLICY_SCORED) and placement rounds (ss_dg_round) through the device-gated context on the GPU:
under the deterministic schedule the device's slot table after every token equals the reference DgCore's replay with
the same policy (with and without a TSSCPRF1 profile of transition counts) or the same rounds, every routed unit's
bytes are the source's, ss_dg_set_policy switches between LRU and SCORED between tokens (refused for a context opened
with LRU, whose score tables do not exist), and the rounds' results sum to the reference's."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle  # noqa: E402
from tierstream_b200 import abi, harness, runtime, synth  # noqa: E402

from test_gpu_dg import expected_sums  # noqa: E402
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
