"""Scored eviction (SS_POLICY_SCORED) through the device-gated context on the GPU: under the deterministic schedule the
device's slot table after every token equals the reference DgCore's replay with the same policy (with and without a
TSSCPRF1 profile of transition counts), every routed unit's bytes are the source's, and ss_dg_set_policy switches
between LRU and SCORED between tokens (refused for a context opened with LRU, whose score tables do not exist)."""
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
