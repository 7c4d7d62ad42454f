"""The device-gated setups the GPU tests open (harness.DgSetup: descriptor, plan, budget, options), checked on the CPU:
the layout ss_open takes for each (tsb_test_dg_layout) has the spare slots, spare blocks, banks, pinned homes, staging
buffers, policy and residents that the reference replay of that GPU test is configured with, so the GPU test compares
the device's tables against a replay of the same cache. Each case names the GPU test whose setup it restates."""
import ctypes as C
import os

import numpy as np
import pytest

from tierstream_b200 import abi, harness, synth

from test_score_profile import identity_of, profile_bytes

N_OUT = 23
(KEYS, R, D, B, P, Q, I, F, S, QUEUE, BLOCKS, PERSISTENT, SLOTS, GUARD, UNIT, STRIDE, DISK, DISK_PF, SCORED, W_T, W_F,
 W_R, N_RES) = range(N_OUT)


def model(name, seed):
    return synth.Model(os.path.join(harness.model_dir(), name), layers=6, units=16, part_bytes=(2048, 2048, 4096),
                       seed=seed, top_k=2, with_hash=True, base=0)


def layout(s):
    out = np.zeros(N_OUT, dtype=np.uint64)
    res = np.zeros(4096, dtype=np.uint32)
    st = abi.load().tsb_test_dg_layout(s.desc.h, s.plan.h, C.byref(s.options),
                                       out.ctypes.data_as(C.POINTER(C.c_uint64)), N_OUT, res.ctypes.data, res.size)
    assert st == abi.SS_OK, abi.load().ss_last_error()
    return out, res[:int(out[N_RES])].tolist()


def expect(out, res, s, persistent_slots, blocks, spare_target, bank_slots=2, home_blocks=None, disk_staging=None,
           scored=0):
    """replay_config's numbers: persistent slots = residents + spare slots, blocks = pinned units + spare blocks, the
    spare target (every spare slot, the default dg_spare_target), the banks, the residents in placement order."""
    assert int(out[PERSISTENT]) == persistent_slots
    assert int(out[BLOCKS]) == blocks
    assert int(out[D]) == spare_target
    assert int(out[B]) == bank_slots
    assert res == s.resident_keys
    if home_blocks is not None:
        assert int(out[DISK]) == 1 and int(out[P]) == home_blocks
    if disk_staging is not None:
        assert int(out[S]) == disk_staging
    assert int(out[SCORED]) == scored
    if scored:
        assert [int(out[W_T]), int(out[W_F]), int(out[W_R])] == [700, 200, 100]


def test_gpu_dg_default_setup():
    """test_gpu_dg.replay_cfg_for: one spare slot and block per layer."""
    m = model("tsb-test-small.bin", 3)
    s = harness.DgSetup(m, residents_per_layer=3, max_ids=2, verify=True)
    out, res = layout(s)
    G, U = m.layers, m.units
    expect(out, res, s, len(s.resident_keys) + G, G * U - len(s.resident_keys) + G, G)


@pytest.mark.parametrize("with_profile", [False, True])
def test_gpu_policies_scored_setup(with_profile):
    """test_zy_gpu_newest.test_scored_tables_match_reference: two spare slots and blocks per layer, SCORED, with and
    without a profile (which the layout checks against the descriptor's identity)."""
    m = model("tsb-test-scored.bin", 13)
    prof = None
    if with_profile:
        ident, units = identity_of(m.desc())
        rng = np.random.default_rng(3)
        prof = profile_bytes(units, ident, [rng.integers(0, 40, size=(u, u), dtype=np.uint32) for u in units])
    s = harness.DgSetup(m, residents_per_layer=3, spare_per_layer=2, max_ids=2, policy=abi.SS_POLICY_SCORED,
                        profile=prof)
    out, res = layout(s)
    G, U = m.layers, m.units
    P_ = G * U - len(s.resident_keys)
    expect(out, res, s, len(s.resident_keys) + 2 * G, P_ + 2 * G, 2 * G, scored=1)


@pytest.mark.parametrize("wb_defer", [0, 1])
def test_gpu_policies_rounds_setup(wb_defer):
    """test_zy_gpu_newest.test_rounds_match_reference."""
    m = model("tsb-test-scored.bin", 13)
    s = harness.DgSetup(m, residents_per_layer=3, max_ids=2, wb_defer=wb_defer)
    out, res = layout(s)
    G, U = m.layers, m.units
    expect(out, res, s, len(s.resident_keys) + G, G * U - len(s.resident_keys) + G, G)


def test_gpu_policies_lru_setup_has_no_score_tables():
    """test_zy_gpu_newest.test_set_policy_needs_scoring_at_open: opened with LRU."""
    s = harness.DgSetup(model("tsb-test-scored.bin", 13), residents_per_layer=3, max_ids=2)
    out, _ = layout(s)
    assert int(out[SCORED]) == 0


@pytest.mark.parametrize("S_", [3])
def test_gpu_dg_file_tier_setup(S_):
    """test_gpu_dg.file_tier_run / file_tier_cfg: per layer 3 residents, 4 pinned units, the rest in the file."""
    m = model("tsb-test-small.bin", 3)
    res = [g * m.units + u for g in range(m.layers) for u in range(3)]
    disk = [g * m.units + u for g in range(m.layers) for u in range(7, m.units)]
    s = harness.DgSetup(m, resident_keys=res, max_ids=2, disk_keys=disk, disk_staging=S_)
    out, got = layout(s)
    G, U = m.layers, m.units
    P_ = G * U - len(res) - len(disk)
    expect(out, got, s, len(res) + G, P_ + G, G, home_blocks=P_, disk_staging=S_)
    assert int(out[F]) == len(disk)


def test_gpu_dg_open_fill_setup():
    """test_zy_gpu_newest.test_open_fill_lands_every_unit: five residents per layer, hashes checked."""
    m = model("tsb-test-small.bin", 3)
    s = harness.DgSetup(m, residents_per_layer=5, max_ids=2, verify=True)
    out, res = layout(s)
    assert int(out[R]) == 5 * m.layers and res == s.resident_keys


@pytest.mark.parametrize("with_profile", [False, True])
def test_gpu_policies_scored_trace_scores(ref, with_profile):
    """test_zy_gpu_newest.test_scored_tables_match_reference's trace and replay, on both caches: victims are chosen by
    score and never fall back to LRU, as that test asserts of the device's context."""
    import oracle
    from tierstream_b200 import runtime
    m = model("tsb-test-scored.bin", 13)
    G, U = m.layers, m.units
    ids = synth.zipf_trace(30, G, U, 2, s=0.8, seed=41, rho=0.5)
    cells = None
    if with_profile:
        rng = np.random.default_rng(3)
        cells = [rng.integers(0, 40, size=(u, u), dtype=np.uint32) for u in [U] * G]
    res = [g * U + u for g in range(G) for u in range(3)]
    cfg = runtime.replay_config([U] * G, list(m.part_bytes), persistent_slots=len(res) + 2 * G, bank_slots=2,
                                blocks=G * U - len(res) + 2 * G, spare_target=2 * G, order=res, tokens=ids.shape[0],
                                n_ids=2, policy=1, profile=cells)
    q_ref = np.zeros((ids.shape[0], 5), dtype=np.uint64)
    q_new = np.zeros((ids.shape[0], 5), dtype=np.uint64)
    oracle.ref_replay(cfg, ids, sstats=q_ref)
    runtime.replay(cfg, ids, sstats=q_new)
    assert np.array_equal(q_new, q_ref)
    assert q_ref[-1][1] > 0 and q_ref[-1][0] == 0


@pytest.mark.parametrize("wb_defer", [0, 1])
def test_gpu_policies_rounds_trace_promotes(ref, wb_defer):
    """test_zy_gpu_newest.test_rounds_match_reference's trace: its six rounds promote units in the reference replay."""
    import oracle
    from tierstream_b200 import runtime
    m = model("tsb-test-scored.bin", 13)
    G, U = m.layers, m.units
    ids = synth.zipf_trace(30, G, U, 2, s=1.2, seed=51)
    res = [g * U + u for g in range(G) for u in range(3)]
    cfg = runtime.replay_config([U] * G, list(m.part_bytes), persistent_slots=len(res) + G, bank_slots=2,
                                blocks=G * U - len(res) + G, spare_target=G, order=res, tokens=ids.shape[0], n_ids=2,
                                wb_defer=wb_defer, round_every=5)
    r_ref = np.zeros((ids.shape[0], 6), dtype=np.uint64)
    oracle.ref_replay(cfg, ids, rstats=r_ref)
    assert r_ref[-1][0] == 6 and r_ref[-1][1] > 0
