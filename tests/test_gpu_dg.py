"""Device-gated decode on the GPU through the C ABI: every routed unit's bytes read by the engine's kernels equal the
source bytes (the oracle's checksum of the model file), the slot table after every token equals the reference
DgCore's on the same trace (deterministic schedule), and the failure paths end the token with an error instead of a
hang."""
import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle  # noqa: E402
from tierstream_b200 import abi, harness, runtime, synth  # noqa: E402


def expected_sums(model, orc):
    """oracle checksum of every unit, layer-major."""
    out = np.zeros(model.layers * model.units, dtype=np.uint64)
    buf = np.empty(model.unit_bytes, dtype=np.uint8)
    for L in range(model.layers):
        for u in range(model.units):
            orc.orc_fill_bytes(model.seed, model.unit_offset(L, u), model.unit_bytes, buf.ctypes.data)
            out[L * model.units + u] = orc.orc_checksum(buf.ctypes.data, model.unit_bytes)
    return out


@pytest.fixture(scope="module")
def small_model():
    m = synth.Model(os.path.join(harness.model_dir(), "tsb-test-small.bin"), layers=6, units=16,
                    part_bytes=(2048, 2048, 4096), seed=3, top_k=2, with_hash=True, base=0)
    m.write()
    return m


def run_tokens(run, ids, want, preds=None):
    for t in range(ids.shape[0]):
        got = run.step(ids[t], preds[t] if preds is not None else None)
        keys = np.arange(run.G)[:, None] * run.U + ids[t]
        assert np.array_equal(got, want[keys]), "token %d read wrong bytes" % t


def replay_cfg_for(run, model, ids):
    P = model.layers * model.units - len(run.resident_keys)
    return runtime.replay_config([model.units] * model.layers, list(model.part_bytes),
                                 persistent_slots=len(run.resident_keys) + model.layers, bank_slots=run.n_ids,
                                 blocks=P + model.layers, spare_target=model.layers, order=run.resident_keys,
                                 tokens=ids.shape[0], n_ids=run.n_ids)


@pytest.mark.parametrize("copy_mode", ["kernel", "ce"])
def test_bytes_and_tables_match_reference(small_model, orc, ref, monkeypatch, copy_mode):
    monkeypatch.setenv("TSB_DG_DETERMINISTIC", "1")
    monkeypatch.setenv("TSB_COPY_MODE", copy_mode)
    m = small_model
    ids = synth.zipf_trace(40, m.layers, m.units, 2, s=1.1, seed=11)
    run = harness.DgRun(m, residents_per_layer=3, max_ids=2, verify=True)
    try:
        want = expected_sums(m, orc)
        t_ref, s_ref = oracle.ref_replay(replay_cfg_for(run, m, ids), ids)
        for t in range(ids.shape[0]):
            got = run.step(ids[t])
            keys = np.arange(m.layers)[:, None] * m.units + ids[t]
            assert np.array_equal(got, want[keys]), "token %d read wrong bytes" % t
            assert np.array_equal(run.ctx.table(run.keys), t_ref[t]), "slot table differs after token %d" % t
        st = run.ctx.stats()
        assert st["misses"] == s_ref[-1][2] and st["fetched"] == s_ref[-1][4] and st["evicted"] == s_ref[-1][10]
        assert st["misses"] > 20
        chk = json.loads(run.ctx.stats_json())["check"]  # every landing hashed on the device, none differed
        assert chk["on"] == 1 and chk["units"] >= st["fetched"] and chk["mismatches"] == 0
        run.ctx.check()
        for L in range(m.layers):
            for u in range(m.units):
                run.ctx.check_unit(L, u)
    finally:
        run.close()


@pytest.mark.parametrize("mode,label", [("ce", "copy-engine"), ("kernel", "land-kernel")])
def test_c2_part_size_movers_match_reference(orc, ref, monkeypatch, mode, label):
    """The benchmark's part size (3 x 33,030,144-byte parts, a 99 MB expert) on both movers: the
    copy engines with stream-written entries and ready words, and the land kernel, whose batches of such parts are cut
    into 4 MiB pieces taken round-robin: 4 layers x 8 experts, 3 residents and 1 spare slot per layer, Zipf(1.1)
    top-2, descriptor hashes checked at the open and every landing hashed on the device. After every token the
    device's slot table equals the reference DgCore's replay, and every routed unit read through the table has the
    oracle's checksum of its source bytes."""
    monkeypatch.setenv("TSB_DG_DETERMINISTIC", "1")
    monkeypatch.setenv("TSB_COPY_MODE", mode)
    path = os.path.join(harness.model_dir(), "tsb-test-c2-parts.bin")
    m = synth.Model(path, layers=4, units=8, part_bytes=(33030144,) * 3, seed=7, top_k=2, with_hash=True)
    m.write()
    ids = synth.zipf_trace(24, m.layers, m.units, 2, s=1.1, seed=21)
    run = harness.DgRun(m, residents_per_layer=3, max_ids=2, verify=True)
    try:
        assert '"copy":"%s"' % label in run.ctx.stats_json()
        want = {}
        buf = np.empty(m.unit_bytes, dtype=np.uint8)
        for k in np.unique((np.arange(m.layers)[None, :, None] * m.units + ids).reshape(-1)):
            orc.orc_fill_bytes(m.seed, m.unit_offset(int(k) // m.units, int(k) % m.units), m.unit_bytes,
                               buf.ctypes.data)
            want[int(k)] = orc.orc_checksum(buf.ctypes.data, m.unit_bytes)
        t_ref, s_ref = oracle.ref_replay(replay_cfg_for(run, m, ids), ids)
        for t in range(ids.shape[0]):
            got = run.step(ids[t])
            for L in range(m.layers):
                for i in range(2):
                    assert int(got[L, i]) == want[L * m.units + int(ids[t, L, i])], "token %d layer %d" % (t, L)
            assert np.array_equal(run.ctx.table(run.keys), t_ref[t]), "slot table differs after token %d" % t
        st = run.ctx.stats()
        assert st["misses"] == s_ref[-1][2] and st["fetched"] == s_ref[-1][4] and st["evicted"] == s_ref[-1][10]
        assert st["misses"] > 10
        chk = json.loads(run.ctx.stats_json())["check"]
        assert chk["on"] == 1 and chk["units"] >= st["fetched"] and chk["mismatches"] == 0
        run.ctx.check()
    finally:
        run.close()
        for f in (path, path + ".xxh64"):
            if os.path.exists(f):
                os.unlink(f)


def test_landing_check_reports_and_repairs_a_corrupt_block(small_model, orc):
    """With verify_hash and descriptor hashes, every unit landed in a slot is hashed on the device and compared with its
    descriptor hash. A byte flipped in a pinned block (tsb_test_dg_corrupt) lands wrong on the unit's next miss: the
    ss_end of that token or of one of the next two fails with SS_E_HASH (not poisoned), the unit is read again from
    its file into its slot and its block, and every later token reads every routed unit's source bytes."""
    m = small_model
    run = harness.DgRun(m, residents_per_layer=3, max_ids=2, verify=True)
    try:
        want = expected_sums(m, orc)
        ids = synth.zipf_trace(24, m.layers, m.units, 2, s=1.1, seed=31)
        for t in range(5):
            got = run.step(ids[t])
            keys = np.arange(m.layers)[:, None] * m.units + ids[t]
            assert np.array_equal(got, want[keys]), "clean token %d read wrong bytes" % t
        table = run.ctx.table(run.keys)
        L = 2
        victim = next(u for u in range(m.units) if table[L * m.units + u] < 0)
        other = next(u for u in range(m.units) if u != victim)
        for t in (5, 9):  # routed on the token after the flip, and again after the repair
            ids[t, L] = [victim, other]
        abi.check(abi.load().tsb_test_dg_corrupt(run.ctx.h, L, victim, 1000))
        failed_at = None
        for t in (5, 6, 7):
            try:
                run.step(ids[t])
            except abi.TsError as e:
                assert e.status == abi.SS_E_HASH, str(e)
                assert "(%d, %d)" % (L, victim) in str(e)
                failed_at = t
                break
        assert failed_at is not None, "the flipped byte was not reported by the ss_end of its token or the next two"
        for t in range(failed_at + 1, ids.shape[0]):
            got = run.step(ids[t])
            keys = np.arange(m.layers)[:, None] * m.units + ids[t]
            assert np.array_equal(got, want[keys]), "token %d after the repair read wrong bytes" % t
        chk = json.loads(run.ctx.stats_json())["check"]
        assert chk["on"] == 1 and chk["mismatches"] == 1 and chk["repaired"] >= 1 and chk["units"] > 20
        run.ctx.check()
        for u in range(m.units):
            run.ctx.check_unit(L, u)
    finally:
        run.close()


def test_predictions_and_boundary_writebacks(small_model, orc):
    m = small_model
    ids = synth.zipf_trace(30, m.layers, m.units, 2, s=0.9, seed=5)
    preds = synth.zipf_trace(30, m.layers, m.units, 2, s=0.9, seed=6)
    run = harness.DgRun(m, residents_per_layer=2, spare_per_layer=2, max_ids=2, n_pred=2, wb_defer=0)
    try:
        run_tokens(run, ids, expected_sums(m, orc), preds)
        st = run.ctx.stats()
        assert st["prefetched"] > 0 and st["writebacks_done"] > 0
        run.ctx.check()
    finally:
        run.close()


def test_reset_open_restores_placement(small_model, orc, monkeypatch):
    monkeypatch.setenv("TSB_DG_DETERMINISTIC", "1")
    m = small_model
    run = harness.DgRun(m, residents_per_layer=3, max_ids=2)
    try:
        open_table = run.ctx.table(run.keys).copy()
        want = expected_sums(m, orc)
        run_tokens(run, synth.zipf_trace(25, m.layers, m.units, 2, s=0.5, seed=9), want)
        assert not np.array_equal(run.ctx.table(run.keys), open_table)
        run.ctx.reset_open()
        assert np.array_equal(run.ctx.table(run.keys), open_table)
        run.ctx.check()
        for L in range(m.layers):
            for u in range(m.units):
                run.ctx.check_unit(L, u)
        run_tokens(run, synth.zipf_trace(5, m.layers, m.units, 2, s=0.5, seed=10), want)
    finally:
        run.close()


def test_bad_id_fails_the_token(small_model):
    m = small_model
    run = harness.DgRun(m, residents_per_layer=3, max_ids=2, timeout_ms=2000)
    try:
        ids = synth.zipf_trace(1, m.layers, m.units, 2, seed=1)[0].copy()
        ids[2, 1] = m.units + 3
        with pytest.raises(abi.TsError) as e:
            run.step(ids)
        assert e.value.status == abi.SS_E_BACKEND and "out of range" in str(e.value)
        with pytest.raises(abi.TsError):  # poisoned
            run.ctx.begin()
    finally:
        run.close()


def test_stopped_service_times_out_on_the_device(small_model):
    """The wait kernel's bounded wait: nothing publishes ready, so it gives up after dg_wait_timeout_ms and the token
    fails on the host; no GPU fault or hang is involved."""
    m = small_model
    run = harness.DgRun(m, residents_per_layer=1, max_ids=2, timeout_ms=300)
    try:
        abi.check(abi.load().ss_test_dg_stop_service(run.ctx.h))
        ids = synth.zipf_trace(1, m.layers, m.units, 2, seed=2)[0]
        with pytest.raises(abi.TsError) as e:
            run.step(ids)
        assert e.value.status == abi.SS_E_BACKEND
    finally:
        run.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_context_on_another_device_keeps_the_callers_device(small_model):
    """A context opened (and driven, and closed) for device 1 from a thread whose current device is 0 runs there and
    leaves the thread on device 0 after every call."""
    m = small_model
    torch.cuda.set_device(1)
    run = harness.DgRun(m, residents_per_layer=3, max_ids=2)
    try:
        assert torch.cuda.current_device() == 1  # the open switched to device 1 and back
        torch.cuda.set_device(0)
        run.ctx.check()  # the library switches to device 1 inside the call and back
        assert torch.cuda.current_device() == 0
        torch.cuda.set_device(1)
        ids = synth.zipf_trace(3, m.layers, m.units, 2, s=1.0, seed=2)
        for t in range(3):
            run.step(ids[t])
        torch.cuda.set_device(0)
        run.ctx.check()
        assert torch.cuda.current_device() == 0
    finally:
        torch.cuda.set_device(1)
        run.close()
        torch.cuda.set_device(0)


@pytest.mark.parametrize("wb_defer", [0, 1])
def test_predictions_tables_match_reference(small_model, orc, ref, monkeypatch, wb_defer):
    """Next-layer predictions (ss_dg_enqueue_predict) under the deterministic schedule: the prefetches the service
    issues from them, and so the slot table after every token, equal the reference DgCore's replay with the same
    predictions; every routed unit's bytes are the source's."""
    monkeypatch.setenv("TSB_DG_DETERMINISTIC", "1")
    m = small_model
    ids = synth.zipf_trace(30, m.layers, m.units, 2, s=0.9, seed=15)
    preds = synth.zipf_trace(30, m.layers, m.units, 2, s=0.9, seed=16)
    run = harness.DgRun(m, residents_per_layer=3, max_ids=2, n_pred=2, wb_defer=wb_defer)
    try:
        P = m.layers * m.units - len(run.resident_keys)
        cfg = runtime.replay_config([m.units] * m.layers, list(m.part_bytes),
                                    persistent_slots=len(run.resident_keys) + m.layers, bank_slots=2,
                                    blocks=P + m.layers, spare_target=m.layers, order=run.resident_keys,
                                    tokens=ids.shape[0], n_ids=2, n_pred=2, wb_defer=wb_defer)
        t_ref, s_ref = oracle.ref_replay(cfg, ids, preds)
        want = expected_sums(m, orc)
        for t in range(ids.shape[0]):
            got = run.step(ids[t], preds[t])
            keys = np.arange(m.layers)[:, None] * m.units + ids[t]
            assert np.array_equal(got, want[keys]), "token %d read wrong bytes" % t
            assert np.array_equal(run.ctx.table(run.keys), t_ref[t]), "slot table differs after token %d" % t
        st = run.ctx.stats()
        assert st["prefetched"] == s_ref[-1][5] and st["prefetched"] > 0
    finally:
        run.close()


def test_predictions_from_the_previous_layer_match_reference(small_model, orc, ref, monkeypatch):
    """predict_prev: each layer's exported id buffer is also ss_dg_enqueue_predict's input for the next layer (read on
    the device, no host predictions), on a trace whose layers repeat their predecessor's experts with probability 0.5
    (BASELINE configs[3]'s correlation). Tables after every token equal the reference's replay given the same ids as
    predictions; every reader's bytes are right; some prefetches are used."""
    monkeypatch.setenv("TSB_DG_DETERMINISTIC", "1")
    m = small_model
    ids = synth.zipf_trace(30, m.layers, m.units, 2, s=0.9, seed=31, rho=0.5)
    run = harness.DgRun(m, residents_per_layer=3, max_ids=2, predict_prev=True)
    try:
        P = m.layers * m.units - len(run.resident_keys)
        cfg = runtime.replay_config([m.units] * m.layers, list(m.part_bytes),
                                    persistent_slots=len(run.resident_keys) + m.layers, bank_slots=2,
                                    blocks=P + m.layers, spare_target=m.layers, order=run.resident_keys,
                                    tokens=ids.shape[0], n_ids=2, n_pred=2)
        t_ref, s_ref = oracle.ref_replay(cfg, ids, ids)
        want = expected_sums(m, orc)
        for t in range(ids.shape[0]):
            got = run.step(ids[t])
            keys = np.arange(m.layers)[:, None] * m.units + ids[t]
            assert np.array_equal(got, want[keys]), "token %d read wrong bytes" % t
            assert np.array_equal(run.ctx.table(run.keys), t_ref[t]), "slot table differs after token %d" % t
        st = run.ctx.stats()
        assert st["prefetched"] == s_ref[-1][5] and st["prefetched"] > 0 and st["prefetch_used"] > 0
    finally:
        run.close()


def test_held_layers_match_reference(small_model, orc, ref, monkeypatch):
    """ss_dg_make_resident on the GPU: after chosen tokens a gated layer's units are made resident and held, and one is
    released later. The engine's graph neither exports nor waits for a held layer (its reader resolves the held units
    through ss_dg_slot). Tables after every token, the held-layer events applied, equal the reference's replay of the
    same events; every reader's bytes are right; check() after every token proves that each table entry the device
    does not hold yet is marked for the next upload (while a layer is held, uploads write only changed entries)."""
    monkeypatch.setenv("TSB_DG_DETERMINISTIC", "1")
    m = small_model
    G, U, T = m.layers, m.units, 30
    events = [(4, 2, (0, 5, 9)), (10, 4, (3, 7, 11)), (18, 2, ())]  # after that token: hold ids, () releases
    active = {}
    held_at = []
    for t in range(T):
        held_at.append(dict(active))
        for te, g, u in events:
            if te == t:
                if u:
                    active[g] = u
                else:
                    active.pop(g, None)
    ids = synth.zipf_trace(T, G, U, 2, s=0.9, seed=51)
    rng = np.random.default_rng(52)
    for t in range(T):  # a held layer routes only to its held units
        for g, u in held_at[t].items():
            ids[t, g] = rng.choice(np.array(u), size=2, replace=False)
    run = harness.DgRun(m, residents_per_layer=3, max_ids=2, wb_defer=1)
    try:
        P = G * U - len(run.resident_keys)
        cfg = runtime.replay_config([U] * G, list(m.part_bytes), persistent_slots=len(run.resident_keys) + G,
                                    bank_slots=2, blocks=P + G, spare_target=G, order=run.resident_keys, tokens=T,
                                    n_ids=2, wb_defer=1, resident_events=events)
        t_ref, s_ref = oracle.ref_replay(cfg, ids)
        want = expected_sums(m, orc)
        for t in range(T):
            held = [g in held_at[t] for g in range(G)]
            got = run.step(ids[t], held=held)
            keys = np.arange(G)[:, None] * U + ids[t]
            assert np.array_equal(got, want[keys]), "token %d read wrong bytes" % t
            for te, g, u in events:
                if te == t:
                    run.ctx.make_resident(g, u)
            assert np.array_equal(run.ctx.table(run.keys), t_ref[t]), "slot table differs after token %d" % t
            run.ctx.check()
        st = run.ctx.stats()
        assert st["resident_units"] > 0 and st["misses"] == s_ref[-1][2]
    finally:
        run.close()


def file_tier_run(m, R=3, pinned=4, S=3, **kw):
    """A DgRun with the file tier: per layer units [0, R) resident, [R, R + pinned) pinned, the rest in the model file
    only (tier DISK)."""
    res = [g * m.units + u for g in range(m.layers) for u in range(R)]
    disk = [g * m.units + u for g in range(m.layers) for u in range(R + pinned, m.units)]
    run = harness.DgRun(m, resident_keys=res, max_ids=2, disk_keys=disk, disk_staging=S, **kw)
    return run, res, disk


def file_tier_cfg(run, m, res, disk, ids, S, **kw):
    flags = [0] * (m.layers * m.units)
    for k in disk:
        flags[k] = 1
    P = m.layers * m.units - len(res) - len(disk)
    return runtime.replay_config([m.units] * m.layers, list(m.part_bytes), persistent_slots=len(res) + m.layers,
                                 bank_slots=run.n_ids, blocks=P + m.layers, spare_target=m.layers, order=res,
                                 tokens=ids.shape[0], n_ids=run.n_ids, disk=flags, home_blocks=P, disk_staging=S,
                                 **kw)


@pytest.mark.parametrize("wb_defer", [0, 1])
def test_file_tier_bytes_and_tables_match_reference(small_model, orc, ref, monkeypatch, wb_defer):
    """The file tier (dg_disk_tier, synchronous reads): units of tier DISK are read from the model file into a pinned
    staging buffer on their miss and copied from there; every routed unit's bytes are the source's, and the slot table
    and the file tier's counters after every token equal the reference DgCore's replay."""
    monkeypatch.setenv("TSB_DG_DETERMINISTIC", "1")
    m = small_model
    ids = synth.zipf_trace(40, m.layers, m.units, 2, s=0.8, seed=21)
    run, res, disk = file_tier_run(m, S=3, verify=True, wb_defer=wb_defer)
    try:
        cfg = file_tier_cfg(run, m, res, disk, ids, 3, wb_defer=wb_defer)
        x_ref = np.zeros((ids.shape[0], 6), dtype=np.uint64)
        t_ref, s_ref = oracle.ref_replay(cfg, ids, xstats=x_ref)
        want = expected_sums(m, orc)
        for t in range(ids.shape[0]):
            got = run.step(ids[t])
            keys = np.arange(m.layers)[:, None] * m.units + ids[t]
            assert np.array_equal(got, want[keys]), "token %d read wrong bytes" % t
            assert np.array_equal(run.ctx.table(run.keys), t_ref[t]), "slot table differs after token %d" % t
        st = run.ctx.stats()
        assert st["misses"] == s_ref[-1][2] and st["evicted"] == s_ref[-1][10]
        assert st["disk_reads"] == x_ref[-1][0] > 0 and st["disk_read_bytes"] == x_ref[-1][1]
        assert st["disk_drops"] == x_ref[-1][3] and st["disk_discards"] == x_ref[-1][4]
        assert st["disk_units"] == x_ref[-1][5]
        run.ctx.check()
        for L in range(m.layers):
            for u in range(m.units):
                run.ctx.check_unit(L, u)
    finally:
        run.close()


@pytest.mark.parametrize("bank_keep", [1, 2])
def test_file_tier_bank_keep_matches_reference(small_model, orc, ref, monkeypatch, bank_keep):
    """dg_bank_keep: a bank-served file miss is read (and hashed) straight into a pinned block, which becomes its home
    when the bank lets it go (1: at the pinned recency front, 2: behind its front half), dropping the least recently
    homed pinned unit to its file when no block is free. Every routed unit's bytes are the source's; the slot table,
    the file counters and the option's counters after every token equal the reference DgCore's replay; every unit's
    live copy (a kept block included) holds its bytes at the end."""
    import json
    monkeypatch.setenv("TSB_DG_DETERMINISTIC", "1")
    m = small_model
    ids = synth.zipf_trace(40, m.layers, m.units, 2, s=0.8, seed=21)
    run, res, disk = file_tier_run(m, S=3, verify=True, bank_keep=bank_keep)
    try:
        cfg = file_tier_cfg(run, m, res, disk, ids, 3, bank_keep=bank_keep)
        x_ref = np.zeros((ids.shape[0], 6), dtype=np.uint64)
        k_ref = np.zeros((ids.shape[0], 4), dtype=np.uint64)
        t_ref, s_ref = oracle.ref_replay(cfg, ids, xstats=x_ref, kstats=k_ref)
        want = expected_sums(m, orc)
        for t in range(ids.shape[0]):
            got = run.step(ids[t])
            keys = np.arange(m.layers)[:, None] * m.units + ids[t]
            assert np.array_equal(got, want[keys]), "token %d read wrong bytes" % t
            assert np.array_equal(run.ctx.table(run.keys), t_ref[t]), "slot table differs after token %d" % t
        st = run.ctx.stats()
        assert st["misses"] == s_ref[-1][2] and st["bank_serves"] == s_ref[-1][8] > 0
        assert st["disk_reads"] == x_ref[-1][0] and st["disk_drops"] == x_ref[-1][3]
        dj = json.loads(run.ctx.stats_json())["dg"]  # (bank_kept: ss_dg_stats.bank_kept)
        assert dj["bank_keep"] == bank_keep and dj["bank_kept"] == k_ref[-1][0] > 0
        assert dj["bank_keep_drops"] == k_ref[-1][1] > 0 and dj["bank_keep_rereads"] == k_ref[-1][2]
        run.ctx.check()
        for L in range(m.layers):
            for u in range(m.units):
                run.ctx.check_unit(L, u)
    finally:
        run.close()


def test_file_tier_adaptive_read_depth(small_model, orc, ref, monkeypatch):
    """dg_disk_queue_adapt with reads in flight (dg_disk_queue AUTO, resolved to 3 with 3 staging buffers): the pool
    runs its demand reads at the depth its controller measures faster, 1 or 3; what is read does not change, so every
    routed unit's bytes and the slot table after every token equal the reference replay at a queue of 3, and the stats
    report the controller (on, calibrations begun, its depth, the reads it measured at each depth)."""
    import json
    monkeypatch.setenv("TSB_DG_DETERMINISTIC", "1")
    m = small_model
    ids = synth.zipf_trace(60, m.layers, m.units, 2, s=0.6, seed=27)
    run, res, disk = file_tier_run(m, S=3, verify=True, disk_queue=0xFFFFFFFF, disk_queue_adapt=1)
    try:
        cfg = file_tier_cfg(run, m, res, disk, ids, 3, disk_queue=3)
        x_ref = np.zeros((ids.shape[0], 6), dtype=np.uint64)
        t_ref, s_ref = oracle.ref_replay(cfg, ids, xstats=x_ref)
        want = expected_sums(m, orc)
        for t in range(ids.shape[0]):
            got = run.step(ids[t])
            keys = np.arange(m.layers)[:, None] * m.units + ids[t]
            assert np.array_equal(got, want[keys]), "token %d read wrong bytes" % t
            assert np.array_equal(run.ctx.table(run.keys), t_ref[t]), "slot table differs after token %d" % t
        st = run.ctx.stats()
        assert st["disk_reads"] == x_ref[-1][0] > 64 and st["misses"] == s_ref[-1][2]
        j = json.loads(run.ctx.stats_json())
        assert j["disk_queue_adapt"] == "on"
        dd = j["disk_depth"]
        assert dd["bound"] == 3 and dd["depth"] in (1, 3) and dd["calibrations"] >= 1 and dd["windows"] >= 1
        assert 0 < dd["reads_1"] + dd["reads_u"] <= st["disk_reads"]
        assert all(v["to"] in (1, 3) for v in dd["ring"])
        run.ctx.check()
        run.ctx.reset_open()  # a fresh calibration
        j = json.loads(run.ctx.stats_json())
        assert j["disk_depth"]["calibrations"] == 1 and j["disk_depth"]["windows"] == 0
    finally:
        run.close()


def test_file_tier_adaptive_read_depth_declined(small_model, monkeypatch):
    """dg_disk_queue_adapt is declined (the pool runs as without it, the stats say why) with a single reader and with
    file prefetches."""
    import json
    for kw, why in ((dict(S=1), "one reader"), (dict(S=3, n_pred=2, disk_prefetch=1), "file prefetches")):
        run, _, _ = file_tier_run(small_model, disk_queue=0xFFFFFFFF, disk_queue_adapt=1, **kw)
        try:
            assert json.loads(run.ctx.stats_json())["disk_queue_adapt"] == "declined: " + why
        finally:
            run.close()


@pytest.mark.parametrize("ttl", [0, 2])
def test_file_tier_landing_blocks_match_reference(small_model, orc, ref, monkeypatch, ttl):
    """dg_landing_blocks with reads in flight: predictions of file-homed units are read (and hashed) into landing
    blocks on the read pool behind the demand reads; a demand copies them from there; unrouted landings expire at
    their layer (TTL 0) or after 2 boundaries. Every routed unit's bytes are the source's, and the slot table, the file
    counters and the landing counters after every token equal the reference DgCore's replay."""
    import json
    monkeypatch.setenv("TSB_DG_DETERMINISTIC", "1")
    m = small_model
    ids = synth.zipf_trace(40, m.layers, m.units, 2, s=0.8, seed=29)
    preds = synth.zipf_trace(40, m.layers, m.units, 2, s=0.8, seed=30)
    run, res, disk = file_tier_run(m, pinned=2, S=3, n_pred=2, disk_queue=0xFFFFFFFF, landing_blocks=4,
                                   landing_ttl=ttl, verify=True)
    try:
        cfg = file_tier_cfg(run, m, res, disk, ids, 3, n_pred=2, disk_queue=3, landing_blocks=4, landing_ttl=ttl)
        x_ref = np.zeros((ids.shape[0], 6), dtype=np.uint64)
        l_ref = np.zeros((ids.shape[0], 9), dtype=np.uint64)
        t_ref, s_ref = oracle.ref_replay(cfg, ids, preds, xstats=x_ref, lstats=l_ref)
        want = expected_sums(m, orc)
        for t in range(ids.shape[0]):
            got = run.step(ids[t], preds[t])
            keys = np.arange(m.layers)[:, None] * m.units + ids[t]
            assert np.array_equal(got, want[keys]), "token %d read wrong bytes" % t
            assert np.array_equal(run.ctx.table(run.keys), t_ref[t]), "slot table differs after token %d" % t
        st = run.ctx.stats()
        assert st["misses"] == s_ref[-1][2] and st["disk_reads"] == x_ref[-1][0]
        lj = json.loads(run.ctx.stats_json())["landing"]
        assert lj["blocks"] == 4 and lj["ttl"] == ttl
        assert lj["issued"] == l_ref[-1][0] > 0 and lj["promoted"] == l_ref[-1][1] > 0
        assert lj["expired"] == l_ref[-1][3] and lj["dropped_full"] == l_ref[-1][4]
        assert lj["read_bytes"] == l_ref[-1][5] and lj["expired_layer"] == l_ref[-1][6]
        assert lj["units"] == l_ref[-1][8] and lj["failed"] == 0
        run.ctx.check()
        for L in range(m.layers):
            for u in range(m.units):
                run.ctx.check_unit(L, u)
        run.ctx.reset_open()  # landings back to their files, every landing block free
        assert json.loads(run.ctx.stats_json())["landing"]["units"] == 0
        run.ctx.check()
    finally:
        run.close()


def test_file_tier_predictions_read_files(small_model, orc, ref, monkeypatch):
    """dg_disk_prefetch: predictions read file units too (on the prefetch stream, covered by the demand's wait)."""
    monkeypatch.setenv("TSB_DG_DETERMINISTIC", "1")
    m = small_model
    ids = synth.zipf_trace(30, m.layers, m.units, 2, s=0.8, seed=23)
    preds = synth.zipf_trace(30, m.layers, m.units, 2, s=0.8, seed=24)
    run, res, disk = file_tier_run(m, pinned=2, S=2, n_pred=2, disk_prefetch=1)
    try:
        cfg = file_tier_cfg(run, m, res, disk, ids, 2, n_pred=2, disk_prefetch=1)
        x_ref = np.zeros((ids.shape[0], 6), dtype=np.uint64)
        t_ref, s_ref = oracle.ref_replay(cfg, ids, preds, xstats=x_ref)
        want = expected_sums(m, orc)
        for t in range(ids.shape[0]):
            got = run.step(ids[t], preds[t])
            keys = np.arange(m.layers)[:, None] * m.units + ids[t]
            assert np.array_equal(got, want[keys]), "token %d read wrong bytes" % t
            assert np.array_equal(run.ctx.table(run.keys), t_ref[t]), "slot table differs after token %d" % t
        st = run.ctx.stats()
        assert st["prefetched"] == s_ref[-1][5] > 0 and st["disk_reads"] == x_ref[-1][0]
    finally:
        run.close()


def test_file_tier_reset_open_reads_files_back(small_model, orc, monkeypatch):
    """ss_dg_reset_open with the file tier: units whose open home is their file give up their slot or block, units
    that came from their file to an open slot or block are read back; the open placement and every byte return."""
    monkeypatch.setenv("TSB_DG_DETERMINISTIC", "1")
    m = small_model
    run, _, _ = file_tier_run(m, R=2, pinned=3, S=2)
    try:
        open_table = run.ctx.table(run.keys).copy()
        want = expected_sums(m, orc)
        run_tokens(run, synth.zipf_trace(25, m.layers, m.units, 2, s=0.5, seed=29), want)
        assert run.ctx.stats()["disk_reads"] > 0
        assert not np.array_equal(run.ctx.table(run.keys), open_table)
        run.ctx.reset_open()
        assert np.array_equal(run.ctx.table(run.keys), open_table)
        run.ctx.check()
        for L in range(m.layers):
            for u in range(m.units):
                run.ctx.check_unit(L, u)
        run_tokens(run, synth.zipf_trace(5, m.layers, m.units, 2, s=0.5, seed=30), want)
    finally:
        run.close()
