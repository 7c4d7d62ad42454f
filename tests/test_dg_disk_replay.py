"""Slot-table parity of the device-gated cache's file tier (the reference's dg_disk_tier with synchronous reads) on the
CPU: this library's slot cache and the reference's own DgCore replay the same trace with pinned and file-homed units;
the slot table, the sixteen counters and the file tier's counters (reads, read bytes, staging waits, pinned units
dropped to their file, victims dropped to their file, file-homed units) must be identical after every token, and the
bytes found through the table must be each unit's own."""
import numpy as np
import pytest

import oracle
from tierstream_b200 import runtime, synth


def make_disk_case(G=6, U=16, parts=(2048, 2048, 4096), R=3, pinned=5, D=1, B=4, Q=None, S=4, tokens=40, s=1.1,
                   seed=11, n_pred=0, disk_prefetch=0, uniform=False, rho=0.0, home_extra=0, **kw):
    """G layers x U units: per layer the R most popular resident, the next `pinned` in pinned blocks, the rest in
    their files; Q spare blocks (default D per layer), S staging buffers; home_extra adds home blocks beyond the
    plan's pinned units (taken by disk units in priority order)."""
    ids = synth.zipf_trace(tokens, G, U, B, s=s, seed=seed, uniform=uniform, rho=rho)
    pop = synth.popularity_order(G, U, s=s, seed=seed)
    order, disk = [], [0] * (G * U)
    for g in range(G):
        order += [g * U + e for e in pop[g][:R]]
        for e in pop[g][R + pinned:]:
            disk[g * U + e] = 1
    P = G * (U - R) - sum(disk)
    Q = Q if Q is not None else D * G
    preds = synth.zipf_trace(tokens, G, U, n_pred, s=s, seed=seed + 1000) if n_pred else None
    cfg = runtime.replay_config([U] * G, list(parts), persistent_slots=len(order) + D * G, bank_slots=B,
                                blocks=P + home_extra + Q, spare_target=D * G, order=order, tokens=tokens, n_ids=B,
                                n_pred=n_pred, disk=disk, home_blocks=P + home_extra, disk_staging=S,
                                disk_prefetch=disk_prefetch, **kw)
    return cfg, ids, preds


CASES = {
    "files_and_pinned": dict(),
    "files_only": dict(pinned=0),
    "boundary_writebacks": dict(wb_defer=0),
    "deferred_on_demand_stream": dict(wb_on_d2h=0),
    "one_staging_buffer": dict(S=1),
    "few_spare_blocks": dict(Q=1, D=2),
    "many_spare_blocks": dict(Q=30),
    "home_blocks_beyond_the_plan": dict(home_extra=7),
    "predictions_demand_only_files": dict(n_pred=2),
    "predictions_read_files": dict(n_pred=2, disk_prefetch=1),
    "predictions_tight_budget": dict(n_pred=3, disk_prefetch=1, prefetch_per_layer=1, prefetch_per_token=4),
    "inclusive_share": dict(inclusive=4, Q=8),
    "uniform_routes": dict(uniform=True, pinned=2),
    "correlated_top8": dict(G=5, U=32, R=6, pinned=8, D=2, B=8, rho=0.5, s=0.9),
    "small_credit": dict(wb_layer_bytes=1024, wb_max_outstanding=4096),
}


def _compare(cfg, ids, preds, **kw):
    x_ref = np.zeros((cfg.tokens, 6), dtype=np.uint64)
    x_new = np.zeros((cfg.tokens, 6), dtype=np.uint64)
    t_ref, s_ref = oracle.ref_replay(cfg, ids, preds, xstats=x_ref, **kw)[:2]
    t_new, s_new = runtime.replay(cfg, ids, preds, xstats=x_new, **kw)[:2]
    for t in range(cfg.tokens):
        assert np.array_equal(t_new[t], t_ref[t]), "slot table differs after token %d" % t
        assert np.array_equal(s_new[t], s_ref[t]), "counters differ after token %d: %s vs %s" % (
            t, s_new[t].tolist(), s_ref[t].tolist())
        assert np.array_equal(x_new[t], x_ref[t]), "file tier counters differ after token %d: %s vs %s" % (
            t, x_new[t].tolist(), x_ref[t].tolist())
    return s_new, x_new


@pytest.mark.parametrize("name", sorted(CASES))
def test_file_tier_tables_match_reference(ref, name):
    cfg, ids, preds = make_disk_case(**CASES[name])
    s, x = _compare(cfg, ids, preds)
    assert s[-1][2] > 0 and x[-1][0] > 0, "the case must read units from their files"


def test_file_tier_drops_and_discards(ref):
    """Few blocks: write-backs need pinned units dropped to their files, and with none left victims go to theirs."""
    cfg, ids, preds = make_disk_case(G=4, U=16, R=2, pinned=1, D=3, Q=1, tokens=60, s=0.8)
    _, x = _compare(cfg, ids, preds)
    assert x[-1][3] > 0, "pinned units dropped to their files"
    assert x[-1][4] > 0, "victims dropped to their files"


def test_file_tier_bytes_through_the_table(ref):
    """Every unit found through the table after a layer's demand holds its own bytes, read from its file when it
    lives there, identically in both replays."""
    G, U, parts = 4, 12, (256, 512, 256)
    cfg, ids, preds = make_disk_case(G=G, U=U, parts=parts, R=2, pinned=3, D=1, B=2, tokens=30, n_pred=2,
                                     disk_prefetch=1)
    cfg.move_bytes = 1
    unit = sum(parts)
    src = np.random.default_rng(5).integers(0, 256, size=G * U * unit, dtype=np.uint8)
    r_new = runtime.replay(cfg, ids, preds, src_units=src, want_reads=True)[2]
    r_ref = oracle.ref_replay(cfg, ids, preds, src_units=src, want_reads=True)[2]
    assert np.array_equal(r_new, r_ref)
    orc = oracle.orc()
    want = [orc.orc_checksum(src[k * unit:].ctypes.data, unit) for k in range(G * U)]
    for t in range(cfg.tokens):
        for g in range(G):
            for i in range(cfg.n_ids):
                assert r_new[t, g, i] == want[g * U + int(ids[t, g, i])], (t, g, i)


def test_file_tier_refuses_bad_options():
    with pytest.raises(Exception, match="staging"):
        cfg, ids, _ = make_disk_case(S=0, tokens=2)
        runtime.replay(cfg, ids)


def random_disk_case(seed):
    r = np.random.default_rng(10_000 + seed)
    G = int(r.integers(2, 8))
    U = int(r.choice([4, 8, 16, 32]))
    B = int(r.integers(1, min(U, 8) + 1))
    R = int(r.integers(0, U - 1))
    pinned = int(r.integers(0, U - R))
    D = int(r.integers(1, max(2, min(4, U - R)) + 1))
    D = min(D, U - R)
    kw = dict(G=G, U=U, B=B, R=R, pinned=pinned, D=D, Q=int(r.integers(1, D * G + 6)), S=int(r.integers(1, 6)),
              tokens=int(r.integers(10, 40)), seed=int(r.integers(1, 10 ** 6)),
              parts=tuple(int(x) * 256 for x in r.integers(1, 9, size=int(r.integers(1, 4)))),
              wb_defer=int(r.integers(0, 2)), wb_on_d2h=int(r.integers(0, 2)),
              home_extra=int(r.integers(0, 4)) if r.random() < 0.3 else 0)
    trace = r.integers(0, 3)
    if trace == 0:
        kw["uniform"] = True
    elif trace == 1:
        kw["s"] = float(r.uniform(0.6, 1.4))
    else:
        kw["s"] = float(r.uniform(0.6, 1.2))
        kw["rho"] = float(r.uniform(0.2, 0.8))
    if r.random() < 0.5:
        kw["n_pred"] = int(r.integers(1, min(U, 4) + 1))
        kw["disk_prefetch"] = int(r.integers(0, 2))
        kw["prefetch_per_layer"] = int(r.integers(1, 5))
        kw["prefetch_per_token"] = int(r.integers(2, 49))
        if r.random() < 0.5:
            kw["prefetch_reserve"] = int(r.integers(0, 3))
    if r.random() < 0.3:
        kw["wb_layer_bytes"] = int(r.integers(1, 8)) * 1024
        kw["wb_max_outstanding"] = int(r.integers(1, 16)) * 4096
    if r.random() < 0.3 and kw["Q"] > 1:
        kw["inclusive"] = int(r.integers(1, kw["Q"]))
    return kw


@pytest.mark.parametrize("seed", range(150))
def test_random_file_tier_configurations_match_reference(ref, seed):
    kw = random_disk_case(seed)
    cfg, ids, preds = make_disk_case(**kw)
    try:
        _compare(cfg, ids, preds)
    except AssertionError as e:
        raise AssertionError("case %s: %s" % (kw, e))


@pytest.mark.parametrize("name,kw", [
    ("two_tier", dict(disk=False)),
    ("two_tier_inclusive", dict(disk=False, inclusive=4, Q=8)),
    ("files_and_pinned", dict()),
    ("files_only", dict(pinned=0)),
    ("file_predictions", dict(n_pred=2, disk_prefetch=1)),
    ("deferred_on_demand_stream", dict(wb_on_d2h=0, pinned=2)),
])
def test_reset_open_mid_trace_matches_reference(ref, name, kw):
    """ss_dg_reset_open between two tokens (after token 19 of 40): both caches restore the open placement, moving
    only misplaced units (file units read back into their open slot or block, units whose open home is their file
    dropped); the tables, counters and file counters stay identical, and every unit read through the table after the
    reset, with real bytes, is its own."""
    disk = kw.pop("disk", True)
    G, U, parts = 4, 12, (256, 512, 256)
    if disk:
        cfg, ids, preds = make_disk_case(G=G, U=U, parts=parts, R=2, D=1, B=2, tokens=40, s=0.7, **kw)
    else:
        from test_dg_replay import make_case
        cfg, ids, preds = make_case(G=G, U=U, parts=parts, R=2, D=1, B=2, tokens=40, s=0.7, **kw)
    cfg.move_bytes = 1
    cfg.reset_at = 20
    unit = sum(parts)
    src = np.random.default_rng(9).integers(0, 256, size=G * U * unit, dtype=np.uint8)
    x_ref = np.zeros((cfg.tokens, 6), dtype=np.uint64)
    x_new = np.zeros((cfg.tokens, 6), dtype=np.uint64)
    t_ref, s_ref, r_ref = oracle.ref_replay(cfg, ids, preds, src_units=src, want_reads=True, xstats=x_ref)
    t_new, s_new, r_new = runtime.replay(cfg, ids, preds, src_units=src, want_reads=True, xstats=x_new)
    for t in range(cfg.tokens):
        assert np.array_equal(t_new[t], t_ref[t]), "slot table differs after token %d" % t
        assert np.array_equal(s_new[t], s_ref[t]), "counters differ after token %d" % t
        assert np.array_equal(x_new[t], x_ref[t]), "file counters differ after token %d" % t
    assert np.array_equal(r_new, r_ref)
    # the table right after the reset is the open one: the same as after a reset following the first token
    cfg.reset_at = 1
    t_first = runtime.replay(cfg, ids, preds)[0]
    assert np.array_equal(t_new[19], t_first[0])
    assert not np.array_equal(t_new[18], t_new[19]), "the reset must have moved units"
    orc = oracle.orc()
    want = [orc.orc_checksum(src[k * unit:].ctypes.data, unit) for k in range(G * U)]
    for t in range(cfg.tokens):
        for g in range(G):
            for i in range(cfg.n_ids):
                assert r_new[t, g, i] == want[g * U + int(ids[t, g, i])], (t, g, i)
