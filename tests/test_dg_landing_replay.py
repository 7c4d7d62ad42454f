"""Slot-table parity of dg_landing_blocks on the CPU. A prediction of a file-homed unit reads it into one of the
landing blocks instead of a slot (nothing evicted, outside the prefetch budgets); a demand copies it from there; at
TTL 0 a landing its layer did not route goes back to its file right after that layer's demand, at TTL N after N
boundaries without a demand; a layer's misses whose landing read still runs are fetched after its other misses. The
reference's rules are in its src/dg_core.cpp:440-612 (advice, reads, expiry), 1146-1162 and 1309-1324 (a demand of a
landing), 1439-1460 (the demand's order and the TTL 0 expiry), 1633 (predictions), 1648-1662 (the boundary),
2499-2511 (ss_dg_make_resident from a landing block) and 2997-2999 (reset). Tables, the sixteen counters, the file
counters and the landing counters (issued, promoted, late, expired, dropped for want of a block, bytes read, expired
at their layer, skipped for a passed layer, units landed) are identical with the reference DgCore after every token,
alone and with the other features; the units read through the table hold their own bytes."""
import numpy as np
import pytest

import oracle
from tierstream_b200 import runtime

from test_dg_disk_replay import make_disk_case


def _compare(cfg, ids, preds, **kw):
    T = cfg.tokens
    x = [np.zeros((T, 6), dtype=np.uint64) for _ in range(2)]
    lst = [np.zeros((T, 9), dtype=np.uint64) for _ in range(2)]
    k = [np.zeros((T, 4), dtype=np.uint64) for _ in range(2)]
    t_ref, s_ref = oracle.ref_replay(cfg, ids, preds, xstats=x[0], lstats=lst[0], kstats=k[0], **kw)[:2]
    t_new, s_new = runtime.replay(cfg, ids, preds, xstats=x[1], lstats=lst[1], kstats=k[1], **kw)[:2]
    for t in range(T):
        assert np.array_equal(t_new[t], t_ref[t]), "slot table differs after token %d" % t
        assert np.array_equal(s_new[t], s_ref[t]), "counters differ after token %d: %s vs %s" % (
            t, s_new[t].tolist(), s_ref[t].tolist())
        assert np.array_equal(x[1][t], x[0][t]), "file counters differ after token %d" % t
        assert np.array_equal(lst[1][t], lst[0][t]), "landing counters differ after token %d: %s vs %s" % (
            t, lst[1][t].tolist(), lst[0][t].tolist())
        assert np.array_equal(k[1][t], k[0][t]), "the pinned recency order differs after token %d" % t
    return s_new[-1], x[1][-1], lst[1][-1]


CASES = {
    "ttl0": dict(landing_blocks=4, n_pred=2, disk_queue=3),
    "ttl0_one_block": dict(landing_blocks=1, n_pred=3, disk_queue=3),
    "ttl0_many_blocks": dict(landing_blocks=32, n_pred=3, disk_queue=3),
    "ttl1": dict(landing_blocks=4, landing_ttl=1, n_pred=2, disk_queue=3),
    "ttl2": dict(landing_blocks=4, landing_ttl=2, n_pred=3, disk_queue=3),
    "ttl5_few_blocks": dict(landing_blocks=2, landing_ttl=5, n_pred=3, disk_queue=3, pinned=2),
    "files_only": dict(landing_blocks=6, n_pred=3, disk_queue=3, pinned=0),
    "with_disk_prefetch": dict(landing_blocks=4, n_pred=3, disk_queue=3, disk_prefetch=1),
    "with_bank_keep": dict(landing_blocks=4, landing_ttl=1, n_pred=2, disk_queue=3, bank_keep=2, Q=1),
    "with_clean_evict": dict(landing_blocks=4, n_pred=2, disk_queue=3, clean_evict=1, Q=1, D=2),
    "with_pf_revert": dict(landing_blocks=4, landing_ttl=2, n_pred=3, disk_queue=3, pf_revert=1, pinned=2),
    "with_rounds": dict(landing_blocks=4, landing_ttl=3, n_pred=2, disk_queue=3, round_every=4),
    "scored": dict(landing_blocks=4, landing_ttl=1, n_pred=2, disk_queue=3, policy=1, D=2),
    "boundary_writebacks": dict(landing_blocks=4, n_pred=2, disk_queue=3, wb_defer=0),
    "synchronous_reads": dict(landing_blocks=4, landing_ttl=1, n_pred=2),
    "correlated_top8": dict(landing_blocks=16, landing_ttl=1, G=5, U=32, R=6, pinned=8, D=2, B=8, n_pred=8,
                            rho=0.5, s=0.9, disk_queue=4),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_landings_match_reference(ref, name):
    cfg, ids, preds = make_disk_case(**CASES[name])
    _, x, lst = _compare(cfg, ids, preds)
    assert lst[0] > 0 and lst[1] > 0, "the case must land units and promote some"
    if "ttl0" in name or name in ("files_only", "with_disk_prefetch", "with_clean_evict", "boundary_writebacks"):
        assert lst[6] > 0, "TTL 0: landings expire at their layer"
    if name.startswith("ttl") and "ttl0" not in name:
        assert lst[3] > 0, "landings expire at the boundary"


def test_landings_with_kept_resident_layers(ref):
    """ss_dg_make_resident of units landed by the previous token's predictions copies them from their landing
    blocks."""
    G, U = 6, 16
    events = [(t, 1 + t % 4, sorted({int(x) for x in np.random.default_rng(t).integers(0, U, 3)})) for t in (5, 12, 20)]
    events += [(28, 1, ())]
    cfg, ids, preds = make_disk_case(landing_blocks=8, landing_ttl=3, n_pred=3, disk_queue=3, resident_events=events,
                                     G=G, U=U, R=2, pinned=3, D=2, tokens=40)
    _compare(cfg, ids, preds)


def test_landings_across_a_reset(ref):
    cfg, ids, preds = make_disk_case(landing_blocks=4, landing_ttl=2, n_pred=3, disk_queue=3, tokens=40)
    cfg.reset_at = 20
    _, _, lst = _compare(cfg, ids, preds)
    assert lst[0] > 0


def test_landed_bytes_through_the_table(ref):
    """Every unit found through the table holds its own bytes, promoted from a landing block or read as any file
    miss, identically in both replays."""
    G, U, parts = 4, 12, (256, 512, 256)
    cfg, ids, preds = make_disk_case(G=G, U=U, parts=parts, R=2, pinned=2, D=1, B=2, tokens=30, n_pred=3,
                                     landing_blocks=4, landing_ttl=1, disk_queue=3)
    cfg.move_bytes = 1
    unit = sum(parts)
    src = np.random.default_rng(6).integers(0, 256, size=G * U * unit, dtype=np.uint8)
    lst = np.zeros((cfg.tokens, 9), dtype=np.uint64)
    r_new = runtime.replay(cfg, ids, preds, src_units=src, want_reads=True, lstats=lst)[2]
    r_ref = oracle.ref_replay(cfg, ids, preds, src_units=src, want_reads=True)[2]
    assert np.array_equal(r_new, r_ref)
    assert lst[-1][1] > 0, "some demands were served from landing blocks"
    orc = oracle.orc()
    want = [orc.orc_checksum(src[k * unit:].ctypes.data, unit) for k in range(G * U)]
    for t in range(cfg.tokens):
        for g in range(G):
            for i in range(cfg.n_ids):
                assert r_new[t, g, i] == want[g * U + int(ids[t, g, i])], (t, g, i)


def test_landings_off_change_nothing(ref):
    """landing_blocks 0: predictions of file units are prefetches (or nothing) as before; no landing counter moves."""
    cfg, ids, preds = make_disk_case(n_pred=3, disk_queue=3, disk_prefetch=1)
    _, _, lst = _compare(cfg, ids, preds)
    assert not lst.any()


@pytest.mark.parametrize("seed", range(30))
def test_landing_fuzz(ref, seed):
    r = np.random.default_rng(61_000 + seed)
    G = int(r.integers(2, 7))
    U = int(r.choice([8, 16, 32]))
    B = int(r.choice([2, 4, 8]))
    kw = dict(G=G, U=U, R=int(r.integers(1, U // 4 + 1)), pinned=int(r.integers(0, U // 2)),
              D=int(r.integers(1, 3)), B=B, Q=int(r.integers(0, 2 * G + 1)), S=int(r.integers(1, 5)),
              tokens=int(r.integers(20, 50)), s=float(r.choice([0.8, 1.1, 1.4])), seed=int(r.integers(0, 1000)),
              n_pred=int(r.integers(1, B + 1)), landing_blocks=int(r.integers(1, 24)),
              landing_ttl=int(r.choice([0, 0, 1, 2, 4])), disk_queue=int(r.choice([0, 2, 3, 4])),
              wb_defer=int(r.integers(0, 2)), rho=float(r.choice([0.0, 0.5])))
    if r.random() < 0.3:
        kw["disk_prefetch"] = 1
    if r.random() < 0.3:
        kw["bank_keep"] = int(r.integers(1, 3))
    if r.random() < 0.2:
        kw["clean_evict"] = 1
    if r.random() < 0.2:
        kw["pf_revert"] = 1
    if r.random() < 0.3:
        kw["policy"] = int(r.integers(1, 3))
    if r.random() < 0.3:
        kw["round_every"] = int(r.integers(3, 7))
    cfg, ids, preds = make_disk_case(**kw)
    if r.random() < 0.2:
        cfg.reset_at = int(r.integers(2, kw["tokens"]))
    _compare(cfg, ids, preds)
