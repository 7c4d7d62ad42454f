"""Slot-table parity of the file tier with reads in flight (dg_disk_queue 2..8: a miss's read begun in its fetch, its
copy and entry enqueued when it ends at a drain point; a prediction's read may run on past the service call that
began it) on the CPU, against the reference's own DgCore with the same queue depth: the tables, the sixteen counters,
the file counters and the queue's own (reads begun while another ran, the most in flight, reads ended in a later
call and their bytes) are identical after every token, and with real bytes every unit read through the table is its
own."""
import numpy as np
import pytest

import oracle
from tierstream_b200 import runtime

from test_dg_disk_replay import make_disk_case


def _compare(cfg, ids, preds, src=None):
    x = [np.zeros((cfg.tokens, 6), dtype=np.uint64) for _ in range(2)]
    q = [np.zeros((cfg.tokens, 4), dtype=np.uint64) for _ in range(2)]
    kw = dict(src_units=src, want_reads=src is not None)
    ref = oracle.ref_replay(cfg, ids, preds, xstats=x[0], qstats=q[0], **kw)
    new = runtime.replay(cfg, ids, preds, xstats=x[1], qstats=q[1], **kw)
    for t in range(cfg.tokens):
        assert np.array_equal(new[0][t], ref[0][t]), "slot table differs after token %d" % t
        assert np.array_equal(new[1][t], ref[1][t]), "counters differ after token %d" % t
        assert np.array_equal(x[1][t], x[0][t]), "file counters differ after token %d" % t
        assert np.array_equal(q[1][t], q[0][t]), "queue counters differ after token %d: %s vs %s" % (
            t, q[1][t].tolist(), q[0][t].tolist())
    if src is not None:
        assert np.array_equal(new[2], ref[2])
    return q[1][-1], new


CASES = {
    "queue_2": dict(disk_queue=2, S=4),
    "queue_4_top8": dict(disk_queue=4, S=8, G=4, U=32, R=4, pinned=4, D=2, B=8),
    "queue_8_more_than_staging": dict(disk_queue=8, S=3, B=4),
    "file_predictions_carried": dict(disk_queue=4, S=6, n_pred=3, disk_prefetch=1),
    "boundary_writebacks": dict(disk_queue=3, S=4, wb_defer=0, D=2),
    "with_rounds_and_scoring": dict(disk_queue=4, S=4, round_every=3, policy=1, D=2),
    "with_revert_and_clean_evict": dict(disk_queue=4, S=4, n_pred=2, disk_prefetch=1, pf_revert=1, clean_evict=1,
                                        Q=2, D=2),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_reads_in_flight_match_reference(ref, name):
    cfg, ids, preds = make_disk_case(**CASES[name])
    q, _ = _compare(cfg, ids, preds)
    assert q[0] > 0 and q[1] > 1, "reads must overlap"
    if name == "file_predictions_carried":
        assert q[2] > 0 and q[3] == q[2] * sum(cfg.part_bytes[i] for i in range(cfg.n_parts))


def test_reads_in_flight_bytes_and_reset(ref):
    G, U, parts = 4, 12, (256, 512, 256)
    cfg, ids, preds = make_disk_case(G=G, U=U, parts=parts, R=2, pinned=3, D=1, B=2, tokens=30, n_pred=2,
                                     disk_prefetch=1, disk_queue=3, S=3)
    cfg.move_bytes = 1
    cfg.reset_at = 16
    unit = sum(parts)
    src = np.random.default_rng(8).integers(0, 256, size=G * U * unit, dtype=np.uint8)
    _, new = _compare(cfg, ids, preds, src)
    orc = oracle.orc()
    want = [orc.orc_checksum(src[k * unit:].ctypes.data, unit) for k in range(G * U)]
    for t in range(cfg.tokens):
        for g in range(G):
            for i in range(cfg.n_ids):
                assert new[2][t, g, i] == want[g * U + int(ids[t, g, i])], (t, g, i)


def random_queue_case(seed):
    r = np.random.default_rng(50_000 + seed)
    G = int(r.integers(2, 7))
    U = int(r.choice([4, 8, 16, 32]))
    B = int(r.integers(1, min(U, 8) + 1))
    R = int(r.integers(0, U - 1))
    D = min(int(r.integers(1, 4)), U - R)
    kw = dict(G=G, U=U, B=B, R=R, D=D, pinned=int(r.integers(0, U - R)), Q=int(r.integers(1, D * G + 4)),
              S=int(r.integers(1, 9)), disk_queue=int(r.integers(1, 9)), tokens=int(r.integers(10, 35)),
              seed=int(r.integers(1, 10 ** 6)), wb_defer=int(r.integers(0, 2)), wb_on_d2h=int(r.integers(0, 2)),
              s=float(r.uniform(0.6, 1.4)))
    if r.random() < 0.6:
        kw["n_pred"] = int(r.integers(1, min(U, 4) + 1))
        kw["disk_prefetch"] = int(r.random() < 0.7)
    for opt in ("pf_revert", "clean_evict", "pf_strict"):
        if r.random() < 0.2:
            kw[opt] = 1
    if r.random() < 0.2:
        kw["round_every"] = int(r.integers(1, 6))
    if r.random() < 0.2:
        kw["policy"] = 1
    return kw


@pytest.mark.parametrize("seed", range(120))
def test_random_queue_configurations_match_reference(ref, seed):
    kw = random_queue_case(seed)
    cfg, ids, preds = make_disk_case(**kw)
    try:
        _compare(cfg, ids, preds)
    except AssertionError as e:
        raise AssertionError("case %s: %s" % (kw, e))
