"""Slot-table parity of placement rounds (ss_dg_round) on the CPU: rounds between tokens in this library's slot cache
and in the reference's own DgCore, on the same traces, move the same units: the table, the sixteen counters, the file
tier's counters and the rounds' sums (rounds, promoted to the device, promoted to pinned, demoted, dropped to their
file, bytes) are identical after every token. The cases vary the limits (units, bytes, hysteresis, decay), the
write-back stream of demotions, clean copies (inclusive shares), the file tier and scored eviction alongside."""
import numpy as np
import pytest

import oracle
from tierstream_b200 import runtime

from test_dg_disk_replay import make_disk_case
from test_dg_replay import make_case


def _compare(cfg, ids, preds):
    x = [np.zeros((cfg.tokens, 6), dtype=np.uint64) for _ in range(2)]
    r = [np.zeros((cfg.tokens, 6), dtype=np.uint64) for _ in range(2)]
    t_ref, s_ref = oracle.ref_replay(cfg, ids, preds, xstats=x[0], rstats=r[0])
    t_new, s_new = runtime.replay(cfg, ids, preds, xstats=x[1], rstats=r[1])
    for t in range(cfg.tokens):
        assert np.array_equal(t_new[t], t_ref[t]), "slot table differs after token %d" % t
        assert np.array_equal(s_new[t], s_ref[t]), "counters differ after token %d: %s vs %s" % (
            t, s_new[t].tolist(), s_ref[t].tolist())
        assert np.array_equal(x[1][t], x[0][t]), "file counters differ after token %d" % t
        assert np.array_equal(r[1][t], r[0][t]), "round sums differ after token %d: %s vs %s" % (
            t, r[1][t].tolist(), r[0][t].tolist())
    return r[1][-1]


CASES = {
    "every_5_tokens": dict(round_every=5),
    "every_token_boundary_writebacks": dict(round_every=1, wb_defer=0, D=2),
    "demotions_on_the_demand_stream": dict(round_every=3, wb_on_d2h=0),
    "few_units_per_round": dict(round_every=2, round_max_units=2),
    "byte_budget": dict(round_every=2, round_budget=3 * 8192 + 100),
    "high_hysteresis": dict(round_every=4, round_hysteresis=3.0),
    "no_decay": dict(round_every=4, round_decay=1.0),
    "full_decay": dict(round_every=4, round_decay=0.0),
    "clean_copies": dict(round_every=3, inclusive=6, Q=10),
    "with_predictions": dict(round_every=3, n_pred=2),
    "with_scored_eviction": dict(round_every=3, policy=1, D=2),
    "correlated_top8": dict(round_every=4, G=5, U=32, R=8, D=2, B=8, rho=0.5, s=0.9),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_rounds_match_reference(ref, name):
    cfg, ids, preds = make_case(**dict(dict(tokens=40, s=1.2), **CASES[name]))
    total = _compare(cfg, ids, preds)
    assert total[0] > 0
    if name not in ("high_hysteresis",):
        assert total[1] > 0, "the case must promote units to the device"


@pytest.mark.parametrize("kw", [dict(), dict(pinned=1, Q=2), dict(wb_defer=0, D=2), dict(n_pred=2, disk_prefetch=1),
                                dict(round_max_units=3), dict(round_budget=5 * 8192)])
def test_rounds_with_the_file_tier_match_reference(ref, kw):
    cfg, ids, preds = make_disk_case(tokens=40, s=1.2, round_every=3, **kw)
    total = _compare(cfg, ids, preds)
    assert total[0] > 0


def test_rounds_promote_file_units_to_pinned(ref):
    cfg, ids, preds = make_disk_case(G=4, U=16, R=2, pinned=4, D=1, tokens=60, s=1.3, round_every=4)
    total = _compare(cfg, ids, preds)
    assert total[2] > 0 and total[4] > 0, total


def random_round_case(seed):
    r = np.random.default_rng(30_000 + seed)
    G = int(r.integers(2, 7))
    U = int(r.choice([4, 8, 16, 32]))
    B = int(r.integers(1, min(U, 6) + 1))
    R = int(r.integers(0, U - 1))
    D = min(int(r.integers(1, 4)), U - R)
    kw = dict(G=G, U=U, B=B, R=R, D=D, tokens=int(r.integers(10, 40)), seed=int(r.integers(1, 10 ** 6)),
              wb_defer=int(r.integers(0, 2)), wb_on_d2h=int(r.integers(0, 2)), s=float(r.uniform(0.7, 1.5)),
              round_every=int(r.integers(1, 6)), round_max_units=int(r.integers(0, 12)),
              round_hysteresis=float(r.choice([1.0, 1.25, 2.0])), round_decay=float(r.choice([0.0, 0.5, 0.85, 1.0])),
              round_budget=int(r.choice([0, 1, 4])) * 8192 * 3)
    if r.random() < 0.3:
        kw["n_pred"] = int(r.integers(1, min(U, 3) + 1))
    if r.random() < 0.3:
        kw["policy"] = 1
    disk = r.random() < 0.5
    if disk:
        kw["pinned"] = int(r.integers(0, U - R))
        kw["S"] = int(r.integers(1, 4))
        kw["Q"] = int(r.integers(1, D * G + 3))
    else:
        kw["Q"] = D * G + int(r.integers(0, 4))
    if r.random() < 0.25 and kw["Q"] > 1:
        kw["inclusive"] = int(r.integers(1, kw["Q"]))
    return kw, disk


@pytest.mark.parametrize("seed", range(100))
def test_random_round_configurations_match_reference(ref, seed):
    kw, disk = random_round_case(seed)
    cfg, ids, preds = (make_disk_case if disk else make_case)(**kw)
    try:
        _compare(cfg, ids, preds)
    except AssertionError as e:
        raise AssertionError("case %s: %s" % (kw, e))
