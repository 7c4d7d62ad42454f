"""Randomized slot-table parity of the device-gated cache on the CPU: seeded random configurations (layer and unit
counts, residents, spare slots, bank width, spare blocks, write-back scheduling and credit, inclusive shares,
prediction budgets, Zipf / uniform / correlated traces) replayed by this library's slot cache and by the reference's
own DgCore; the slot table and the sixteen counters must be identical after every token. The configurations stay
within the rules the reference's layout enforces (spare blocks cover the spare slots; the inclusive share stays
below the spare blocks)."""
import numpy as np
import pytest

import oracle
from tierstream_b200 import runtime

from test_dg_replay import make_case


def random_case(seed):
    r = np.random.default_rng(seed)
    G = int(r.integers(2, 9))
    U = int(r.choice([4, 8, 16, 32]))
    B = int(r.integers(1, min(U, 8) + 1))
    R = int(r.integers(0, U - 1))
    D = int(r.integers(1, max(2, min(4, U - R)) + 1))
    D = min(D, U - R)
    Q = D * G + int(r.integers(0, 6))
    kw = dict(G=G, U=U, B=B, R=R, D=D, Q=Q, tokens=int(r.integers(10, 40)), seed=int(r.integers(1, 10 ** 6)),
              parts=tuple(int(x) * 256 for x in r.integers(1, 9, size=int(r.integers(1, 4)))),
              wb_defer=int(r.integers(0, 2)), wb_on_d2h=int(r.integers(0, 2)))
    trace = r.integers(0, 3)
    if trace == 0:
        kw["uniform"] = True
    elif trace == 1:
        kw["s"] = float(r.uniform(0.6, 1.4))
    else:
        kw["s"] = float(r.uniform(0.6, 1.2))
        kw["rho"] = float(r.uniform(0.2, 0.8))
    if r.random() < 0.4:
        kw["n_pred"] = int(r.integers(1, min(U, 4) + 1))
        kw["prefetch_per_layer"] = int(r.integers(1, 5))
        kw["prefetch_per_token"] = int(r.integers(2, 49))
        if r.random() < 0.5:
            kw["prefetch_reserve"] = int(r.integers(0, 3))
    if r.random() < 0.3:
        kw["wb_layer_bytes"] = int(r.integers(1, 8)) * 1024
        kw["wb_max_outstanding"] = int(r.integers(1, 16)) * 4096
    if r.random() < 0.35:
        inc = int(r.integers(1, 12))
        kw["inclusive"] = inc
        kw["Q"] = max(Q, inc + 1)
    return kw


@pytest.mark.parametrize("seed", range(200))
def test_random_configurations_match_reference(ref, seed):
    kw = random_case(seed)
    cfg, ids, preds = make_case(**kw)
    t_ref, s_ref = oracle.ref_replay(cfg, ids, preds)
    t_new, s_new = runtime.replay(cfg, ids, preds)
    for t in range(cfg.tokens):
        assert np.array_equal(t_new[t], t_ref[t]), "case %s: slot table differs after token %d" % (kw, t)
        assert np.array_equal(s_new[t], s_ref[t]), "case %s: counters differ after token %d: %s vs %s" % (
            kw, t, s_new[t].tolist(), s_ref[t].tolist())
