"""Slot-table parity of the reference's opt-in device-gated policies on the CPU: dg_no_admit (every demand miss
through its layer's bank slot, nothing admitted, no boundary eviction, no prefetch), dg_clean_evict (file tier: a
victim with no free block goes to its file, no pinned unit dropped for it), dg_pf_revert_unused (an unused prefetch
goes back at the boundary) and dg_pf_strict_admit (a prefetch leaves the spare target's slots free too), alone and
together with the other features. Tables, the sixteen counters, the file counters, the rounds' sums and the policies'
own counters (clean drops and bytes, reverts and bytes, strict refusals) are identical after every token."""
import numpy as np
import pytest

import oracle
from tierstream_b200 import runtime

from test_dg_disk_replay import make_disk_case
from test_dg_replay import make_case


def _compare(cfg, ids, preds):
    x = [np.zeros((cfg.tokens, 6), dtype=np.uint64) for _ in range(2)]
    r = [np.zeros((cfg.tokens, 6), dtype=np.uint64) for _ in range(2)]
    p = [np.zeros((cfg.tokens, 5), dtype=np.uint64) for _ in range(2)]
    t_ref, s_ref = oracle.ref_replay(cfg, ids, preds, xstats=x[0], rstats=r[0], pstats=p[0])
    t_new, s_new = runtime.replay(cfg, ids, preds, xstats=x[1], rstats=r[1], pstats=p[1])
    for t in range(cfg.tokens):
        assert np.array_equal(t_new[t], t_ref[t]), "slot table differs after token %d" % t
        assert np.array_equal(s_new[t], s_ref[t]), "counters differ after token %d: %s vs %s" % (
            t, s_new[t].tolist(), s_ref[t].tolist())
        assert np.array_equal(x[1][t], x[0][t]), "file counters differ after token %d" % t
        assert np.array_equal(r[1][t], r[0][t]), "round sums differ after token %d" % t
        assert np.array_equal(p[1][t], p[0][t]), "policy counters differ after token %d: %s vs %s" % (
            t, p[1][t].tolist(), p[0][t].tolist())
    return s_new[-1], x[1][-1], p[1][-1]


TWO_TIER = {
    "no_admit": dict(no_admit=1),
    "no_admit_with_predictions": dict(no_admit=1, n_pred=2),
    "no_admit_with_rounds": dict(no_admit=1, round_every=4),
    "pf_revert": dict(pf_revert=1, n_pred=3),
    "pf_revert_boundary_writebacks": dict(pf_revert=1, n_pred=3, wb_defer=0),
    "pf_revert_scored": dict(pf_revert=1, n_pred=2, policy=1, D=2),
    "pf_strict": dict(pf_strict=1, n_pred=3, D=3, prefetch_reserve=0),
    "pf_strict_and_revert": dict(pf_strict=1, pf_revert=1, n_pred=3, D=3),
}


@pytest.mark.parametrize("name", sorted(TWO_TIER))
def test_two_tier_policies_match_reference(ref, name):
    cfg, ids, preds = make_case(**TWO_TIER[name])
    s, _, p = _compare(cfg, ids, preds)
    if "no_admit" in name:
        assert s[8] > 0 and s[10] == 0, "misses served through banks, nothing evicted"
    if "revert" in name and "strict" not in name:  # (strict admission may leave no prefetch to revert)
        assert p[2] > 0
    if name == "pf_strict":
        assert p[4] > 0


FILE_TIER = {
    "clean_evict": dict(clean_evict=1, pinned=3, Q=2, D=2),
    "clean_evict_boundary_writebacks": dict(clean_evict=1, pinned=2, Q=1, D=3, wb_defer=0),
    "clean_evict_with_rounds": dict(clean_evict=1, pinned=3, Q=1, D=2, round_every=3),
    "pf_revert_files": dict(pf_revert=1, n_pred=3, disk_prefetch=1, pinned=2),
    "no_admit_files": dict(no_admit=1, pinned=3),
    "everything": dict(clean_evict=1, pf_revert=1, pf_strict=1, n_pred=2, disk_prefetch=1, pinned=2, Q=2, D=2,
                       round_every=5, policy=1),
}


@pytest.mark.parametrize("name", sorted(FILE_TIER))
def test_file_tier_policies_match_reference(ref, name):
    cfg, ids, preds = make_disk_case(**FILE_TIER[name])
    _, x, p = _compare(cfg, ids, preds)
    if name.startswith("clean_evict"):
        assert p[0] > 0 and p[1] == p[0] * sum(cfg.part_bytes[i] for i in range(cfg.n_parts))


def random_option_case(seed):
    r = np.random.default_rng(40_000 + seed)
    G = int(r.integers(2, 7))
    U = int(r.choice([4, 8, 16]))
    B = int(r.integers(1, min(U, 6) + 1))
    R = int(r.integers(0, U - 1))
    D = min(int(r.integers(1, 4)), U - R)
    kw = dict(G=G, U=U, B=B, R=R, D=D, tokens=int(r.integers(10, 35)), seed=int(r.integers(1, 10 ** 6)),
              wb_defer=int(r.integers(0, 2)), wb_on_d2h=int(r.integers(0, 2)), s=float(r.uniform(0.6, 1.4)),
              no_admit=int(r.random() < 0.25), pf_revert=int(r.random() < 0.5), pf_strict=int(r.random() < 0.5))
    if r.random() < 0.6:
        kw["n_pred"] = int(r.integers(1, min(U, 4) + 1))
    if r.random() < 0.3:
        kw["round_every"] = int(r.integers(1, 6))
    if r.random() < 0.3:
        kw["policy"] = int(r.integers(1, 3))
    disk = r.random() < 0.5
    if disk:
        kw["pinned"] = int(r.integers(0, U - R))
        kw["S"] = int(r.integers(1, 4))
        kw["Q"] = int(r.integers(1, D * G + 3))
        kw["clean_evict"] = int(r.random() < 0.5)
        if "n_pred" in kw:
            kw["disk_prefetch"] = int(r.integers(0, 2))
    else:
        kw["Q"] = D * G + int(r.integers(0, 4))
    return kw, disk


@pytest.mark.parametrize("seed", range(120))
def test_random_option_configurations_match_reference(ref, seed):
    kw, disk = random_option_case(seed)
    cfg, ids, preds = (make_disk_case if disk else make_case)(**kw)
    try:
        _compare(cfg, ids, preds)
    except AssertionError as e:
        raise AssertionError("case %s: %s" % (kw, e))
