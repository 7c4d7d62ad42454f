"""Slot-table parity of dg_bank_keep on the CPU. A demand file miss served through a bank slot is read into a pinned
block (a free one, else the least recently homed pinned unit's, dropped to its file), which becomes its home when the
bank lets it go: at the front of the pinned recency list (1) or behind its front half (2). The reference's rules are
in its src/dg_core.cpp:142-160 (the middle insert), 200-213 (the release), 237-250 (the block), 1286-1303 and
1330-1333 (the read and the churn count). Tables, the sixteen counters, the file counters, the option's own counters
(bank_kept, bank_keep_drops, bank_keep_rereads) and the pinned homes' recency order (a hash after every token) are
identical with the reference DgCore after every token, alone and with the other file-tier features."""
import numpy as np
import pytest

import oracle
from tierstream_b200 import runtime

from test_dg_disk_replay import make_disk_case


def _compare(cfg, ids, preds):
    T = cfg.tokens
    x = [np.zeros((T, 6), dtype=np.uint64) for _ in range(2)]
    p = [np.zeros((T, 5), dtype=np.uint64) for _ in range(2)]
    k = [np.zeros((T, 4), dtype=np.uint64) for _ in range(2)]
    t_ref, s_ref = oracle.ref_replay(cfg, ids, preds, xstats=x[0], pstats=p[0], kstats=k[0])
    t_new, s_new = runtime.replay(cfg, ids, preds, xstats=x[1], pstats=p[1], kstats=k[1])
    for t in range(T):
        assert np.array_equal(t_new[t], t_ref[t]), "slot table differs after token %d" % t
        assert np.array_equal(s_new[t], s_ref[t]), "counters differ after token %d: %s vs %s" % (
            t, s_new[t].tolist(), s_ref[t].tolist())
        assert np.array_equal(x[1][t], x[0][t]), "file counters differ after token %d" % t
        assert np.array_equal(p[1][t], p[0][t]), "policy counters differ after token %d" % t
        assert np.array_equal(k[1][t][:3], k[0][t][:3]), "bank keep counters differ after token %d: %s vs %s" % (
            t, k[1][t][:3].tolist(), k[0][t][:3].tolist())
        assert k[1][t][3] == k[0][t][3], "the pinned recency order differs after token %d" % t
    return s_new[-1], x[1][-1], k[1][-1]


CASES = {
    "front": dict(bank_keep=1),
    "middle": dict(bank_keep=2),
    "front_no_spare_blocks": dict(bank_keep=1, Q=0),
    "middle_no_spare_blocks": dict(bank_keep=2, Q=0, pinned=7),
    "middle_few_blocks": dict(bank_keep=2, Q=1, D=2),
    "front_reads_in_flight": dict(bank_keep=1, disk_queue=3, Q=1),
    "middle_reads_in_flight": dict(bank_keep=2, disk_queue=4, S=4),
    "middle_predictions_read_files": dict(bank_keep=2, n_pred=2, disk_prefetch=1),
    "middle_clean_evict": dict(bank_keep=2, clean_evict=1, Q=1, D=2),
    "front_rounds": dict(bank_keep=1, round_every=4),
    "middle_scored": dict(bank_keep=2, policy=1, D=2),
    "middle_boundary_writebacks": dict(bank_keep=2, wb_defer=0),
    "middle_pf_revert": dict(bank_keep=2, pf_revert=1, n_pred=3, disk_prefetch=1, pinned=2),
    "middle_top8": dict(bank_keep=2, G=5, U=32, R=6, pinned=8, D=2, B=8, rho=0.5, s=0.9),
    "front_files_only": dict(bank_keep=1, pinned=0),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_bank_keep_matches_reference(ref, name):
    cfg, ids, preds = make_disk_case(**CASES[name])
    s, x, k = _compare(cfg, ids, preds)
    assert s[8] > 0, "no bank serve: the case does not reach the option"
    assert k[0] > 0, "no bank-served file read was kept"
    if "no_spare_blocks" in name:
        assert k[1] > 0, "a kept read never had to drop a pinned unit"


def test_bank_keep_has_no_effect_with_no_admit_or_off(ref):
    """With dg_no_admit homes never change (the option keeps nothing), and off it is the plain file tier."""
    for kw in (dict(bank_keep=1, no_admit=1), dict(bank_keep=0)):
        cfg, ids, preds = make_disk_case(**kw)
        _, _, k = _compare(cfg, ids, preds)
        assert k[0] == 0 and k[1] == 0


def test_bank_keep_across_a_reset(ref):
    """ss_dg_reset_open mid-trace restores the open placement and pinned order; the kept reads after it match."""
    cfg, ids, preds = make_disk_case(bank_keep=2, Q=1, D=2, tokens=40)
    cfg.reset_at = 20
    _, _, k = _compare(cfg, ids, preds)
    assert k[0] > 0


@pytest.mark.parametrize("seed", range(24))
def test_bank_keep_fuzz(ref, seed):
    r = np.random.default_rng(52_000 + seed)
    G = int(r.integers(2, 7))
    U = int(r.choice([8, 16, 32]))
    R = int(r.integers(1, U // 4 + 1))
    B = int(r.choice([2, 4, 8]))
    kw = dict(G=G, U=U, R=R, pinned=int(r.integers(0, U // 2)), D=int(r.integers(1, 3)), B=B,
              Q=int(r.integers(0, 2 * G + 1)), S=int(r.integers(1, 5)), tokens=int(r.integers(20, 50)),
              s=float(r.choice([0.8, 1.1, 1.4])), seed=int(r.integers(0, 1000)), bank_keep=int(r.integers(1, 3)),
              disk_queue=int(r.choice([0, 1, 3])), wb_defer=int(r.integers(0, 2)))
    if r.random() < 0.4:
        kw.update(n_pred=int(r.integers(1, 4)), disk_prefetch=int(r.integers(0, 2)))
    if r.random() < 0.3:
        kw["clean_evict"] = 1
    if r.random() < 0.3:
        kw["policy"] = int(r.integers(1, 3))
    if r.random() < 0.3:
        kw["round_every"] = int(r.integers(3, 7))
    cfg, ids, preds = make_disk_case(**kw)
    _compare(cfg, ids, preds)
