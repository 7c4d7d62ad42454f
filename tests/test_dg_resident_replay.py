"""Slot-table parity of kept-resident layers (ss_dg_make_resident) on the CPU: between tokens a gated layer's chosen
units are made resident in both this library's slot cache and the reference's own DgCore (victims by the policy's
order with the boundary's lower-tier rules, write-backs, drops to files, copies in from blocks or files), the layer is
not exported while held and its units are kept at every boundary and round, and a release returns it to the normal
flow. Tables, the sixteen counters, the file counters and the resident counters (units copied in, evicted, file reads,
write-back bytes) are identical after every token; with real bytes every unit read through the table is its own."""
import re

import numpy as np
import pytest

import oracle
from tierstream_b200 import runtime

from test_dg_disk_replay import make_disk_case
from test_dg_replay import make_case


def _compare(cfg, ids, preds, src=None):
    x = [np.zeros((cfg.tokens, 6), dtype=np.uint64) for _ in range(2)]
    m = [np.zeros((cfg.tokens, 4), dtype=np.uint64) for _ in range(2)]
    kw = dict(src_units=src, want_reads=src is not None)
    ref = oracle.ref_replay(cfg, ids, preds, xstats=x[0], mstats=m[0], **kw)
    new = runtime.replay(cfg, ids, preds, xstats=x[1], mstats=m[1], **kw)
    for t in range(cfg.tokens):
        assert np.array_equal(new[0][t], ref[0][t]), "slot table differs after token %d" % t
        assert np.array_equal(new[1][t], ref[1][t]), "counters differ after token %d" % t
        assert np.array_equal(x[1][t], x[0][t]), "file counters differ after token %d" % t
        assert np.array_equal(m[1][t], m[0][t]), "resident counters differ after token %d: %s vs %s" % (
            t, m[1][t].tolist(), m[0][t].tolist())
    if src is not None:
        assert np.array_equal(new[2], ref[2])
    return m[1][-1], new


def events(G, U, seed, n=4, max_ids=3, tokens=40):
    r = np.random.default_rng(seed)
    out = []
    held = set()
    for t in sorted(r.choice(np.arange(2, tokens - 2), size=n, replace=False).tolist()):
        g = int(r.integers(0, G))
        if g in held and r.random() < 0.5:
            out.append((t, g, ()))
            held.discard(g)
            continue
        k = int(r.integers(1, max_ids + 1))
        out.append((t, g, tuple(int(u) for u in r.choice(U, size=k, replace=False))))
        held.add(g)
    return out


CASES = {
    "hold_and_release": dict(kw=dict(D=3, B=2), n=4),
    "boundary_writebacks": dict(kw=dict(D=3, B=2, wb_defer=0), n=5),
    "scored": dict(kw=dict(D=3, B=2, policy=1), n=4),
    "clean_copies": dict(kw=dict(D=3, B=2, inclusive=6, Q=12), n=4),
    "with_rounds": dict(kw=dict(D=3, B=2, round_every=4), n=4),
    "with_predictions": dict(kw=dict(D=3, B=2, n_pred=2), n=4),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_make_resident_matches_reference(ref, name):
    c = CASES[name]
    ev = events(6, 16, 7, n=c["n"])
    cfg, ids, preds = make_case(tokens=40, resident_events=ev, **c["kw"])
    m, _ = _compare(cfg, ids, preds)
    assert m[0] > 0, "units must be copied in"


@pytest.mark.parametrize("kw", [dict(pinned=3, D=3, B=2), dict(pinned=0, D=3, B=2, Q=4), dict(pinned=2, D=3, B=2,
                                disk_queue=3, S=4), dict(pinned=2, D=3, B=2, clean_evict=1, Q=2)])
def test_make_resident_with_the_file_tier_matches_reference(ref, kw):
    ev = events(6, 16, 11, n=5)
    cfg, ids, preds = make_disk_case(tokens=40, resident_events=ev, **kw)
    m, _ = _compare(cfg, ids, preds)
    assert m[0] > 0 and m[2] > 0, "units must be read from their files"


def test_make_resident_bytes(ref):
    G, U, parts = 4, 12, (256, 512, 256)
    ev = [(5, 1, (0, 3, 7)), (12, 2, (1, 2)), (20, 1, ()), (25, 3, (4, 5, 6))]
    cfg, ids, preds = make_disk_case(G=G, U=U, parts=parts, R=2, pinned=3, D=3, B=2, tokens=30, resident_events=ev)
    cfg.move_bytes = 1
    unit = sum(parts)
    src = np.random.default_rng(2).integers(0, 256, size=G * U * unit, dtype=np.uint8)
    _, new = _compare(cfg, ids, preds, src)
    orc = oracle.orc()
    want = [orc.orc_checksum(src[k * unit:].ctypes.data, unit) for k in range(G * U)]
    held = {}
    for t in range(cfg.tokens):
        for g in range(G):
            if g in held:  # not exported while held (the held units are resident; nothing read here)
                continue
            for i in range(cfg.n_ids):
                assert new[2][t, g, i] == want[g * U + int(ids[t, g, i])], (t, g, i)
        for (te, g, u) in ev:
            if te == t:
                if u:
                    held[g] = u
                else:
                    held.pop(g, None)
    # a held unit stays resident: its entry holds a slot after every later token while held
    for (te, g, u) in ev:
        if not u:
            continue
        end = next((t2 for (t2, g2, u2) in ev if g2 == g and t2 > te), cfg.tokens)
        for t in range(te, min(end, cfg.tokens)):
            for x in u:
                assert new[0][t][g * U + x] >= 0, (t, g, x)


def test_make_resident_refusals_match(ref):
    """More units than the persistent slots allow: both refuse (the replay fails the same way)."""
    cfg, ids, preds = make_case(D=1, B=2, R=1, tokens=10, resident_events=[(3, 0, tuple(range(16)))])
    with pytest.raises(Exception, match="persistent slots"):
        runtime.replay(cfg, ids, preds)
    with pytest.raises(RuntimeError, match="persistent slots"):
        oracle.ref_replay(cfg, ids, preds)


@pytest.mark.parametrize("seed", range(80))
def test_random_make_resident_matches_reference(ref, seed):
    r = np.random.default_rng(60_000 + seed)
    G = int(r.integers(2, 7))
    U = int(r.choice([8, 16, 32]))
    B = int(r.integers(1, 5))
    R = int(r.integers(0, 4))
    D = int(r.integers(2, 5))
    tokens = int(r.integers(15, 40))
    kw = dict(G=G, U=U, B=B, R=R, D=D, tokens=tokens, seed=int(r.integers(1, 10 ** 6)),
              wb_defer=int(r.integers(0, 2)), wb_on_d2h=int(r.integers(0, 2)), s=float(r.uniform(0.7, 1.4)),
              resident_events=events(G, U, seed, n=int(r.integers(1, 6)), max_ids=min(3, D), tokens=tokens))
    if r.random() < 0.3:
        kw["policy"] = 1
    if r.random() < 0.3:
        kw["n_pred"] = int(r.integers(1, 3))
    if r.random() < 0.25:
        kw["round_every"] = int(r.integers(2, 6))
    disk = r.random() < 0.5
    if disk:
        kw.update(pinned=int(r.integers(0, U - R)), S=int(r.integers(1, 4)), Q=int(r.integers(1, D * G + 3)),
                  disk_queue=int(r.integers(1, 4)))
    else:
        kw["Q"] = D * G + int(r.integers(0, 4))
    cfg, ids, preds = (make_disk_case if disk else make_case)(**kw)
    try:
        _compare(cfg, ids, preds)
    except RuntimeError as e:  # a capacity refusal must come from both
        with pytest.raises(Exception, match=re.escape(str(e).split(": ")[-1][:40])):
            runtime.replay(cfg, ids, preds)
    except AssertionError as e:
        raise AssertionError("case %s: %s" % ({k: v for k, v in kw.items()}, e))
