"""The host forward mode's resident set on the CPU, LRU and SCORED, against the reference's own ResidentSet (compiled
from its sources) driven the same way (its host mode's ingest order: busy units, prefetched units that are neither
hits nor admitted, an admission with an eviction cap, an observation): every unit's slot and the step's counts (hits,
admitted, evicted, transient, deferred) are identical after every step; SCORED decides differently from LRU."""
import numpy as np
import pytest

import oracle
from tierstream_b200 import abi


def case(seed, n_units=16, capacity=6, steps=60, k=4, policy=1, window=16, p_busy=0.05, p_pf=0.1, p_cap=0.3,
         p_noadmit=0.1, n_place=3, pin=1):
    r = np.random.default_rng(seed)
    pop = r.permutation(n_units)
    w = 1.0 / np.arange(1, n_units + 1) ** 1.1
    w /= w.sum()
    routed = np.full((steps, k), -1, dtype=np.int32)
    for t in range(steps):
        ids = r.choice(n_units, size=k, replace=False, p=w)
        routed[t] = pop[ids]
        if r.random() < 0.2:
            routed[t, -1] = -1
    flags = np.zeros((steps, n_units), dtype=np.uint8)
    flags |= (r.random((steps, n_units)) < p_busy).astype(np.uint8)
    pf = (r.random((steps, n_units)) < p_pf)
    flags |= (pf.astype(np.uint8) << 1)
    max_ev = np.where(r.random(steps) < p_cap, r.integers(0, 3, size=steps), -1).astype(np.int32)
    admit = (r.random(steps) >= p_noadmit).astype(np.uint8)
    place = pop[:n_place].astype(np.int32)
    pins = np.zeros(n_place, dtype=np.uint8)
    pins[:pin] = 1
    return dict(n_units=n_units, capacity=capacity, policy=policy, window=window, place=place, pins=pins,
                routed=routed, flags=flags, max_ev=max_ev, admit=admit)


def run(c, ref=False):
    steps, k = c["routed"].shape
    slots = np.zeros((steps, c["n_units"]), dtype=np.int32)
    counts = np.zeros((steps, 5), dtype=np.int32)
    args = [c["n_units"], c["capacity"], c["policy"], c["window"], c["place"].ctypes.data, c["pins"].ctypes.data,
            len(c["place"]), steps, c["routed"].ctypes.data, k, c["flags"].ctypes.data, c["max_ev"].ctypes.data,
            c["admit"].ctypes.data, slots.ctypes.data, counts.ctypes.data]
    if ref:
        import ctypes as C
        err = C.create_string_buffer(256)
        assert oracle.ref().oref_resident_replay(*args, err, 256) == 0, err.value
    else:
        abi.check(abi.load().tsb_test_resident_replay(*args))
    return slots, counts


@pytest.mark.parametrize("policy", [0, 1])
@pytest.mark.parametrize("seed", range(40))
def test_resident_set_matches_reference(ref, policy, seed):
    r = np.random.default_rng(seed)
    c = case(seed, n_units=int(r.choice([4, 8, 16, 32])), capacity=int(r.integers(0, 8)), policy=policy,
             window=int(r.integers(1, 20)), k=int(r.integers(1, 5)), n_place=int(r.integers(0, 4)),
             pin=int(r.integers(0, 2)))
    c["capacity"] = min(c["capacity"], c["n_units"])
    c["place"] = c["place"][:min(len(c["place"]), c["capacity"])]
    c["pins"] = c["pins"][:len(c["place"])]
    s_new, n_new = run(c)
    s_ref, n_ref = run(c, ref=True)
    for t in range(len(s_new)):
        assert np.array_equal(s_new[t], s_ref[t]), "slots differ after step %d" % t
        assert np.array_equal(n_new[t], n_ref[t]), "counts differ after step %d: %s vs %s" % (
            t, n_new[t].tolist(), n_ref[t].tolist())


def test_scored_decides_differently_from_lru(ref):
    c = case(3, n_units=16, capacity=5, steps=80, k=3, p_busy=0.0, p_pf=0.0, p_cap=0.0, p_noadmit=0.0)
    s_scored, _ = run(c)
    c0 = dict(c, policy=0)
    s_lru, _ = run(c0)
    assert not np.array_equal(s_scored, s_lru)
