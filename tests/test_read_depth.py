"""The adaptive read depth's controller (dg_disk_queue_adapt) against the reference's, on the CPU: both fed the same
busy periods (reads, bytes, ns) return the same depth after every period, and end with the same counters (depth
changes, calibrations, windows, per-depth reads / bytes / busy time, verdicts) and the same verdict ring. The periods
come from rate regimes that change over time, with noise, so that every path is taken: U kept, 1 kept with back-off,
split verdicts measured again, re-checks, drifts, empty and zero-time periods."""
import ctypes as C

import numpy as np
import pytest

import oracle
from tierstream_b200 import abi

P64 = C.POINTER(C.c_uint64)


def _run(fn, bound, params, reads, nbytes, ns):
    n = len(reads)
    depth = np.zeros(n, dtype=np.uint32)
    counters = np.zeros(11, dtype=np.uint64)
    ring = np.zeros((16, 7), dtype=np.float64)
    nv = C.c_uint32()
    pr = (C.c_double * 6)(*params) if params is not None else None
    rc = fn(C.c_uint32(bound), pr, C.c_uint32(n), reads.ctypes.data_as(P64), nbytes.ctypes.data_as(P64),
            ns.ctypes.data_as(P64), depth.ctypes.data_as(C.POINTER(C.c_uint32)), counters.ctypes.data_as(P64),
            ring.ctypes.data_as(C.POINTER(C.c_double)), C.byref(nv))
    assert rc == 0
    return depth, counters, ring[:nv.value]


def periods(seed, n):
    """Busy periods whose rate moves between regimes (a drive's behaviour changing) with noise around each, so that
    calibrations see depth U win, lose and split, and held depths see drifts."""
    r = np.random.default_rng(seed)
    unit = int(r.choice([1 << 20, 33 << 20, 7 << 16]))
    reads = np.zeros(n, dtype=np.uint64)
    nbytes = np.zeros(n, dtype=np.uint64)
    ns = np.zeros(n, dtype=np.uint64)
    rate = float(r.uniform(2.0, 7.0))  # bytes per ns
    for i in range(n):
        if r.random() < 0.02:
            rate = float(r.uniform(1.0, 9.0))  # a new regime
        k = int(r.integers(1, 40)) if r.random() > 0.03 else 0
        reads[i] = k
        nbytes[i] = k * unit
        ns[i] = 0 if r.random() < 0.01 else int(k * unit / (rate * float(r.uniform(0.85, 1.15))))
    return reads, nbytes, ns


def case(seed):
    r = np.random.default_rng(900 + seed)
    bound = int(r.choice([2, 3, 4, 8, 16]))
    params = None
    if seed % 3 == 1:  # small windows and short holds: many calibrations in a short run
        params = [int(r.integers(1, 8)), int(r.integers(8, 64)), int(r.integers(16, 128)), int(r.integers(64, 512)),
                  float(r.choice([0.0, 0.03, 0.1])), float(r.choice([0.1, 0.25, 0.5]))]
    return (bound, params) + periods(7000 + seed, 3000)


@pytest.mark.parametrize("seed", range(40))
def test_depth_matches_reference(ref, seed):
    bound, params, reads, nbytes, ns = case(seed)
    lib, refl = abi.load(), oracle.ref()
    a = _run(lib.tsb_test_read_depth, bound, params, reads, nbytes, ns)
    b = _run(refl.oref_read_depth, bound, params, reads, nbytes, ns)
    assert np.array_equal(a[0], b[0]), "depths differ first at period %d" % int(np.argmax(a[0] != b[0]))
    assert np.array_equal(a[1], b[1]), "counters %s vs %s" % (a[1].tolist(), b[1].tolist())
    assert np.array_equal(a[2], b[2]), "verdict rings differ"


def test_paths_are_taken(ref):
    """Over the cases above: U kept and 1 kept, split verdicts, re-checks and drifts all occur."""
    lib = abi.load()
    reasons, depths = set(), set()
    for seed in range(40):
        bound, params, reads, nbytes, ns = case(seed)
        d, c, ring = _run(lib.tsb_test_read_depth, bound, params, reads, nbytes, ns)
        reasons |= {int(x) for x in ring[:, 6]}
        depths |= set(np.unique(d).tolist())
        assert c[1] >= 1  # the first calibration starts at once
    assert {1, 2, 3} <= reasons, reasons  # keep U, keep 1, split (re-checks and drifts start calibrations)
    assert 1 in depths and len(depths) >= 2


def test_bound_one_never_changes(ref):
    lib = abi.load()
    reads = np.full(200, 33, dtype=np.uint64)
    d, c, ring = _run(lib.tsb_test_read_depth, 1, None, reads, reads * 4096, reads * 1000)
    assert (d == 1).all() and c[2] == 0 and len(ring) == 0
