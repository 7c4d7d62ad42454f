"""Host read-ahead on the CPU (tsb_test_read_ahead, csrc/read_ahead.cpp): requests read units from a file into a set of
buffers as buffers come free; a fetch copies from the buffer when the read started (waiting for its end), reads the
file itself when the request had not started (the request is dropped) or had failed (a fallback), and fails with the
read's error when the read fails after the fetch claimed it; buffers come back after the fetch's copy or at the
forward's end, except a buffer whose copy failed after it started. Each forward counts its requests, reads, landings,
unused reads, failures and bytes once, as the reference's reconcile does (src/stream_ctx.cpp:805-832)."""
import ctypes as C

import numpy as np
import pytest

from tierstream_b200 import abi

UNIT = 12_345
N = 12
FILE_BYTES = N * 16384 + 777
BAD = 10 ** 9  # an offset past the file's end: its read fails with SS_E_IO


@pytest.fixture(scope="module")
def data_file(tmp_path_factory):
    p = tmp_path_factory.mktemp("ra") / "units.bin"
    data = np.random.default_rng(5).integers(0, 256, size=FILE_BYTES, dtype=np.uint8)
    data.tofile(p)
    return str(p), data


def checksum(b):
    return int((b.astype(np.uint64) * (np.arange(b.size, dtype=np.uint64) % 251 + 1)).sum())


REQ, FETCH, END, SLEEP = 0, 1, 2, 3


def run(path, script, buffers=4, threads=2, delay_us=0, offsets=None):
    offsets = offsets if offsets is not None else [u * 16384 for u in range(N)]
    off = np.asarray(offsets, dtype=np.uint64)
    sc = np.asarray(script, dtype=np.int32).reshape(-1, 3)
    fetches = int((sc[:, 0] == FETCH).sum())
    ends = int((sc[:, 0] == END).sum())
    sums = np.zeros(max(1, fetches), dtype=np.uint64)
    codes = np.zeros(max(1, fetches), dtype=np.int32)
    stats = np.zeros((max(1, ends), 7), dtype=np.uint64)
    st = abi.load().tsb_test_read_ahead(path.encode(), off.ctypes.data_as(C.POINTER(C.c_uint64)), len(offsets), UNIT,
                                        buffers, threads, delay_us, sc.ctypes.data_as(C.POINTER(C.c_int32)), len(sc),
                                        sums.ctypes.data_as(C.POINTER(C.c_uint64)),
                                        codes.ctypes.data_as(C.POINTER(C.c_int32)),
                                        stats.ctypes.data_as(C.POINTER(C.c_uint64)))
    assert st == abi.SS_OK, abi.load().ss_last_error()
    return sums[:fetches], codes[:fetches], stats[:ends]


def want(data, u):
    return checksum(data[u * 16384:u * 16384 + UNIT])


def test_every_request_lands_its_own_bytes(data_file):
    path, data = data_file
    script = [(REQ, u, 0) for u in range(8)] + [(SLEEP, 0, 20000)] + [(FETCH, u, 0) for u in range(8)] + [(END, 0, 0)]
    sums, codes, stats = run(path, script)
    assert codes.tolist() == [1] * 8
    assert sums.tolist() == [want(data, u) for u in range(8)]
    assert stats[0].tolist() == [8, 8, 8, 0, 0, 0, 8 * UNIT]  # four buffers served eight reads: each came back


def test_reads_nobody_fetched_are_unused(data_file):
    path, _ = data_file
    _, _, stats = run(path, [(REQ, u, 0) for u in range(4)] + [(SLEEP, 0, 20000), (END, 0, 0)])
    assert stats[0].tolist() == [4, 4, 0, 4, 0, 0, 4 * UNIT]


def test_a_request_not_started_is_dropped_and_the_file_read(data_file):
    """One buffer and slow reads: the third request is still waiting when its fetch comes (the file is read instead);
    the first is read while its fetch waits; the second starts when the first's buffer comes back."""
    path, data = data_file
    script = [(REQ, 0, 0), (REQ, 1, 0), (REQ, 2, 0), (FETCH, 2, 0), (FETCH, 0, 0), (FETCH, 1, 0), (END, 0, 0)]
    sums, codes, stats = run(path, script, buffers=1, threads=1, delay_us=30000)
    assert codes.tolist() == [0, 1, 1]
    assert sums.tolist() == [0, want(data, 0), want(data, 1)]
    assert stats[0].tolist() == [3, 2, 2, 0, 0, 0, 2 * UNIT]


def test_a_read_that_failed_before_its_fetch_falls_back(data_file):
    path, _ = data_file
    offsets = [u * 16384 for u in range(N)]
    offsets[3] = BAD
    sums, codes, stats = run(path, [(REQ, 3, 0), (SLEEP, 0, 20000), (FETCH, 3, 0), (END, 0, 0)], offsets=offsets)
    assert codes.tolist() == [0]
    assert stats[0].tolist()[:6] == [1, 0, 0, 0, 1, 1]


def test_a_read_that_fails_after_its_fetch_fails_the_fetch(data_file):
    path, _ = data_file
    offsets = [u * 16384 for u in range(N)]
    offsets[3] = BAD
    sums, codes, stats = run(path, [(REQ, 3, 0), (FETCH, 3, 0), (END, 0, 0)], delay_us=20000, offsets=offsets)
    assert codes.tolist() == [-abi.SS_E_IO]
    assert stats[0].tolist()[:6] == [1, 0, 0, 0, 1, 0]


def test_a_buffer_whose_copy_failed_midway_is_never_reused(data_file):
    """Forward 1: the only buffer's copy fails after it started; forward 2: a request never gets a buffer, its fetch
    reads the file."""
    path, _ = data_file
    script = [(REQ, 0, 0), (SLEEP, 0, 10000), (FETCH, 0, 2), (END, 0, 0),
              (REQ, 1, 0), (SLEEP, 0, 10000), (FETCH, 1, 0), (END, 0, 0)]
    _, codes, stats = run(path, script, buffers=1)
    assert codes.tolist() == [1, 0]
    assert stats[0].tolist()[:5] == [1, 1, 0, 1, 0] and stats[1].tolist()[:5] == [1, 0, 0, 0, 0]


def test_a_copy_that_failed_before_it_started_gives_the_buffer_back(data_file):
    path, data = data_file
    script = [(REQ, 0, 0), (SLEEP, 0, 10000), (FETCH, 0, 1), (END, 0, 0),
              (REQ, 1, 0), (SLEEP, 0, 10000), (FETCH, 1, 0), (END, 0, 0)]
    sums, codes, stats = run(path, script, buffers=1)
    assert codes.tolist() == [1, 1] and sums[1] == want(data, 1)
    assert stats[0].tolist()[:5] == [1, 1, 0, 1, 0] and stats[1].tolist()[:5] == [1, 1, 1, 0, 0]


def test_a_unit_is_requested_once_per_forward(data_file):
    path, _ = data_file
    script = [(REQ, 0, 0), (REQ, 0, 0), (SLEEP, 0, 10000), (FETCH, 0, 0), (FETCH, 0, 0), (END, 0, 0),
              (REQ, 0, 0), (SLEEP, 0, 10000), (END, 0, 0)]
    _, codes, stats = run(path, script)
    assert codes.tolist() == [1, 0]  # the second fetch in a forward reads its file
    assert stats[0].tolist()[:4] == [1, 1, 1, 0] and stats[1].tolist()[:4] == [1, 1, 0, 1]


@pytest.mark.parametrize("seed", range(30))
def test_random_scripts_keep_bytes_and_accounting(data_file, seed):
    path, data = data_file
    r = np.random.default_rng(seed)
    offsets = [u * 16384 for u in range(N)]
    bad = set(int(x) for x in r.choice(N, size=int(r.integers(0, 3)), replace=False))
    for u in bad:
        offsets[u] = BAD
    script, fetch_units, fw_requests = [], [], []
    for _ in range(int(r.integers(1, 4))):
        asked = set()
        for _ in range(int(r.integers(1, 25))):
            op = int(r.choice([REQ, REQ, FETCH, SLEEP]))
            u = int(r.integers(0, N))
            if op == REQ:
                asked.add(u)
                script.append((REQ, u, 0))
            elif op == FETCH:
                script.append((FETCH, u, int(r.choice([0, 0, 0, 1]))))
                fetch_units.append(u)
            else:
                script.append((SLEEP, 0, int(r.integers(0, 3000))))
        script.append((END, 0, 0))
        fw_requests.append(len(asked))
    sums, codes, stats = run(path, script, buffers=int(r.integers(1, 5)), threads=int(r.integers(1, 4)),
                             delay_us=int(r.choice([0, 500, 3000])), offsets=offsets)
    for u, s, c in zip(fetch_units, sums, codes):
        if c == 1:
            assert u not in bad and s == want(data, u)
        elif c < 0:
            assert u in bad and c == -abi.SS_E_IO
    for f, n in zip(stats, fw_requests):
        requested, read, landed, unused, failed = (int(x) for x in f[:5])
        assert requested == n and landed + unused == read and read + failed <= requested
        assert int(f[6]) == read * UNIT
