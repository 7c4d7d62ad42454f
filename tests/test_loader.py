"""The open's fill pipeline on the CPU (tsb_test_load, csrc/loader.cpp): reader threads read units from a file into a
ring of buffers (units with a slot) or in place (pinned units), and the calling thread hands each buffer's batch to a
copy engine and waits for its copies before the buffer is read into again. The copy engine here is the hook's own
(a thread copying each batch a set delay after it was submitted), so a buffer handed back to a reader too early lands
wrong bytes. Every slot and every host block equals the file's bytes at its unit's offset, nothing else is written,
the batch count is the packing's, the ring is never over-committed, and failures (a read past the file's end, a copy
engine that refuses a batch, bad arguments) end the run with their status instead of hanging."""
import ctypes as C

import numpy as np
import pytest

from tierstream_b200 import abi

FILE_BYTES = (24 << 20) + 777


def last_error():
    return abi.load().ss_last_error().decode(errors="replace")


@pytest.fixture(scope="module")
def data_file(tmp_path_factory):
    p = tmp_path_factory.mktemp("load") / "model.bin"
    data = np.random.default_rng(11).integers(0, 256, size=FILE_BYTES, dtype=np.uint8)
    data.tofile(p)
    return str(p), data


def run(path, offsets, targets, unit_bytes, buffers, buffer_bytes, readers, direct, delay_us, fail_batch=-1,
        n_slots=None, n_host=None):
    stride = (unit_bytes + 4095) // 4096 * 4096
    n_slots = n_slots if n_slots is not None else max([t + 1 for t in targets if t >= 0], default=0)
    n_host = n_host if n_host is not None else max([-t for t in targets if t < 0], default=0)
    device = np.full(max(1, n_slots) * stride, 0xAB, dtype=np.uint8)
    host = np.full(max(1, n_host) * stride + 4096, 0xCD, dtype=np.uint8)
    hbase = (host.ctypes.data + 4095) // 4096 * 4096  # 4 KiB aligned blocks, as pinned blocks are
    off = np.asarray(offsets, dtype=np.uint64)
    tg = np.asarray(targets, dtype=np.int32)
    stats = np.zeros(6, dtype=np.uint64)
    st = abi.load().tsb_test_load(path.encode(), off.ctypes.data_as(C.POINTER(C.c_uint64)),
                                  tg.ctypes.data_as(C.POINTER(C.c_int32)), len(targets), unit_bytes,
                                  device.ctypes.data, hbase, buffers, buffer_bytes, readers, direct, delay_us,
                                  fail_batch, stats.ctypes.data_as(C.POINTER(C.c_uint64)))
    hview = host[hbase - host.ctypes.data:][:max(1, n_host) * stride]
    return st, device, hview, stats, stride


def expected_batches(targets, buffer_bytes, stride):
    per = buffer_bytes // stride
    n = sum(1 for t in targets if t >= 0)
    return (n + per - 1) // per


def check(data, offsets, targets, unit_bytes, device, host, stride):
    slot_units = {t: o for t, o in zip(targets, offsets) if t >= 0}
    host_units = {-t - 1: o for t, o in zip(targets, offsets) if t < 0}
    for s in range(device.size // stride):
        got = device[s * stride:(s + 1) * stride]
        if s in slot_units:
            o = slot_units[s]
            assert np.array_equal(got[:unit_bytes], data[o:o + unit_bytes]), "slot %d" % s
            assert (got[unit_bytes:] == 0xAB).all()
        else:
            assert (got == 0xAB).all(), "slot %d written" % s
    for b in range(host.size // stride):
        got = host[b * stride:(b + 1) * stride]
        if b in host_units:
            o = host_units[b]
            assert np.array_equal(got[:unit_bytes], data[o:o + unit_bytes]), "block %d" % b
        else:
            assert (got == 0xCD).all(), "block %d written" % b


@pytest.mark.parametrize("seed", range(40))
def test_every_unit_lands_where_its_target_says(data_file, seed):
    path, data = data_file
    r = np.random.default_rng(500 + seed)
    unit_bytes = int(r.choice([4096, 8192, 5000, 65536, 200_000, 1 << 20]))
    n = int(r.integers(1, 48))
    aligned = r.random() < 0.5
    offsets = [int(r.integers(0, FILE_BYTES - unit_bytes) // (4096 if aligned else 1) * (4096 if aligned else 1))
               for _ in range(n)]
    n_slot = int(r.integers(0, n + 1))
    kinds = r.permutation([1] * n_slot + [0] * (n - n_slot))
    slots = list(r.permutation(n_slot + int(r.integers(0, 3))))[:n_slot]
    blocks = list(r.permutation(n - n_slot + int(r.integers(0, 3))))[:n - n_slot]
    targets, si, bi = [], 0, 0
    for k in kinds:
        if k:
            targets.append(int(slots[si]))
            si += 1
        else:
            targets.append(-int(blocks[bi]) - 1)
            bi += 1
    stride = (unit_bytes + 4095) // 4096 * 4096
    buffers = int(r.integers(1 if n_slot else 0, 6))
    buffer_bytes = stride * int(r.integers(1, 5)) + int(r.integers(0, 4096))
    readers = int(r.integers(1, 12))
    delay = int(r.choice([0, 0, 200, 1500]))
    st, device, host, stats, stride = run(path, offsets, targets, unit_bytes, buffers, buffer_bytes, readers,
                                          int(r.integers(0, 2)), delay,
                                          n_slots=max(slots, default=-1) + 1 + int(r.integers(0, 2)),
                                          n_host=max(blocks, default=-1) + 1 + int(r.integers(0, 2)))
    assert st == abi.SS_OK, last_error()
    check(data, offsets, targets, unit_bytes, device, host, stride)
    assert stats[0] == n_slot and stats[1] == n - n_slot
    assert stats[2] == expected_batches(targets, buffer_bytes, stride)
    assert stats[5] <= max(buffers, 0)


def test_one_buffer_many_readers_recycles_under_slow_copies(data_file):
    """A ring of one buffer, eight readers and copies that take 2 ms: readers wait for the buffer and the opening thread
    recycles it for them; the bytes are still every unit's own."""
    path, data = data_file
    n, unit_bytes = 24, 65536
    offsets = [i * 65536 * 3 for i in range(n)]
    targets = list(range(n))
    st, device, host, stats, stride = run(path, offsets, targets, unit_bytes, 1, unit_bytes, 8, 1, 2000)
    assert st == abi.SS_OK, last_error()
    check(data, offsets, targets, unit_bytes, device, host, stride)
    assert stats[2] == n and stats[3] > 0 and stats[4] > 0 and stats[5] == 1


def test_pinned_units_are_read_while_the_ring_is_busy(data_file):
    """Slot units and pinned units mixed, two buffers and slow copies: every byte lands, the ring is never over-committed
    and pinned units are read while readers wait for buffers."""
    path, data = data_file
    n, unit_bytes = 40, 100_000
    r = np.random.default_rng(9)
    offsets = [int(x) for x in r.integers(0, FILE_BYTES - unit_bytes, size=n)]
    targets = [i // 2 if i % 2 == 0 else -(i // 2) - 1 for i in range(n)]
    st, device, host, stats, stride = run(path, offsets, targets, unit_bytes, 2, 2 * 102400, 6, 0, 1000)
    assert st == abi.SS_OK, last_error()
    check(data, offsets, targets, unit_bytes, device, host, stride)
    assert stats[2] == 10 and stats[5] <= 2


@pytest.mark.parametrize("where", ["slot", "host"])
def test_a_read_past_the_end_fails_the_run(data_file, where):
    path, _ = data_file
    unit_bytes = 65536
    offsets = [0, 65536, FILE_BYTES - 100, 131072, 196608, 262144]
    targets = [0, 1, 2 if where == "slot" else -1, 3, -2, 4]
    st, *_ = run(path, offsets, targets, unit_bytes, 2, unit_bytes, 4, 0, 300)
    assert st == abi.SS_E_IO, last_error()


@pytest.mark.parametrize("fail_batch", [0, 3, 7])
def test_a_refused_copy_fails_the_run(data_file, fail_batch):
    path, _ = data_file
    n = 16
    offsets = [i * 4096 for i in range(n)]
    targets = [i if i % 4 else -(i // 4) - 1 for i in range(n)]
    st, *_ = run(path, offsets, targets, 4096, 3, 4096, 5, 1, 500, fail_batch=fail_batch)
    assert st == abi.SS_E_BACKEND, last_error()
    assert "refused" in last_error()


def test_bad_arguments_are_refused(data_file):
    path, _ = data_file
    st, *_ = run(path, [0, 4096], [0, 1], 4096, 0, 4096, 2, 0, 0)
    assert st == abi.SS_E_INVALID  # slot units and no ring
    st, *_ = run(path, [0], [0], 8192, 1, 4096, 2, 0, 0)
    assert st == abi.SS_E_INVALID  # a buffer smaller than a unit
    st, *_ = run(path, [], [], 4096, 0, 4096, 2, 0, 0)
    assert st == abi.SS_OK  # nothing to read


def test_only_pinned_units_need_no_ring(data_file):
    path, data = data_file
    offsets = [i * 12345 for i in range(30)]
    targets = [-i - 1 for i in range(30)]
    st, device, host, stats, stride = run(path, offsets, targets, 12345, 0, 16384, 7, 0, 0)
    assert st == abi.SS_OK, last_error()
    check(data, offsets, targets, 12345, device, host, stride)
    assert list(stats[:3]) == [0, 30, 0]
