"""The file tier's reads on the CPU (tsb_test_file_read): a file read in pieces by the reader pool, buffered and
unbuffered (O_DIRECT: straight into an aligned destination, else through the bounce buffer), equals the file's bytes
for aligned and unaligned offsets, sizes and destinations; a read past the end fails with SS_E_IO."""
import ctypes as C
import mmap
import os

import numpy as np
import pytest

from tierstream_b200 import abi


@pytest.fixture(scope="module")
def data_file(tmp_path_factory):
    p = tmp_path_factory.mktemp("reads") / "src.bin"
    data = np.random.default_rng(3).integers(0, 256, size=(24 << 20) + 777, dtype=np.uint8)
    data.tofile(p)
    return str(p), data


@pytest.mark.parametrize("direct", [0, 1])
@pytest.mark.parametrize("offset,bytes_,piece,threads,dst_off", [
    (0, 24 << 20, 8 << 20, 8, 0),            # aligned: straight into the destination
    (4096, 9 << 20, 1 << 20, 4, 0),          # aligned, more pieces than threads
    (123, 5 << 20, 777 << 10, 3, 0),         # unaligned offset and pieces
    (8192, 3 << 20, 1 << 20, 2, 17),         # aligned file range, unaligned destination
    ((24 << 20) - 4096, 4096 + 777, 4096, 5, 0),  # the unaligned tail of the file
    (0, 1, 1, 1, 0),
])
def test_pieces_read_by_the_pool_equal_the_file(data_file, direct, offset, bytes_, piece, threads, dst_off):
    path, data = data_file
    buf = mmap.mmap(-1, bytes_ + dst_off + 4096)  # page aligned
    base = C.addressof(C.c_char.from_buffer(buf))
    abi.check(abi.load().tsb_test_file_read(path.encode(), offset, bytes_, base + dst_off, piece, threads, direct))
    got = np.frombuffer(buf, dtype=np.uint8, count=bytes_, offset=dst_off)
    assert np.array_equal(got, data[offset:offset + bytes_])
    del got
    buf.close()


def test_read_past_the_end_fails(data_file):
    path, data = data_file
    out = np.empty(8192, dtype=np.uint8)
    st = abi.load().tsb_test_file_read(path.encode(), data.size - 100, 8192, out.ctypes.data, 4096, 2, 1)
    assert st == abi.SS_E_IO
    assert st == abi.load().tsb_test_file_read(os.devnull.encode() + b"-missing", 0, 1, out.ctypes.data, 1, 1, 0)


@pytest.mark.parametrize("threads,reverse", [(1, 0), (3, 0), (4, 1), (8, 1)])
def test_reads_in_flight_equal_the_file(data_file, threads, reverse):
    """The file tier's reads in flight (dg_disk_queue > 1): many reads begun at once on a few reader threads and ended
    in order or in reverse each land their own bytes."""
    path, data = data_file
    rng = np.random.default_rng(threads)
    n, size = 24, 256 << 10
    offs = (rng.integers(0, (data.size - size) // 4096, size=n) * 4096).astype(np.uint64)
    buf = mmap.mmap(-1, n * size)
    base = C.addressof(C.c_char.from_buffer(buf))
    abi.check(abi.load().tsb_test_async_reads(path.encode(), offs.ctypes.data_as(C.POINTER(C.c_uint64)), n, size, base,
                                              threads, reverse))
    got = np.frombuffer(buf, dtype=np.uint8, count=n * size).reshape(n, size)
    for i in range(n):
        assert np.array_equal(got[i], data[int(offs[i]):int(offs[i]) + size]), i
    del got
    buf.close()


def test_a_failed_read_in_flight_is_reported_after_all_ended(data_file):
    path, data = data_file
    offs = np.array([0, data.size + 4096, 8192], dtype=np.uint64)  # the second one reads past the end
    out = mmap.mmap(-1, 3 * 4096)
    base = C.addressof(C.c_char.from_buffer(out))
    st = abi.load().tsb_test_async_reads(path.encode(), offs.ctypes.data_as(C.POINTER(C.c_uint64)), 3, 4096, base, 2, 0)
    assert st == abi.SS_E_IO
    got = np.frombuffer(out, dtype=np.uint8, count=3 * 4096)
    assert np.array_equal(got[:4096], data[:4096]) and np.array_equal(got[8192:], data[8192:12288])
    del got
    out.close()
