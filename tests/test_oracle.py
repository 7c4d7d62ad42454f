"""The oracle (oracle/oracle.c) pinned against the reference's own known answers and its compiled sources, and the
library's host xxh64 against both."""
import ctypes as C

import numpy as np
import pytest

# tests/test_core.cpp:64-82 of the reference: XXH64 known answers (seed 0)
KATS = [(b"", 0xEF46DB3751D8E999), (b"a", 0xD24EC4F1A98C6E5B), (b"abc", 0x44BC2CF5AD770999),
        (b"Nobody inspects the spammish repetition", 0xFBCEA83C8A378BF1)]


@pytest.mark.parametrize("data,want", KATS)
def test_oracle_xxh64_known_answers(orc, data, want):
    assert orc.orc_xxh64(data, len(data), 0) == want


@pytest.mark.parametrize("data,want", KATS)
def test_library_host_xxh64_known_answers(lib, data, want):
    buf = C.create_string_buffer(data, len(data) or 1)
    assert lib.tsb_xxh64(buf, len(data), 0) == want


def test_oracle_streaming_equals_one_shot(orc):
    # the reference test's pattern: bytes i*131+7, fed in pieces of growing size (test_core.cpp:74-81)
    big = np.array([(i * 131 + 7) & 0xFF for i in range(10007)], dtype=np.uint8)
    ptrs, lens, pos, step = [], [], 0, 1
    while pos < big.size:
        n = min(step, big.size - pos)
        ptrs.append(big.ctypes.data + pos)
        lens.append(n)
        pos += n
        step = step * 3 + 1
    P = (C.c_void_p * len(ptrs))(*ptrs)
    L = (C.c_uint64 * len(lens))(*lens)
    assert orc.orc_xxh64_spans(P, L, len(ptrs), 0) == orc.orc_xxh64(big.ctypes.data, big.size, 0)


@pytest.mark.parametrize("size", [0, 1, 3, 4, 7, 8, 31, 32, 33, 63, 64, 100, 255, 256, 4096, 65537, 1 << 20])
def test_oracle_and_library_match_reference_xxh64(orc, ref, lib, size):
    rng = np.random.default_rng(size)
    for seed in (0, 1, 0x9E3779B97F4A7C15):
        data = rng.integers(0, 256, size=max(size, 1), dtype=np.uint8)
        want = ref.oref_xxh64(data.ctypes.data, size, seed)
        assert orc.orc_xxh64(data.ctypes.data, size, seed) == want
        assert lib.tsb_xxh64(data.ctypes.data, size, seed) == want


def test_fill_bytes_restates_fixture_generator(orc):
    # byte_at(file_id, i) of the reference fixtures (tests/fixture.hpp:16-22), restated in Python
    def byte_at(fid, i):
        m = (1 << 64) - 1
        x = (((i + 1) * 0x9E3779B97F4A7C15) & m) ^ (((fid + 7) * 0xC2B2AE3D27D4EB4F) & m)
        x ^= x >> 29
        x = (x * 0xBF58476D1CE4E5B9) & m
        x ^= x >> 32
        return x & 0xFF
    out = np.empty(300, dtype=np.uint8)
    orc.orc_fill_bytes(3, 1000, 300, out.ctypes.data)
    assert [int(v) for v in out] == [byte_at(3, 1000 + i) for i in range(300)]


def test_engine_filler_matches_oracle(orc):
    from tierstream_b200 import abi
    eng = abi.load_engine()
    a = np.empty(1 << 16, dtype=np.uint8)
    b = np.empty(1 << 16, dtype=np.uint8)
    eng.tse_fill_bytes(5, 123457, a.size, a.ctypes.data, 4)
    orc.orc_fill_bytes(5, 123457, b.size, b.ctypes.data)
    assert np.array_equal(a, b)


def test_export_mask_and_slot_rules(orc):
    slot_of = np.array([3, -1, 7, -1, 0, 2], dtype=np.int32)
    base = np.array([0, 4, 6], dtype=np.uint32)  # two gated layers of 4 and 2 units
    ids = np.array([0, 1, 3, 2, 1], dtype=np.int32)
    bad = C.c_uint32()
    m = orc.orc_export_mask(slot_of.ctypes.data, 0, 4, ids.ctypes.data, 5, C.byref(bad))
    assert m == 0b10110 and bad.value == 0
    ids2 = np.array([0, 4], dtype=np.int32)
    orc.orc_export_mask(slot_of.ctypes.data, 4, 2, ids2.ctypes.data, 2, C.byref(bad))
    assert bad.value == 1
    absent = C.c_uint32(0)
    assert orc.orc_dg_slot(slot_of.ctypes.data, base.ctypes.data, 0, 2, 99, 0, C.byref(absent)) == 7
    assert orc.orc_dg_slot(slot_of.ctypes.data, base.ctypes.data, 1, 5, 99, 0, C.byref(absent)) == 99
    assert absent.value == 0
    assert orc.orc_dg_slot(slot_of.ctypes.data, base.ctypes.data, 0, 1, 99, 0, C.byref(absent)) == 99
    assert absent.value == 1
    assert orc.orc_dg_slot(slot_of.ctypes.data, base.ctypes.data, 0, 0, 99, 1, C.byref(absent)) == 99
