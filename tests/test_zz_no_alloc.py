"""tsb_xxh64_units_static (the device xxh64 with its unit table in the library's own device array) against
tsb_xxh64_units (caller scratch) and the oracle's xxh64, on two calls in a row. Collected last, and independent of
what ran before it."""
import ctypes as C

import numpy as np
import pytest

from tierstream_b200 import abi

MAX_UNITS = 4096


def _tables(units):
    n = len(units)
    spans = (C.c_void_p * (4 * n))()
    sb = (C.c_uint64 * (4 * n))()
    ns = (C.c_uint32 * n)()
    for i, u in enumerate(units):
        ns[i] = len(u)
        for s, (p, b) in enumerate(u):
            spans[4 * i + s] = p
            sb[4 * i + s] = b
    return spans, sb, ns


def test_static_refuses_more_units_than_its_table():
    lib = abi.load()
    one = (C.c_uint32 * 1)(1)
    st = lib.tsb_xxh64_units_static(None, None, one, MAX_UNITS + 1, None, None, None, None)
    assert st == abi.SS_E_INVALID
    assert b"at most 4096 units" in lib.ss_last_error()


@pytest.mark.gpu
def test_static_table_matches_caller_scratch_twice(orc):
    torch = pytest.importorskip("torch")
    lib = abi.load()
    rng = np.random.default_rng(11)
    data = torch.from_numpy(rng.integers(0, 256, size=8 << 20, dtype=np.uint8)).cuda()
    h = data.cpu().numpy()
    base = data.data_ptr()
    s = torch.cuda.Stream()

    def make(layouts, start):
        units, want, pos = [], [], start
        for spans in layouts:
            u, blob = [], []
            for b in spans:
                pos = (pos + 255) // 256 * 256
                u.append((base + pos, b))
                blob.append(h[pos:pos + b])
                pos += b
            units.append(u)
            cat = np.concatenate(blob)
            want.append(orc.orc_xxh64(cat.ctypes.data, cat.size, 0))
        return units, want

    first = make([[n] for n in [1, 31, 32, 33, 1000, 65536, (1 << 20) + 5]] + [[2048, 2048, 4096], [3, 5, 7, 9]], 0)
    # the second call hashes fewer units than the first: what the first left in the table must not matter
    second = make([[7], [4096, 17], [100000]], 4 << 20)
    for units, want in (first, second):
        n = len(units)
        spans, sb, ns = _tables(units)
        exp = torch.tensor(np.array(want, dtype=np.uint64).view(np.int64), device="cuda")
        exp[1] ^= 1  # one planted mismatch in the expectations
        out_a = torch.zeros(n, dtype=torch.int64, device="cuda")
        out_b = torch.zeros(n, dtype=torch.int64, device="cuda")
        mism_a = torch.zeros(1, dtype=torch.int32, device="cuda")
        mism_b = torch.zeros(1, dtype=torch.int32, device="cuda")
        scratch = torch.zeros(n * 72 // 8 + 1, dtype=torch.int64, device="cuda")
        # the zero fills and the planted mismatch ran on torch's current stream: the calls' stream waits for them
        s.wait_stream(torch.cuda.current_stream())
        abi.check(lib.tsb_xxh64_units(spans, sb, ns, n, scratch.data_ptr(), exp.data_ptr(), out_a.data_ptr(),
                                      mism_a.data_ptr(), s.cuda_stream))
        abi.check(lib.tsb_xxh64_units_static(spans, sb, ns, n, exp.data_ptr(), out_b.data_ptr(), mism_b.data_ptr(),
                                             s.cuda_stream))
        got_a = [int(x) for x in out_a.cpu().numpy().view(np.uint64)]
        got_b = [int(x) for x in out_b.cpu().numpy().view(np.uint64)]
        assert got_b == got_a == want
        assert int(mism_b.item()) == int(mism_a.item()) == 1
