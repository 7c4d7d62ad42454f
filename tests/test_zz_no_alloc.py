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


_DEVICE1_FIRST = r"""
import json, sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
sys.path.insert(0, sys.argv[1] + "/tests")
from tierstream_b200 import abi
from test_zz_no_alloc import _tables
torch.cuda.set_device(1)  # nothing of the library has run on any device of this process yet
h = np.random.default_rng(13).integers(0, 256, size=(2 << 20) + 64, dtype=np.uint8)
data = torch.from_numpy(h).cuda()
base = data.data_ptr()
units = [[(base, 1 << 20)], [(base + (1 << 20), (1 << 20) + 64)]]
spans, sb, ns = _tables(units)
out = torch.zeros(2, dtype=torch.int64, device="cuda")
s = torch.cuda.Stream()
s.wait_stream(torch.cuda.current_stream())
got = []
for _ in range(2):  # two calls in a row on device 1
    abi.check(abi.load().tsb_xxh64_units_static(spans, sb, ns, 2, None, out.data_ptr(), None, s.cuda_stream))
    got.append([int(x) for x in out.cpu().numpy().view(np.uint64)])
print(json.dumps(got))
"""


@pytest.mark.gpu
def test_static_table_on_a_second_device_first(orc):
    """tsb_xxh64_units_static whose first call in a fresh process is on device 1 (its table looked up and its kernel's
    shared-memory attribute raised there, for that device): twice in a row, the oracle's hashes."""
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import json
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _DEVICE1_FIRST, root], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    got = json.loads(r.stdout.strip().splitlines()[-1])
    h = np.random.default_rng(13).integers(0, 256, size=(2 << 20) + 64, dtype=np.uint8)
    a, b = np.ascontiguousarray(h[:1 << 20]), np.ascontiguousarray(h[1 << 20:])
    want = [orc.orc_xxh64(a.ctypes.data, a.size, 0), orc.orc_xxh64(b.ctypes.data, b.size, 0)]
    assert got == [want, want]
