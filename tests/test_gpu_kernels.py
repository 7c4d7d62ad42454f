"""The data-path kernels through the C ABI (tsb_land, tsb_xxh64_units) against the oracle: land copies are byte
exact in every direction and alignment, their entries and ready word are published, and the device xxh64 equals the
reference's host xxh64 bit for bit."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from tierstream_b200 import abi  # noqa: E402

P = C.POINTER


def land(srcs, dsts, sizes, stream, slot_of=None, keys=(), vals=(), ready=None, ready_val=0, counter=None, blocks=0):
    n = len(srcs)
    s = (C.c_void_p * max(n, 1))(*srcs)
    d = (C.c_void_p * max(n, 1))(*dsts)
    b = (C.c_uint64 * max(n, 1))(*sizes)
    k = (C.c_uint32 * max(len(keys), 1))(*keys)
    v = (C.c_int32 * max(len(vals), 1))(*vals)
    abi.check(abi.load().tsb_land(s, d, b, n, slot_of, k, v, len(keys), ready, ready_val, counter, blocks, stream))


def test_land_host_to_device_any_alignment():
    rng = np.random.default_rng(1)
    host = torch.from_numpy(rng.integers(0, 256, size=8 << 20, dtype=np.uint8)).pin_memory()
    dev = torch.zeros(8 << 20, dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())  # after the inputs torch made on its own stream
    # copies of assorted sizes and offsets, disjoint destinations
    plan, pos = [], 0
    for size in [1, 15, 16, 17, 255, 4096, 65535, 65536, 65537, 1 << 20, 3 * 1000 + 7, 2 << 20]:
        src_off = int(rng.integers(0, 64))
        plan.append((src_off + pos, pos + int(rng.integers(0, 32)), size))
        pos += size + 64
    land([host.data_ptr() + a for a, _, _ in plan], [dev.data_ptr() + b for _, b, _ in plan], [n for *_, n in plan],
         s.cuda_stream)
    s.synchronize()
    h, d = host.numpy(), dev.cpu().numpy()
    for a, b, n in plan:
        assert np.array_equal(d[b:b + n], h[a:a + n]), (a, b, n)


def test_land_publishes_entries_and_ready_after_copies():
    rng = np.random.default_rng(2)
    n_units, unit = 24, 3 << 20
    host = torch.from_numpy(rng.integers(0, 256, size=n_units * unit, dtype=np.uint8)).pin_memory()
    dev = torch.zeros(n_units * unit, dtype=torch.uint8, device="cuda")
    slot_of = torch.full((64,), -1, dtype=torch.int32, device="cuda")
    words = torch.zeros(4, dtype=torch.int32, device="cuda")  # [0] counter, [1] ready
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())  # after the inputs torch made on its own stream
    order = rng.permutation(n_units)
    land([host.data_ptr() + int(u) * unit for u in order], [dev.data_ptr() + i * unit for i in range(n_units)],
         [unit] * n_units, s.cuda_stream, slot_of=slot_of.data_ptr(), keys=[int(u) for u in order],
         vals=list(range(n_units)), ready=words.data_ptr() + 4, ready_val=77, counter=words.data_ptr())
    s.synchronize()
    so = slot_of.cpu().numpy()
    for i, u in enumerate(order):
        assert so[u] == i
    assert words[1].item() == 77 and words[0].item() == 0  # ready published, counter re-zeroed
    assert np.array_equal(dev.cpu().numpy(), host.numpy().reshape(n_units, unit)[order].reshape(-1))


def test_land_device_to_host_and_device_to_device():
    rng = np.random.default_rng(3)
    src = torch.from_numpy(rng.integers(0, 256, size=4 << 20, dtype=np.uint8)).cuda()
    host = torch.zeros(4 << 20, dtype=torch.uint8).pin_memory()
    dev2 = torch.zeros(4 << 20, dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())  # after the inputs torch made on its own stream
    half = 2 << 20
    land([src.data_ptr(), src.data_ptr() + half], [host.data_ptr(), dev2.data_ptr() + half], [half, half],
         s.cuda_stream, blocks=7)
    s.synchronize()
    a = src.cpu().numpy()
    assert np.array_equal(host.numpy()[:half], a[:half])
    assert np.array_equal(dev2.cpu().numpy()[half:], a[half:])


def xxh_units(units, expect=None):
    """units: list of lists of (device ptr, bytes). Returns (hashes, mismatches)."""
    lib = abi.load()
    n = len(units)
    spans = (C.c_void_p * (4 * n))()
    sb = (C.c_uint64 * (4 * n))()
    ns = (C.c_uint32 * n)()
    for i, u in enumerate(units):
        ns[i] = len(u)
        for j, (p, b) in enumerate(u):
            spans[4 * i + j] = p
            sb[4 * i + j] = b
    scratch = torch.zeros(n * 72 // 8 + 1, dtype=torch.int64, device="cuda")
    out = torch.zeros(n, dtype=torch.int64, device="cuda")
    mism = torch.zeros(1, dtype=torch.int32, device="cuda")
    exp = torch.tensor(np.array(expect, dtype=np.uint64).view(np.int64), device="cuda") if expect else None
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())  # the zero fills and the expectations were made on torch's stream
    abi.check(lib.tsb_xxh64_units(spans, sb, ns, n, scratch.data_ptr(), exp.data_ptr() if exp is not None else None,
                                  out.data_ptr(), mism.data_ptr() if exp is not None else None, s.cuda_stream))
    return out.cpu().numpy().view(np.uint64), int(mism.item())


def test_device_xxh64_matches_oracle(orc):
    rng = np.random.default_rng(4)
    data = torch.from_numpy(rng.integers(0, 256, size=16 << 20, dtype=np.uint8)).cuda()
    h = data.cpu().numpy()
    base = data.data_ptr()
    units, want, pos = [], [], 0
    # one-span units of every tail length, multi-span units (32-byte multiples but the last), odd spans (one-lane path)
    layouts = [[n] for n in [0, 1, 5, 8, 31, 32, 33, 64, 100, 1024, 1025, 4096 + 17, 65536, 1 << 20, (3 << 20) + 3]]
    layouts += [[2048, 2048, 4096], [256, 512, 256, 1000], [32, 32], [4096, 9]]
    layouts += [[1000, 24], [3, 5, 7], [33, 64]]
    for spans in layouts:
        u, blob = [], []
        for b in spans:
            pos = (pos + 255) // 256 * 256
            u.append((base + pos, b))
            blob.append(h[pos:pos + b])
            pos += b
        units.append(u)
        cat = np.concatenate(blob) if blob else np.zeros(0, dtype=np.uint8)
        want.append(orc.orc_xxh64(cat.ctypes.data, cat.size, 0))
    got, _ = xxh_units(units)
    assert [int(x) for x in got] == want
    bad = list(want)
    bad[3] ^= 1
    _, mism = xxh_units(units, expect=bad)
    assert mism == 1


def test_device_xxh64_many_units_random_layouts(orc):
    """Many CTAs (16 units each), units of 1-4 spans whose chunk boundaries cross span boundaries, staged and
    one-lane units mixed in one launch."""
    rng = np.random.default_rng(12)
    data = torch.from_numpy(rng.integers(0, 256, size=48 << 20, dtype=np.uint8)).cuda()
    h = data.cpu().numpy()
    base = data.data_ptr()
    units, want, pos = [], [], 0
    for i in range(150):
        n_sp = int(rng.integers(1, 5))
        spans = [int(rng.integers(1, 3000)) * 32 for _ in range(n_sp - 1)] + [int(rng.integers(0, 90000))]
        misalign = i % 13 == 5  # a span off the 16-byte grid: the one-lane path
        u, blob = [], []
        for b in spans:
            pos = (pos + 255) // 256 * 256 + (8 if misalign else 0)
            u.append((base + pos, b))
            blob.append(h[pos:pos + b])
            pos += b
        units.append(u)
        cat = np.concatenate(blob)
        want.append(orc.orc_xxh64(cat.ctypes.data, cat.size, 0))
    assert pos < h.size
    got, _ = xxh_units(units)
    assert [int(x) for x in got] == want


def test_move_kernel_copies_and_publishes():
    """K4 (tsb_move): HBM -> HBM batches through shared memory by TMA bulk copies, 16-byte aligned copies of assorted
    sizes (below, at and above the 64 KiB chunk, many in one batch), then the entries and the ready word published, on
    two launches in a row with the same completion counter."""
    rng = np.random.default_rng(7)
    plans = []
    for rep in range(2):
        plan, pos = [], 0
        for size in [16, 4096, 65520, 65536, 65552, 1 << 20, 3 * (1 << 20) + 48] + [4096 * int(x) for x in
                                                                                      rng.integers(1, 64, size=200)]:
            plan.append((pos, pos, size))
            pos += (size + 255) // 256 * 256
        plans.append((plan, pos))
    total = max(pos for _, pos in plans)
    src = torch.from_numpy(rng.integers(0, 256, size=total, dtype=np.uint8)).cuda()
    dst = torch.zeros(total, dtype=torch.uint8, device="cuda")
    table = torch.full((64,), -1, dtype=torch.int32, device="cuda")
    words = torch.zeros(4, dtype=torch.int32, device="cuda")  # [0] ready, [1] counter
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())  # after the inputs torch made on its own stream
    lib = abi.load()
    for rep, (plan, pos) in enumerate(plans):
        assert pos <= src.numel() and pos <= dst.numel()
        dst.zero_()
        n = len(plan)
        sp = (C.c_void_p * n)(*[src.data_ptr() + a for a, _, _ in plan])
        dp = (C.c_void_p * n)(*[dst.data_ptr() + b for _, b, _ in plan])
        by = (C.c_uint64 * n)(*[z for *_, z in plan])
        assert n <= 384 and all(a + z <= total and a % 16 == 0 and z % 16 == 0 for a, _, z in plan)
        s.wait_stream(torch.cuda.current_stream())
        keys = (C.c_uint32 * 3)(3, 9, 60)
        vals = (C.c_int32 * 3)(7 + rep, 8 + rep, 9 + rep)
        abi.check(lib.tsb_move(sp, dp, by, n, C.c_void_p(table.data_ptr()), keys, vals, 3,
                               C.c_void_p(words.data_ptr()), 41 + rep, C.c_void_p(words.data_ptr() + 4), 0,
                               s.cuda_stream))
        s.synchronize()
        assert lib.tsb_move_timeouts() == 0
        h, d = src.cpu().numpy(), dst.cpu().numpy()
        for a, b, z in plan:
            assert np.array_equal(d[b:b + z], h[a:a + z]), "copy of %d bytes differs" % z
        t = table.cpu().numpy()
        assert t[3] == 7 + rep and t[9] == 8 + rep and t[60] == 9 + rep
        assert int(words[0].item()) == 41 + rep and int(words[1].item()) == 0  # the counter is back at zero


def test_move_kernel_refuses_unaligned():
    lib = abi.load()
    src = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    sp = (C.c_void_p * 1)(src.data_ptr() + 8)
    dp = (C.c_void_p * 1)(src.data_ptr() + 512)
    by = (C.c_uint64 * 1)(64)
    st = lib.tsb_move(sp, dp, by, 1, None, None, None, 0, None, 0, None, 0, None)
    assert st == abi.SS_E_INVALID and b"multiple of 16" in lib.ss_last_error()


_DEVICE_CHILD = r"""
import json, sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
sys.path.insert(0, sys.argv[1] + "/tests")
from test_gpu_kernels import xxh_units
out = {}
for dev in (0, 1):  # device 0 first: device 1's first K3 launch comes after the library already ran on device 0
    torch.cuda.set_device(dev)
    h = np.random.default_rng(7).integers(0, 256, size=(3 << 20) + 40, dtype=np.uint8)
    data = torch.from_numpy(h).cuda()
    base = data.data_ptr()
    units = [[(base, 1 << 20)], [(base + (1 << 20), 1 << 20), (base + (2 << 20), (1 << 20) + 40)]]
    got, _ = xxh_units(units)
    out[dev] = [int(x) for x in got]
print(json.dumps(out))
"""


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_xxh64_on_a_second_device_of_a_fresh_process(orc):
    """K3's shared-memory attribute is set per device: a fresh process that hashes on device 0 and then, with nothing
    of the library opened on device 1, on device 1 gets the oracle's hashes on both."""
    import json
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _DEVICE_CHILD, root], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    got = json.loads(r.stdout.strip().splitlines()[-1])
    h = np.random.default_rng(7).integers(0, 256, size=(3 << 20) + 40, dtype=np.uint8)
    a, b = h[:1 << 20], h[1 << 20:]
    want = [orc.orc_xxh64(np.ascontiguousarray(a).ctypes.data, a.size, 0),
            orc.orc_xxh64(np.ascontiguousarray(b).ctypes.data, b.size, 0)]
    assert got["0"] == want and got["1"] == want
