"""Measures the two movers the runtime chooses between, per piece size, on the current GPU: the copy engines
(cudaMemcpyAsync, through torch's copy_) and this library's land kernel (tsb_land, one launch per batch), for pinned
host -> HBM, HBM -> pinned host and HBM -> HBM. The runtime's default threshold (copy engines from 8 MiB parts up) comes
from this table on B200; TSB_CE_MIN_BYTES moves it.

    python -m tierstream_b200.calibrate [--total-mib 1024]
"""
import argparse
import ctypes as C
import json

import torch

from . import abi

SIZES = [128 << 10, 512 << 10, 2 << 20, 8 << 20, 14680064, 33030144]


def _time(fn, stream, reps=5):
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    fn()
    stream.synchronize()
    best = None
    for _ in range(reps):
        a.record(stream)
        fn()
        b.record(stream)
        b.synchronize()
        ms = a.elapsed_time(b)
        best = ms if best is None else min(best, ms)
    return best


def land(pairs, stream):
    n = len(pairs)
    for first in range(0, n, 384):
        part = pairs[first:first + 384]
        src = (C.c_void_p * len(part))(*[p[0] for p in part])
        dst = (C.c_void_p * len(part))(*[p[1] for p in part])
        by = (C.c_uint64 * len(part))(*[p[2] for p in part])
        abi.check(abi.load().tsb_land(src, dst, by, len(part), None, None, None, 0, None, 0, None, 0,
                                      stream.cuda_stream))


def concurrent_h2d(host, dev, size):
    """Pinned host -> HBM over the whole buffer in `size` parts, with the parts dealt round-robin to several movers
    running at once (each on a stream of its own; the time from the first start to the last end): one copy-engine
    stream, two, one with the land kernel, two with the land kernel. GB/s per arrangement."""
    n = host.numel() // size
    moved = n * size
    streams = [torch.cuda.Stream() for _ in range(3)]
    hp, dp = host.data_ptr(), dev.data_ptr()

    def run(movers):
        parts = [[i for i in range(n) if i % len(movers) == m] for m in range(len(movers))]
        start = torch.cuda.Event()
        start.record(streams[0])
        ends = []
        for m, kind in enumerate(movers):
            st = streams[m]
            st.wait_event(start)
            with torch.cuda.stream(st):
                if kind == "ce":
                    for i in parts[m]:
                        dev[i * size:(i + 1) * size].copy_(host[i * size:(i + 1) * size], non_blocking=True)
                else:
                    land([(hp + i * size, dp + i * size, size) for i in parts[m]], st)
            e = torch.cuda.Event()
            e.record(st)
            ends.append(e)
        for e in ends:
            streams[0].wait_event(e)

    out = {}
    for name, movers in (("ce_1_stream", ["ce"]), ("ce_2_streams", ["ce", "ce"]), ("ce_and_kernel", ["ce", "kernel"]),
                         ("ce_2_streams_and_kernel", ["ce", "ce", "kernel"])):
        out[name] = round(moved / _time(lambda: run(movers), streams[0]) / 1e6, 2)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--total-mib", type=int, default=1024)
    a = ap.parse_args()
    total = a.total_mib << 20
    host = torch.empty(total, dtype=torch.uint8).pin_memory()
    dev = torch.empty(total, dtype=torch.uint8, device="cuda")
    dev2 = torch.empty(total, dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    rows = []
    for size in SIZES:
        n = total // size
        moved = n * size
        r = {"piece_bytes": size, "pieces": n}
        with torch.cuda.stream(s):
            def ce(dst, src):
                return lambda: [dst[i * size:(i + 1) * size].copy_(src[i * size:(i + 1) * size], non_blocking=True)
                                for i in range(n)]
            r["h2d_ce_gbs"] = moved / _time(ce(dev, host), s) / 1e6
            r["d2h_ce_gbs"] = moved / _time(ce(host, dev), s) / 1e6
            r["d2d_ce_gbs"] = moved / _time(ce(dev2, dev), s) / 1e6
            hp, dp, d2p = host.data_ptr(), dev.data_ptr(), dev2.data_ptr()
            r["h2d_kernel_gbs"] = moved / _time(lambda: land([(hp + i * size, dp + i * size, size) for i in range(n)], s),
                                                s) / 1e6
            r["d2h_kernel_gbs"] = moved / _time(lambda: land([(dp + i * size, hp + i * size, size) for i in range(n)], s),
                                                s) / 1e6
            r["d2d_kernel_gbs"] = moved / _time(lambda: land([(dp + i * size, d2p + i * size, size) for i in range(n)],
                                                            s), s) / 1e6
        rows.append({k: (round(v, 2) if isinstance(v, float) else v) for k, v in r.items()})
        print(json.dumps(rows[-1]), flush=True)
    # the smallest piece size from which the copy engines beat the kernel on H2D, and stay ahead
    ce_min = None
    for r in rows:
        if r["h2d_ce_gbs"] >= r["h2d_kernel_gbs"]:
            ce_min = ce_min or r["piece_bytes"]
        else:
            ce_min = None
    print(json.dumps({"suggested_ce_min_bytes": ce_min, "device": torch.cuda.get_device_name()}))
    print(json.dumps({"h2d_concurrent_gbs": concurrent_h2d(host, dev, 33030144), "part_bytes": 33030144}))


if __name__ == "__main__":
    main()
