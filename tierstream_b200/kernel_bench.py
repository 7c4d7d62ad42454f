"""Per-kernel rates through the C ABI, each timed with CUDA events on the launching stream after warm-up, with inputs
larger than L2: the land kernel (K1: one tsb_land launch per repetition) for pinned host -> HBM, HBM -> pinned host
and HBM -> HBM, the move kernel (K4: one tsb_move launch, HBM -> HBM, `--kernel move`), and the device xxh64 (K3: tsb_xxh64_units) for one unit alone (its serial chain) and for many
units at once (aggregate). Also the small cases the committed ncu summaries were captured on.

    python -m tierstream_b200.kernel_bench land --dir h2d --part-bytes 33030144 --parts 15
    python -m tierstream_b200.kernel_bench xxh64 --units 296 --part-bytes 12582912
"""
import argparse
import ctypes as C
import json

import torch

from . import abi


def _events(stream, fn, reps, warmup):
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(warmup):
        fn()
    stream.synchronize()
    times = []
    for _ in range(reps):
        a.record(stream)
        fn()
        b.record(stream)
        b.synchronize()
        times.append(a.elapsed_time(b))
    return times


def land(direction, part_bytes, parts, reps, warmup, kernel="land"):
    """One tsb_land launch (or tsb_move, HBM -> HBM through shared memory) of `parts` copies of part_bytes each (at
    most 384), grid chosen by the library."""
    assert 1 <= parts <= 384
    total = part_bytes * parts
    dev = torch.empty(total, dtype=torch.uint8, device="cuda")
    other = (torch.empty(total, dtype=torch.uint8).pin_memory() if direction in ("h2d", "d2h")
             else torch.empty(total, dtype=torch.uint8, device="cuda"))
    src, dst = {"h2d": (other, dev), "d2h": (dev, other), "d2d": (other, dev)}[direction]
    sp = (C.c_void_p * parts)(*[src.data_ptr() + i * part_bytes for i in range(parts)])
    dp = (C.c_void_p * parts)(*[dst.data_ptr() + i * part_bytes for i in range(parts)])
    by = (C.c_uint64 * parts)(*([part_bytes] * parts))
    s = torch.cuda.Stream()
    lib = abi.load()

    fn = lib.tsb_move if kernel == "move" else lib.tsb_land

    def once():
        abi.check(fn(sp, dp, by, parts, None, None, None, 0, None, 0, None, 0, s.cuda_stream))

    t = _events(s, once, reps, warmup)
    ms = sorted(t)[len(t) // 2]
    if kernel == "move":
        assert lib.tsb_move_timeouts() == 0
        assert torch.equal(dst[:1 << 20], src[:1 << 20]) and torch.equal(dst[-(1 << 20):], src[-(1 << 20):])
    return {"kernel": kernel, "dir": direction, "part_bytes": part_bytes, "parts": parts, "bytes": total,
            "ms_median": round(ms, 4), "gbs": round(total / ms / 1e6, 2),
            "hbm_traffic_gbs": round(total * (2 if direction == "d2d" else 1) / ms / 1e6, 2)}


def xxh64(units, part_bytes, n_parts, reps, warmup):
    """tsb_xxh64_units over `units` units of n_parts spans of part_bytes each, all in HBM."""
    unit_bytes = part_bytes * n_parts
    data = torch.empty(units * unit_bytes, dtype=torch.uint8, device="cuda")
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    data.random_(0, 256, generator=g)
    spans = (C.c_void_p * (4 * units))()
    sb = (C.c_uint64 * (4 * units))()
    ns = (C.c_uint32 * units)(*([n_parts] * units))
    for i in range(units):
        for p in range(n_parts):
            spans[4 * i + p] = data.data_ptr() + i * unit_bytes + p * part_bytes
            sb[4 * i + p] = part_bytes
    scratch = torch.empty(units * 72 // 8 + 1, dtype=torch.int64, device="cuda")
    out = torch.empty(units, dtype=torch.int64, device="cuda")
    s = torch.cuda.Stream()
    lib = abi.load()

    def once():
        # tsb_xxh64_units returns after its kernel ran; the events bracket the upload and the kernel
        abi.check(lib.tsb_xxh64_units(spans, sb, ns, units, scratch.data_ptr(), None, out.data_ptr(), None,
                                      s.cuda_stream))

    t = _events(s, once, reps, warmup)
    ms = sorted(t)[len(t) // 2]
    total = units * unit_bytes
    return {"kernel": "xxh64", "units": units, "unit_bytes": unit_bytes, "bytes": total, "ms_median": round(ms, 4),
            "gbs": round(total / ms / 1e6, 2), "per_unit_gbs": round(unit_bytes / ms / 1e6, 3)}


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="what", required=True)
    a1 = sub.add_parser("land")
    a1.add_argument("--dir", default="h2d", choices=["h2d", "d2h", "d2d"])
    a1.add_argument("--part-bytes", type=int, default=33030144)
    a1.add_argument("--parts", type=int, default=15)
    a1.add_argument("--kernel", default="land", choices=["land", "move"],
                    help="move: tsb_move (HBM -> HBM through shared memory by TMA bulk copies; --dir d2d only)")
    a2 = sub.add_parser("xxh64")
    a2.add_argument("--units", type=int, default=296)
    a2.add_argument("--part-bytes", type=int, default=12582912)
    a2.add_argument("--n-parts", type=int, default=3)
    for p in (a1, a2):
        p.add_argument("--reps", type=int, default=10)
        p.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    if a.what == "land":
        assert a.kernel == "land" or a.dir == "d2d", "the move kernel copies HBM -> HBM only"
        r = land(a.dir, a.part_bytes, a.parts, a.reps, a.warmup, a.kernel)
    else:
        r = xxh64(a.units, a.part_bytes, a.n_parts, a.reps, a.warmup)
    print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
