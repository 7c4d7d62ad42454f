"""Host forward mode workloads of bench.py (`--workload c1-host`, `--workload llama3-70b-host`)
and configs[2], the reference's host-mode submit path (src/stream_ctx.cpp:433-470, ss_layer_all at :1391) on one GPU.

c1-host (C1): 8 layers x 16 experts x 3 parts of 131,072 random bytes (generator seed 0), top-2 routes per token
uniform (seed 1), plan order "ranked", 4 experts per layer resident in VRAM and the other 12 pinned, a 4-slot stream
ring, inclusive tiers, every unit checked against its descriptor xxh64 at the open (verify_hash).

llama3-70b-host (C3): 80 layers, one blob per layer of 1,711,308,800 bytes (Llama-3-70B's 855,654,400 bf16
parameters per layer: q and o 8192 x 8192, k and v 8192 x 1024, gate / up / down 8192 x 28672, two 8192 norms) as
random bytes, prefix order, the first 35 layers resident (59.9 GB: the 60 GB VRAM budget), the other 45 pinned and
streamed every token through a 2-slot ring with ss_layer_all. The model file (137 GB) is larger than the GPU box's
disk, so it is a sparse file: after the open every kept copy (the residents' slots and the pinned blocks) is written
on the device from the byte generator (tsb_test_host_unit gives their addresses), so the streamed bytes are the
generator's and every reader's checksum is compared with the generator's.

One token is one forward of tse_host_forward (libtsb_engine.so): an engine's native loop over the layers - routes,
ss_acquire on the engine stream, a reader of every routed unit through the acquired device table, ss_release - then
ss_end. The metric is the streamed bytes (units copied to the device by the forwards: admitted + transient) per
second. No oracle is used here: bench.py adds the reference's CPU backend beside it.
"""
import ctypes as C
import json
import os
import time

import numpy as np

from . import abi, harness, runtime, synth

C3_BLOB = 8192 * 8192 * 2 + 8192 * 1024 * 2 + 3 * 8192 * 28672 + 2 * 8192  # parameters per layer
WORKLOADS = {
    "c1-host": dict(layers=8, units=16, parts=(131072,) * 3, top_k=2, resident=4, ring=4, seed=0, order="ranked",
                    blob=False, sparse=False, hashed=True, slices=16, steps=64, warmup=8,
                    metric="host-mode stream GB/s (C1: 8 x 16 experts of 3 x 128 KiB, top-2 uniform routes)",
                    file="tsb-bench-c1-host.bin"),
    "llama3-70b-host": dict(layers=80, units=1, parts=(2 * C3_BLOB,), top_k=1, resident=35, ring=2, seed=7,
                            order="prefix", blob=True, sparse=True, hashed=False, slices=1184, steps=12, warmup=3,
                            metric="host-mode stream GB/s (C3: Llama-3-70B-shaped dense blobs through a 2-slot ring)",
                            file="tsb-bench-llama3-70b-host.bin"),
}


def model_of(name):
    w = WORKLOADS[name]
    return synth.Model(os.path.join(harness.model_dir(), w["file"]), w["layers"], w["units"], w["parts"],
                       seed=w["seed"], top_k=w["top_k"], with_hash=w["hashed"])


def desc_of(name, m):
    w = WORKLOADS[name]
    d = json.loads(m.desc(order=w["order"]))
    if w["blob"]:
        for lay in d["layers"]:
            lay["kind"] = "blob"
            lay.pop("top_k")
            lay["parts"][0]["name"] = "blob"
    return json.dumps(d)


def tiers_of(name):
    w = WORKLOADS[name]
    if w["blob"]:
        return [abi.SS_TIER_RESIDENT] * w["resident"] + [abi.SS_TIER_PINNED] * (w["layers"] - w["resident"])
    per = [abi.SS_TIER_RESIDENT] * w["resident"] + [abi.SS_TIER_PINNED] * (w["units"] - w["resident"])
    return per * w["layers"]


def budget_options(name, m):
    """(ss_budget, ss_options) of the workload: the VRAM of its residents and ring, the pinned RAM of its other units."""
    w = WORKLOADS[name]
    b = abi.budget_defaults()
    residents = w["resident"] if w["blob"] else w["resident"] * w["layers"]
    b.device_bytes = (residents + w["ring"] + 4) * m.unit_bytes + (1 << 30)
    b.margin_gib = 1.0 / 1024
    b.margin_fraction = 0.0
    b.ring_slots = w["ring"]
    b.dynamic_slots_per_layer = 0
    b.host_pinned_bytes = m.layers * m.units * m.unit_bytes + (1 << 30)
    o = abi.options_defaults()
    o.forward_mode = abi.SS_FORWARD_HOST
    o.verify_hash = 1 if w["hashed"] else 0
    return b, o


def routes_of(name, tokens):
    """int32 [tokens][layers][top_k]: C1's uniform top-2 routes from seed 1; C3's whole layers (unit 0)."""
    w = WORKLOADS[name]
    if w["blob"]:
        return np.zeros((tokens, w["layers"], 1), dtype=np.int32)
    return synth.zipf_trace(tokens, w["layers"], w["units"], w["top_k"], seed=1, uniform=True)


def fill_from_generator(ctx, m, torch):
    """Every kept copy of every unit (its pinned block, its resident slot) written on the device from the byte
    generator; the first and last units' pinned bytes checked against the host generator. (Sparse model files.)"""
    eng = abi.load_engine()
    s = torch.cuda.Stream()
    kept = []
    for L in range(m.layers):
        for u in range(m.units):
            off = np.array([m.unit_offset(L, u)], dtype=np.uint64)
            for addr in ctx.unit_home(L, u):
                if addr:
                    rc = eng.tse_fill_units_device(m.seed, off.ctypes.data_as(C.POINTER(C.c_uint64)), 1,
                                                   m.unit_bytes, C.c_void_p(addr), s.cuda_stream)
                    assert rc == 0, "device fill failed: %d" % rc
            kept.append((L, u))
    s.synchronize()
    for L, u in (kept[0], kept[-1]):
        host, _ = ctx.unit_home(L, u)
        if host:  # mapped pinned memory: readable from the host at the same address
            got = np.ctypeslib.as_array((C.c_uint8 * min(m.unit_bytes, 1 << 20)).from_address(host))
            want = np.empty(got.size, dtype=np.uint8)
            eng.tse_fill_bytes(m.seed, m.unit_offset(L, u), want.size, want.ctypes.data, 4)
            assert np.array_equal(got, want), "pinned fill of (%d, %d) differs from the generator" % (L, u)


def streamed_units(ctx, layers):
    tot = 0
    for L in range(layers):
        s = ctx.layer_stats(L)
        tot += s["admitted"] + s["transient"]
    return tot


def run(name, steps, warmup, torch, clocks_cls, local):
    """The GPU leg: (line fields, routes of the timed device leg, routes of the e2e leg) - device-timed forwards with the
    ids already in pinned memory and the results kept on the device, then the e2e forwards each followed by the
    results' copy back and a synchronize; every reader's checksum compared with the generator's."""
    w = WORKLOADS[name]
    m = model_of(name)
    t_file = time.perf_counter()
    if w["sparse"]:
        m.create_sparse()
    else:
        m.write()
    t_file = time.perf_counter() - t_file
    desc_json = desc_of(name, m)
    desc = runtime.Desc(desc_json)
    b, o = budget_options(name, m)
    plan = runtime.Plan(desc, b, tiers=tiers_of(name))
    trace = routes_of(name, warmup + 2 * steps + 1)
    all_layers = np.full(m.layers, 1 if w["blob"] else 0, dtype=np.uint8)
    n_ids = trace.shape[2]
    keys_all = np.arange(m.layers)[None, :, None] * m.units + trace
    eng = abi.load_engine()
    t_open = time.perf_counter()
    ctx = runtime.HostContext(desc, plan, o)
    try:
        t_open = time.perf_counter() - t_open
        t_fill = time.perf_counter()
        if w["sparse"]:
            fill_from_generator(ctx, m, torch)
        t_fill = time.perf_counter() - t_fill
        # expected checksums of every unit in both modes, from the generator on the device (outside the timed regions)
        t_exp = time.perf_counter()
        want = {mode: harness.expected_sums(m, np.arange(m.layers * m.units), mode, slices=w["slices"])
                for mode in (0, 1)}
        t_exp = time.perf_counter() - t_exp
        routes_h = torch.from_numpy(trace.reshape(trace.shape[0], -1).copy()).pin_memory()
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        ids_dev = torch.zeros(m.layers * n_ids, dtype=torch.int32, device="cuda")
        outs_dev = torch.zeros((steps, m.layers * n_ids), dtype=torch.int64, device="cuda")
        out_e2e = torch.zeros(m.layers * n_ids, dtype=torch.int64, device="cuda")
        out_host = torch.zeros(m.layers * n_ids, dtype=torch.int64).pin_memory()

        def forward(t, out, mode):
            rc = eng.tse_host_forward(ctx.h, desc.h, C.c_void_p(routes_h[t].data_ptr()), n_ids,
                                      all_layers.ctypes.data_as(C.c_void_p), C.c_void_p(ids_dev.data_ptr()),
                                      C.c_void_p(out.data_ptr()), w["slices"], mode, C.c_void_p(stream.cuda_stream))
            if rc != 0:
                raise RuntimeError("tse_host_forward failed: %d (%s)" % (rc, abi.load().ss_last_error().decode()))

        for t in range(warmup):
            forward(t, out_e2e, 1)
        stream.synchronize()
        # (1) device-timed: ids in pinned host memory, results kept on the device
        u0 = streamed_units(ctx, m.layers)
        l0 = json.loads(ctx.stats_json())["land_launches"]
        clocks = clocks_cls(local)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for t in range(steps):
            forward(warmup + t, outs_dev[t], 1)
        e1.record(stream)
        e1.synchronize()
        clk = clocks.stop()
        dev_ms = e0.elapsed_time(e1)
        u1 = streamed_units(ctx, m.layers)
        l1 = json.loads(ctx.stats_json())["land_launches"]
        # (2) end to end: the results copied back and waited for every forward, positional checksums
        base = warmup + steps
        forward(base, out_e2e, 0)
        stream.synchronize()
        outs2 = np.zeros((steps, m.layers * n_ids), dtype=np.uint64)
        u2 = streamed_units(ctx, m.layers)
        import gc
        gc.collect()  # the interpreter's collector off while the host drives the timed forwards (on again after)
        gc.disable()
        try:
            w0 = time.perf_counter()
            for t in range(steps):
                forward(base + 1 + t, out_e2e, 0)
                with torch.cuda.stream(stream):
                    out_host.copy_(out_e2e, non_blocking=True)
                stream.synchronize()
                outs2[t] = out_host.numpy().view(np.uint64)
            e2e_s = time.perf_counter() - w0
        finally:
            gc.enable()
        u3 = streamed_units(ctx, m.layers)
        stats = json.loads(ctx.stats_json())
    finally:
        ctx.close()
    got1 = outs_dev.cpu().numpy().view(np.uint64)
    keys1 = keys_all[warmup:warmup + steps].reshape(steps, -1)
    keys2 = keys_all[base + 1:base + 1 + steps].reshape(steps, -1)
    if w["blob"]:  # one unit per layer: only each layer's first id slot is read
        got1, keys1, outs2, keys2 = got1[:, ::n_ids], keys1[:, ::n_ids], outs2[:, ::n_ids], keys2[:, ::n_ids]
    bad = int((got1 != want[1][keys1]).sum()) + int((outs2 != want[0][keys2]).sum())
    moved = (u1 - u0) * m.unit_bytes
    moved_e2e = (u3 - u2) * m.unit_bytes
    line = {
        "metric": w["metric"], "value": round(moved / (dev_ms / 1e3) / 1e9, 3), "unit": "GB/s", "n_gpus": 1,
        "steps": steps, "warmup": warmup, "ms_per_step": round(dev_ms / steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic (seeded random bytes%s)" % (", uniform routes" if not w["blob"] else ""),
        "config": {"workload": name, "layers": m.layers, "units_per_layer": m.units, "unit_bytes": m.unit_bytes,
                   "parts": list(w["parts"]), "top_k": w["top_k"] if not w["blob"] else None,
                   "resident": w["resident"], "ring_slots": w["ring"], "order": w["order"], "mode": "host forward",
                   "model_file": "sparse; kept copies written from the generator" if w["sparse"] else "written",
                   "l2": "inputs larger than L2" if m.unit_bytes * m.layers > (126 << 20) else
                         "C1's whole model (50 MB) fits L2; each forward's copies land in new slots"},
        "tokens_per_s": round(steps / (dev_ms / 1e3), 3),
        "streamed_units_per_token": round((u1 - u0) / steps, 3),
        "e2e": {"value": round(moved_e2e / e2e_s / 1e9, 3), "unit": "GB/s",
                "h2d_bytes_per_step": m.layers * n_ids * 4, "d2h_bytes_per_step": m.layers * n_ids * 8,
                "tokens_per_s": round(steps / e2e_s, 3)},
        "verified": {"tokens": 2 * steps, "units": int(got1.size + outs2.size), "mismatches": bad,
                     "how": "every unit each forward's reader read through the acquired device table: word sums in the "
                            "device-timed leg, positional checksums in the e2e leg, against sums computed on the "
                            "device from the byte generator alone (%.1f s, outside the timed regions)" % t_exp},
        "gpu_launches": int(l1 - l0) + steps * m.layers,  # device-timed leg: the runtime's land kernels + readers
        "clocks": clk,
        "open_s": round(t_open, 2), "fill_s": round(t_fill, 2), "file_s": round(t_file, 2),
        "host_stats": {"forwards": stats["forwards"], "land_launches": stats["land_launches"], "total": stats["total"]},
    }
    return line, trace, bad
