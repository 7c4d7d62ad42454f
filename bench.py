"""Benchmark: the expert-miss stream of device-gated decode (Mixtral-8x7B-shaped MoE on one B200).

Workload "mixtral-8x7b-dg": 32 MoE layers x 8 experts, each expert three parts (gate / up / down) of 33,030,144 bytes
(14336 x 4096 x 4.5 bits), random bytes (the synthetic generator, seeded); VRAM budget 40 % of the experts (102
residents, the most popular by layer, +1 spare slot per layer, 2 banks of 2 + the guard), the rest in pinned RAM,
exclusive tiers; batch-1 decode with top-2 Zipf(1.1) routes, one token = one step: ss_begin, the captured graph
(begin; per layer export -> wait -> the engine's reader of the two routed experts; end), ss_end.

Printed metric: expert-miss stream GB/s = bytes landed by the miss service (demand + prefetch copies) per second of
decode, aggregated over ranks. N > 1 (one process per GPU) runs the peer tier by default ("mixtral-8x7b-dg-peer"):
each rank decodes its own trace, every expert is owned by one rank's HBM store (owners planned from the ranks' summed
routing counts, one NCCL all-reduce), and a miss is copied from its owner's store over NVLink (or from the rank's own
store) instead of pinned RAM; `--tier pinned` runs N independent pinned-RAM replicas instead. `--tier file` (one GPU)
runs the file tier ("mixtral-8x7b-dg-file"): every non-resident expert lives in the model file only and a miss reads
it (O_DIRECT) into a pinned staging buffer, then copies it to HBM.
`value` is device time (CUDA events on the engine stream) with the routed ids already in HBM; `e2e` is the same steps
through the public ABI with the ids copied from pinned host memory and the readers' results copied back each step,
timed by the host clock. `--impl reference` times the reference's own DgCore (compiled from its sources) with a host
memcpy transport on the host cores, the same trace and metric.
"""
import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LAYERS, UNITS, PART = 32, 8, 33030144
TOP_K, ZIPF, RESIDENTS, SPARE, RHO = 2, 1.1, 102, 1, 0.0
METRIC = "expert-miss stream GB/s (device-gated decode, Mixtral-8x7B-shaped MoE)"
WORKLOAD, MODEL_FILE = "mixtral-8x7b-dg", "tsb-bench-mixtral-dg.bin"
# BASELINE configs[4] (C5): 94 layers x 128 experts of 3 x 12,582,912 B (4096 x 1536 bf16), top-8 Zipf(1.2), one
# decode stream per GPU with its own seed, every expert owned by one GPU's store (454 GB over the GPUs' HBM, so 4 or
# more GPUs); each GPU keeps its 8 most popular experts per layer resident (752 units, 28.4 GB) and 4 spare slots
# per layer for the misses (a top-8 layer misses several experts at once). The stores are written on the device from
# the model's byte generator (the model file is sparse: 454 GB is more than host RAM).
QWEN3 = dict(LAYERS=94, UNITS=128, PART=12582912, TOP_K=8, ZIPF=1.2, RESIDENTS=94 * 8, SPARE=4,
             METRIC="expert-miss stream GB/s (device-gated decode, Qwen3-235B-A22B-shaped MoE, peer tier)",
             WORKLOAD="qwen3-235b-a22b-peer", MODEL_FILE="tsb-bench-qwen3-peer.bin")
# BASELINE configs[3] (C4): 58 MoE layers x 256 routed experts of 3 x 14,680,064 B (7168 x 2048 fp8 e4m3 as random
# bytes), top-8 Zipf(0.9) routes whose layers repeat their predecessor's experts with probability 0.5 (the config's
# layer-to-layer correlation), exclusive tiers, 48 GB of VRAM per GPU for the gated slots (12 residents and 6 spare
# slots per layer with the banks: 46.7 GB), each layer's routed ids predicting the next layer's on the device
# (ss_dg_enqueue_predict from the export's own buffer). The 654 GB of experts live in the peer tier's stores (82 GB
# per GPU at 8 GPUs; fewer GPUs take fewer layers with --layers), written on the device from the generator.
DEEPSEEK = dict(LAYERS=58, UNITS=256, PART=14680064, TOP_K=8, ZIPF=0.9, RHO=0.5, RESIDENTS=58 * 12, SPARE=6,
                METRIC="expert-miss stream GB/s (device-gated decode, DeepSeek-V3-shaped MoE, peer tier)",
                WORKLOAD="deepseek-v3-peer", MODEL_FILE="tsb-bench-deepseek-peer.bin")
DEVICE_FILLED = ("qwen3-235b-a22b-peer", "deepseek-v3-peer")  # sparse model files, stores written from the generator


def args_():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None, help="timed steps (default: 64; c1-host 64, llama3-70b-host 12)")
    p.add_argument("--warmup", type=int, default=None, help="warm-up steps (default: 8; llama3-70b-host 3)")
    p.add_argument("--impl", default="tierstream", choices=["tierstream", "reference", "reference-cuda"],
                   help="reference: the reference's CPU DgCore (the reference arm); reference-cuda (context only): the "
                        "reference library built with its own CUDA backend, decoding on this GPU")
    p.add_argument("--copy-mode", default=os.environ.get("TSB_COPY_MODE", "auto"), choices=["auto", "kernel", "ce"])
    p.add_argument("--wb-defer", type=int, default=0,
                   help="ss_options.dg_wb_defer: 0 (here) enqueues a boundary's write-backs on the write-back stream "
                        "at once, where one of B200's copy engines overlaps them with the demand copies; the "
                        "reference's default 1 defers them part by part (tuned for a single copy engine)")
    p.add_argument("--inclusive", type=int, default=-1,
                   help="ss_options.dg_inclusive_blocks: device units keeping their pinned block as a clean copy "
                        "(an eviction is then a drop, no write-back); -1 = every pinned unit")
    p.add_argument("--wb-stream", type=int, default=1, help="ss_options.dg_wb_stream (the reference default 1)")
    p.add_argument("--spare", type=int, default=0,
                   help="spare slots per layer (dynamic_slots_per_layer); 0 = the workload's (1 Mixtral, 4 Qwen3)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--tier", default="auto", choices=["auto", "pinned", "peer", "file"],
                   help="where non-resident experts live: pinned RAM, or the peer tier (every expert owned by one "
                        "rank's HBM store, owners planned from the ranks' summed routing counts by one all-reduce; a "
                        "miss is copied from its owner's store, NVLink for a peer, HBM for the rank's own), or the "
                        "file tier (one GPU: in the model file only, read on a miss through a pinned staging buffer); "
                        "auto = pinned at one GPU, peer at several")
    p.add_argument("--pinned-per-layer", type=int, default=0,
                   help="file tier: non-resident experts per layer that keep a pinned block (the rest in the file)")
    p.add_argument("--staging", type=int, default=4, help="file tier: staging buffers (ss_options.dg_disk_staging)")
    p.add_argument("--disk-queue", type=int, default=0,
                   help="file tier: file reads in flight (ss_options.dg_disk_queue; 0 / 1 = each inside its fetch)")
    p.add_argument("--policy", default="lru", choices=["lru", "scored", "scored_auto"],
                   help="device-gated eviction policy (ss_options.policy)")
    p.add_argument("--round-every", type=int, default=0,
                   help="a placement round (ss_dg_round, defaults) after every N tokens, inside the timed steps")
    p.add_argument("--workload", default="mixtral-8x7b-dg",
                   choices=["mixtral-8x7b-dg", "qwen3-235b-a22b-peer", "deepseek-v3-peer", "c1-host",
                            "llama3-70b-host"],
                   help="mixtral-8x7b-dg: BASELINE configs[1] (default); qwen3-235b-a22b-peer: configs[4], the peer "
                        "tier on 4 or more GPUs; deepseek-v3-peer: configs[3], the peer tier on 8 GPUs (fewer with "
                        "--layers); c1-host and llama3-70b-host: configs[0] and [2] in the host forward "
                        "mode on one GPU (tierstream_b200/host_bench.py)")
    p.add_argument("--ref-threads", type=int, default=0,
                   help="host workloads, --impl reference: the reference's reader_threads, pinned to that many CPUs "
                        "(0: every CPU this process may use, at most 64)")
    p.add_argument("--layers", type=int, default=0,
                   help="qwen3 / deepseek only: fewer layers than the config's, for fewer GPUs (the "
                        "line then names the layer count; not the config's number)")
    p.add_argument("--peer-layout", default="auto", choices=["auto", "whole", "striped"],
                   help="peer tier stores: whole units at their owners, every unit striped over all GPUs (a miss "
                        "reads a stripe from each), or auto (the default): striped for the Mixtral shape (3,537 "
                        "against 2,950 GB/s for whole units at 8 GPUs, 1,959 against 1,723 at 4, 1,222 against 1,156 "
                        "at 2), whole units for the top-8 shapes (measured that way)")
    p.add_argument("--peer-copy", default="auto", choices=["auto", "kernel", "ce"],
                   help="peer tier mover: the copy engines, the land kernel's SM loads, or auto (the default): the "
                        "land kernel for striped stores (it pulls every stripe at once; one copy-engine stream takes "
                        "them in turn: 1,611 GB/s at 4 GPUs); for whole units the copy engines for the Mixtral shape "
                        "(one or two misses a layer: 2,950 against 2,751 GB/s at 8 GPUs) and the land kernel for the "
                        "top-8 shapes (several owners' units a layer pulled at once: 2,161 against 1,886 GB/s for "
                        "DeepSeek at 4 GPUs)")
    return p.parse_args()


def resident_keys(seed):
    from tierstream_b200 import synth
    pop = synth.popularity_order(LAYERS, UNITS, s=ZIPF, seed=seed)
    per = [RESIDENTS // LAYERS + (1 if g < RESIDENTS % LAYERS else 0) for g in range(LAYERS)]
    return [g * UNITS + e for g in range(LAYERS) for e in pop[g][:per[g]]]


def model_path():
    from tierstream_b200 import harness
    return os.path.join(harness.model_dir(), MODEL_FILE)


def configure(a):
    """Sets the workload's shape (the module constants) and resolves --peer-layout and --peer-copy auto."""
    mixtral = a.workload == "mixtral-8x7b-dg"
    if a.peer_layout == "auto":
        a.peer_layout = "striped" if mixtral else "whole"
    if a.peer_copy == "auto":
        a.peer_copy = "ce" if mixtral and a.peer_layout == "whole" else "kernel"
    shapes = {"qwen3-235b-a22b-peer": (QWEN3, 8), "deepseek-v3-peer": (DEEPSEEK, 12)}
    if a.workload in shapes:
        shape, per_layer = shapes[a.workload]
        g = globals()
        g.update(shape)
        if a.layers:
            g["LAYERS"] = a.layers
            g["RESIDENTS"] = a.layers * per_layer
            g["MODEL_FILE"] = shape["MODEL_FILE"].replace(".bin", "-%d.bin" % a.layers)
        if a.tier == "file":  # every byte written (never the peer tier's sparse file of the same shape)
            g["MODEL_FILE"] = g["MODEL_FILE"].replace(".bin", "-file.bin")


class Clocks:
    """SM clock and clock-event reasons sampled during the timed region: NVML read every 10 ms from a thread (read-only
    queries; the device found by its UUID, so CUDA_VISIBLE_DEVICES cannot shift it), else nvidia-smi every 200 ms."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, index):
        self.index = index
        self.sm, self.mx, self.reasons, self.failed = [], None, set(), False
        self.p = self.f = self.t = None
        try:
            import threading
            import pynvml
            import torch
            pynvml.nvmlInit()
            try:  # this process's CUDA device `index`, by its UUID
                h = pynvml.nvmlDeviceGetHandleByUUID("GPU-" + str(torch.cuda.get_device_properties(index).uuid))
            except Exception:
                vis = os.environ.get("CUDA_VISIBLE_DEVICES")
                h = pynvml.nvmlDeviceGetHandleByIndex(int(vis.split(",")[index]) if vis else index)
            self.mx = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            self.stop_ev = threading.Event()

            def run():
                while not self.stop_ev.is_set():
                    try:
                        self.sm.append(float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)))
                        bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        for n, b in self.BITS.items():
                            if bits & b:
                                self.reasons.add(n)
                    except Exception:  # a query NVML refuses: the samples taken so far stand
                        self.failed = True
                    self.stop_ev.wait(0.01)

            self.t = threading.Thread(target=run, daemon=True)
            self.t.start()
            return
        except Exception:
            self.t = None
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", "--query-gpu=" + self.Q, "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.t is not None:
            self.stop_ev.set()
            self.t.join(5)
            return {"sm_mhz": statistics.median(self.sm) if self.sm else None, "sm_max_mhz": self.mx,
                    "reasons": sorted(self.reasons), "samples": len(self.sm), "source": "nvml, 10 ms"}
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(5)
            except subprocess.TimeoutExpired:
                self.p.kill()
        self.f.seek(0)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            c = [x.strip() for x in line.split(",")]
            if len(c) < 9 or c[0] != str(self.index):
                continue
            try:
                sm.append(float(c[1]))
                mx = float(c[2])
            except ValueError:
                continue
            for n, v in zip(names, c[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi, 200 ms"}


def h2d_peak(torch):
    """Best-of-5 copy-engine pinned -> HBM bandwidth of 1 GiB (the host-link denominator; MEASURED_PEAKS.json has no
    host-link figure)."""
    n = 1 << 30
    h = torch.empty(n, dtype=torch.uint8).pin_memory()
    d = torch.empty(n, dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = None
    with torch.cuda.stream(s):
        for i in range(6):
            a.record(s)
            d.copy_(h, non_blocking=True)
            b.record(s)
            b.synchronize()
            if i:
                ms = a.elapsed_time(b)
                best = ms if best is None else min(best, ms)
    del h, d
    return n / (best / 1e3) / 1e9


def miss_layer_path(ctx, layers):
    """Where a missing layer's time goes, over the last timed token's layers that missed (means, microseconds):
    export written -> seen by the service, the service's serve, the demand copies on the device, the wait kernel's
    wait; and the layers counted."""
    rows = [ctx.timeline(g) for g in range(layers)]
    rows = [r for r in rows if r["misses"] > 0 and r["dma_ms"] >= 0]
    if not rows:
        return None

    def mean(k, scale=1.0):
        v = [r[k] * scale for r in rows if r[k] >= 0]
        return round(sum(v) / len(v), 2) if v else None

    return {"layers_with_misses": len(rows), "misses_per_layer": mean("misses"), "seen_us": mean("seen_us"),
            "serve_us": mean("serve_us"), "copies_us": mean("dma_ms", 1000.0), "gpu_wait_us": mean("gpu_wait_us"),
            "export_to_ready_us": mean("gpu_export_ready_us")}


def hbm_copy_peak():
    """The measured HBM copy rate (GB/s copied; MEASURED_PEAKS.json counts read + write), else the pool's fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]) / 2
    except (OSError, KeyError, ValueError):
        return 6650.0 / 2


def inclusive_of(a):
    if a.tier == "file":
        return 0 if a.inclusive < 0 else a.inclusive
    return LAYERS * UNITS - RESIDENTS if a.inclusive < 0 else a.inclusive


def disk_keys(a, residents):
    """File tier: per layer every non-resident expert except the first --pinned-per-layer by popularity."""
    from tierstream_b200 import synth
    pop = synth.popularity_order(LAYERS, UNITS, s=ZIPF, seed=1)
    res = set(residents)
    out = []
    for g in range(LAYERS):
        rest = [g * UNITS + e for e in pop[g] if g * UNITS + e not in res]
        out += rest[a.pinned_per_layer:]
    return out


def host_hash_rate(unit, reps=3):
    """GB/s of the library's host xxh64 over one unit-sized buffer on one thread (best of reps)."""
    from tierstream_b200 import abi
    buf = np.random.default_rng(0).integers(0, 256, size=unit, dtype=np.uint8)
    best = None
    for _ in range(reps):
        t0 = time.perf_counter()
        abi.load().tsb_xxh64(buf.ctypes.data, buf.size, 0)
        dt = time.perf_counter() - t0
        best = dt if best is None else min(best, dt)
    return unit / best / 1e9


def file_read_peak(path, unit, units=20, threads=8):
    """The sequential read rate of the model file (GB/s) as the file tier reads it: whole units one after another,
    each in 8 MiB pieces by a pool of `threads` readers, O_DIRECT (the library's own reads, tsb_test_file_read)."""
    import mmap
    from tierstream_b200 import abi
    buf = mmap.mmap(-1, unit)
    dst = C.addressof(C.c_char.from_buffer(buf))
    lib = abi.load()
    units = min(units, os.path.getsize(path) // unit)
    t0 = time.perf_counter()
    for i in range(units):
        abi.check(lib.tsb_test_file_read(path.encode(), i * unit, unit, dst, 8 << 20, threads, 1))
    dt = time.perf_counter() - t0
    return units * unit / dt / 1e9 if units and dt > 0 else None


def reference_sample(ids, tokens, a):
    """The reference DgCore + memcpy transport on `tokens` tokens of the trace (oracle/_ref): (miss bytes, seconds)."""
    import oracle
    from tierstream_b200 import runtime
    keys = resident_keys(1)
    P = LAYERS * UNITS - len(keys)
    inc = inclusive_of(a)
    cfg = runtime.replay_config([UNITS] * LAYERS, [PART] * 3, persistent_slots=len(keys) + a.spare * LAYERS,
                                bank_slots=TOP_K, blocks=P + a.spare * LAYERS + inc, spare_target=a.spare * LAYERS,
                                order=keys, tokens=tokens, n_ids=TOP_K, move_bytes=2, wb_defer=a.wb_defer,
                                wb_on_d2h=a.wb_stream, inclusive=inc)
    t0 = time.perf_counter()
    _, stats = oracle.ref_replay(cfg, ids[:tokens])
    dt = time.perf_counter() - t0
    moved = int(stats[-1][4] + stats[-1][5]) * 3 * PART  # fetched + prefetched units
    return moved, dt


def host_l3_bytes():
    """The host's last-level cache per socket (bytes), from sysfs; None when not found."""
    try:
        with open("/sys/devices/system/cpu/cpu0/cache/index3/size") as f:
            v = f.read().strip()
        mult = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}.get(v[-1:].upper(), 1)
        return int(v.rstrip("KMGkmg")) * mult
    except (OSError, ValueError):
        return None


def reference_measure(ids, a):
    """The reference arm's measurement (also the in-line cpu_baseline): the reference DgCore with the memcpy transport
    over warmup + steps tokens of the trace, less a run of the warm-up tokens alone (the replay cannot split them):
    (GB/s, seconds of the timed tokens)."""
    moved, dt = reference_sample(ids, a.warmup + a.steps, a)
    w_moved, w_dt = reference_sample(ids, a.warmup, a) if a.warmup else (0, 0.0)
    moved, dt = moved - w_moved, max(dt - w_dt, 1e-9)
    return moved / dt / 1e9, dt


def reference_sample_text(a, dt):
    import oracle
    l3 = host_l3_bytes()
    return ("%d tokens of the trace (after %d warm-up tokens, subtracted) through the reference DgCore (oracle/_ref) "
            "with a host memcpy transport on %d host threads, %.1f s; every copy moves its real bytes, slots and blocks "
            "alias 16 unit buffers each (%.1f GB, host L3 %s)" % (
                a.steps, a.warmup, int(oracle.ref().oref_copy_threads()), dt, 32 * 3 * PART / 1e9,
                "%.0f MB" % (l3 / 1e6) if l3 else "unknown"))


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from tierstream_b200 import synth
    ids = synth.zipf_trace(a.warmup + a.steps, LAYERS, UNITS, TOP_K, s=ZIPF, seed=1)
    import oracle
    if not oracle.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libtsref.so (the reference's sources "
                                                              "compiled by oracle/Makefile) is not built"}))
        return 0
    v, dt = reference_measure(ids, a)
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "GB/s", "n_gpus": a.gpus,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(dt * 1e3 / a.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
            "config": {"workload": WORKLOAD, "layers": LAYERS, "experts": UNITS, "part_bytes": PART,
                       "top_k": TOP_K, "zipf": ZIPF, "residents": RESIDENTS, "tokens": a.steps},
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": int(oracle.ref().oref_copy_threads()),
                             "kind": "reference", "sample": reference_sample_text(a, dt)},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


HOST_WORKLOADS = ("c1-host", "llama3-70b-host")


def host_reference_case(name):
    """The reference's host-mode case for a host workload: (desc JSON, tiers, budget, options, unit bytes, sample text).
    C1 runs whole; C3 is sampled on 8 layers of the same 1.71 GB blobs (3 resident, 5 streamed through the 2-slot
    ring): the reference's CPU backend keeps its "device" copies in host RAM too, and all 80 layers would not fit."""
    from tierstream_b200 import abi, harness, host_bench, synth
    w = host_bench.WORKLOADS[name]
    if name == "c1-host":
        m = host_bench.model_of(name)
        m.write()
        tiers = host_bench.tiers_of(name)
        what = "C1 whole"
    else:
        m = synth.Model(os.path.join(harness.model_dir(), "tsb-bench-llama3-ref-sample.bin"), 8, 1, w["parts"],
                        seed=w["seed"], top_k=1)
        m.create_sparse()
        tiers = [abi.SS_TIER_RESIDENT] * 3 + [abi.SS_TIER_PINNED] * 5
        what = "8 layers of C3's 1.71 GB blobs (3 resident, 5 streamed per token through the 2-slot ring)"
    b, o = host_bench.budget_options(name, m)
    if name != "c1-host":
        b.device_bytes = (3 + w["ring"] + 4) * m.unit_bytes + (1 << 30)
    return host_bench.desc_of(name, m), tiers, b, o, m.unit_bytes, what


def host_reference_measure(name, trace, warmup, steps, threads):
    """The reference's host forward mode on its CPU backend (oracle/_ref, synchronous memcpy copies on its reader
    threads) over warmup + steps forwards of the trace, less a run of the warm-up forwards alone: (GB/s streamed,
    seconds of the timed forwards, sample text)."""
    import oracle
    desc_json, tiers, b, o, unit, what = host_reference_case(name)
    o.reader_threads = threads
    layers = json.loads(desc_json)["layers"]
    all_layers = [1 if lay["kind"] == "blob" else 0 for lay in layers]
    tr = trace[:, :len(layers)]

    def timed(n):
        t0 = time.perf_counter()
        _, st = oracle.ref_host_replay(desc_json, tiers, b, o, tr[:n], all_layers)
        return float(st[:, :, 2].sum() + st[:, :, 3].sum()) * unit, time.perf_counter() - t0

    moved, dt = timed(warmup + steps)
    w_moved, w_dt = timed(warmup) if warmup else (0.0, 0.0)
    moved, dt = moved - w_moved, max(dt - w_dt, 1e-9)
    text = ("%s: %d forwards (after %d warm-up forwards, subtracted) through the reference's host forward mode on its CPU "
            "backend (oracle/_ref: ss_open / ss_layer_routes or ss_layer_all / ss_acquire / ss_release / ss_end, "
            "every copy a memcpy of the real bytes), reader_threads %d, %.1f s" % (what, steps, warmup, threads, dt))
    return moved / dt / 1e9, dt, text


def host_reference(a):
    """--impl reference for a host workload: the reference CPU backend with every usable CPU (reader_threads up to 64)
    and, in a child process pinned to one CPU, with one."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    import oracle
    from tierstream_b200 import host_bench
    if not oracle.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libtsref.so (the reference's sources "
                                                              "compiled by oracle/Makefile) is not built"}))
        return 0
    cpus = sorted(os.sched_getaffinity(0))
    threads = a.ref_threads or min(64, len(cpus))
    if a.ref_threads:
        os.sched_setaffinity(0, set(cpus[:a.ref_threads]))
    w = host_bench.WORKLOADS[a.workload]
    trace = host_bench.routes_of(a.workload, a.warmup + a.steps)
    v, dt, text = host_reference_measure(a.workload, trace, a.warmup, a.steps, threads)
    line = {"impl": "reference", "metric": w["metric"], "value": round(v, 3), "unit": "GB/s", "n_gpus": a.gpus,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(dt * 1e3 / a.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
            "config": {"workload": a.workload, "layers": w["layers"], "units_per_layer": w["units"],
                       "parts": list(w["parts"]), "resident": w["resident"], "ring_slots": w["ring"]},
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
                             "sample": text},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if not a.ref_threads:  # the same with one CPU, in a child pinned to it
        r = subprocess.run([sys.executable, os.path.abspath(__file__), "--impl", "reference", "--workload",
                            a.workload, "--steps", str(a.steps), "--warmup", str(a.warmup), "--ref-threads", "1"],
                           capture_output=True, text=True)
        one = [json.loads(x) for x in r.stdout.splitlines() if x.startswith("{")]
        line["one_core"] = {"value": one[0]["value"], "sample": one[0]["cpu_baseline"]["sample"]} if one and \
            "value" in one[0] else {"error": (r.stderr or r.stdout)[-300:]}
    print(json.dumps(line))
    return 0


def host_main(a):
    """A host workload's GPU leg (tierstream_b200/host_bench.py) with the roofline against this run's host-link copy
    rate and, after the context closed, the reference's CPU backend on the same trace as the cpu_baseline."""
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        raise SystemExit("the host-mode workloads run on one GPU")
    import torch
    from tierstream_b200 import host_bench
    torch.cuda.set_device(0)
    peak = h2d_peak(torch)
    line, trace, bad = host_bench.run(a.workload, a.steps, a.warmup, torch, Clocks, 0)
    line["roofline"] = {
        "bound": "link", "kernel": "the forward's stream (pinned -> ring and slot copies, the readers behind them)",
        "achieved": line["value"], "peak": round(peak, 3) if peak else None, "unit": "GB/s",
        "frac": round(line["value"] / peak, 4) if peak else None, "traffic": None,
        "peak_source": "measured in this run: copy-engine pinned->HBM 1 GiB, best of 5 (MEASURED_PEAKS.json has no "
                       "host-link figure)",
        "note": "achieved over the whole forward (the copies are not timed apart from the routes, acquires and readers "
                "in host mode)"}
    if not a.no_cpu_baseline:
        cpus = sorted(os.sched_getaffinity(0))
        threads = min(64, len(cpus))
        v, _, text = host_reference_measure(a.workload, trace, a.warmup, a.steps, threads)
        line["cpu_baseline"] = {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
                                "sample": text}
    print(json.dumps(line))
    return 1 if bad else 0


def reference_cuda_dir(model, setup, ids, want, n_ids):
    """A directory of the files oracle/_ref/ref_dg_cuda opens: descriptor, tiers, budget and options (as bytes), the
    shape, the trace and (when given) every key's expected word-sum checksum."""
    d = tempfile.mkdtemp(prefix="tsb-refcu-")
    with open(os.path.join(d, "desc.json"), "w") as f:
        f.write(model.desc())
    np.asarray(setup.tiers, dtype=np.uint8).tofile(os.path.join(d, "tiers.u8"))
    with open(os.path.join(d, "budget.bin"), "wb") as f:
        f.write(bytes(setup.budget))
    with open(os.path.join(d, "options.bin"), "wb") as f:
        f.write(bytes(setup.options))
    with open(os.path.join(d, "meta.txt"), "w") as f:
        f.write("%d %d %d\n" % (model.layers, model.units, n_ids))
    np.ascontiguousarray(ids, dtype=np.int32).tofile(os.path.join(d, "ids.i32"))
    if want is not None:
        np.asarray(want, dtype=np.uint64).tofile(os.path.join(d, "want.u64"))
    return d


def run_reference_cuda(a):
    """--impl reference-cuda, for context only: the reference library's own GPU decode on this B200
    (oracle/_ref/ref_dg_cuda: its sources built with their CUDA backend for sm_100a, the ready word in mapped host
    memory as the reference keeps it) driven by the same engine stand-in graph, on the same model, trace, options and
    tokens as this library's line; its readers' checksums are compared with the generator's. Beside it, its
    zero-miss protocol cost measured as this library's is (the graph less the readers alone, per layer)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    exe = os.path.join(ROOT, "oracle", "_ref", "ref_dg_cuda")
    if not os.path.exists(exe):
        print(json.dumps({"impl": "reference-cuda", "unavailable": "oracle/_ref/ref_dg_cuda (the reference's sources "
                                                                   "built with their CUDA backend) is not built"}))
        return 0
    import shutil
    import torch
    from tierstream_b200 import harness, synth
    torch.cuda.set_device(0)
    model = synth.Model(model_path(), LAYERS, UNITS, [PART] * 3, seed=0, top_k=TOP_K, with_hash=True)
    model.write()
    model.hashes()
    setup = harness.DgSetup(model, resident_keys=resident_keys(1), spare_per_layer=a.spare, max_ids=TOP_K,
                            test_hooks=False, wb_defer=a.wb_defer, wb_stream=a.wb_stream, verify=True,
                            inclusive=inclusive_of(a))
    # the reference's open reads the residents through a ring of 4 pinned buffers of at least a unit each, which it
    # admits against the host budget on top of the pinned units (its dg_layout.cpp:425-443)
    setup.budget.host_pinned_bytes += 4 * model.unit_bytes + (256 << 20)
    ids = synth.zipf_trace(a.warmup + a.steps, LAYERS, UNITS, TOP_K, s=ZIPF, seed=1)
    want = harness.expected_sums(model, np.arange(LAYERS * UNITS), 1)
    d = reference_cuda_dir(model, setup, ids, want, TOP_K)
    try:
        r = subprocess.run([exe, "stream", d, str(a.warmup), str(a.steps), "512"], capture_output=True, text=True,
                           timeout=1200)
    finally:
        shutil.rmtree(d, ignore_errors=True)
    got = [json.loads(x) for x in r.stdout.splitlines() if x.startswith("{")]
    if r.returncode != 0 or not got or "value" not in got[-1]:
        print(json.dumps({"impl": "reference-cuda", "error": (got[-1] if got else None),
                          "stderr": r.stderr[-500:], "rc": r.returncode}))
        return 1
    line = got[-1]
    # the zero-miss protocol cost on the model tierstream_b200/dg_overhead.py uses (32 x 8 units, 7 resident per layer,
    # routes only to residents)
    zm = synth.Model(os.path.join(harness.model_dir(), "tsb-overhead-32.bin"), layers=32, units=8,
                     part_bytes=(256 << 10,) * 3, seed=9, top_k=2)
    zm.write()
    zs = harness.DgSetup(zm, residents_per_layer=7, spare_per_layer=1, max_ids=2, test_hooks=False)
    zs.budget.host_pinned_bytes += 4 * zm.unit_bytes + (256 << 20)
    d = reference_cuda_dir(zm, zs, np.tile(np.arange(2, dtype=np.int32), (32, 1))[None], None, 2)
    try:
        z = subprocess.run([exe, "zero", d, "100"], capture_output=True, text=True, timeout=600)
    finally:
        shutil.rmtree(d, ignore_errors=True)
    zero = [json.loads(x) for x in z.stdout.splitlines() if x.startswith("{")]
    out = {"impl": "reference-cuda", "metric": METRIC, "value": line["value"], "unit": "GB/s", "n_gpus": 1,
           "steps": a.steps, "warmup": a.warmup, "ms_per_step": line["ms_per_step"], "higher_is_better": True,
           "dtype": "u8", "data": "synthetic", "note": "context only: the reference library built with its own CUDA "
                                                      "backend for sm_100a, on this GPU",
           "config": {"workload": WORKLOAD, "layers": LAYERS, "experts": UNITS, "part_bytes": PART, "top_k": TOP_K,
                      "zipf": ZIPF, "residents": RESIDENTS, "spare_slots_per_layer": a.spare,
                      "wb_defer": a.wb_defer, "inclusive_blocks": inclusive_of(a)},
           "misses_per_token": round(line["misses"] / max(1, a.warmup + a.steps), 3),
           "verified": {"tokens": a.steps, "units": line["reads"], "mismatches": line["mismatches"]},
           "dg_zero_miss": zero[-1] if zero else {"error": z.stderr[-300:]}}
    if zero and "overhead_us_per_layer" in zero[-1]:
        out["dg_zero_miss_us_per_layer"] = zero[-1]["overhead_us_per_layer"]
    print(json.dumps(out))
    return 1 if line["mismatches"] else 0


def main():
    a = args_()
    if a.workload in HOST_WORKLOADS:
        from tierstream_b200 import host_bench
        w = host_bench.WORKLOADS[a.workload]
        a.steps = a.steps if a.steps is not None else w["steps"]
        a.warmup = a.warmup if a.warmup is not None else w["warmup"]
        return host_reference(a) if a.impl == "reference" else host_main(a)
    a.steps = a.steps if a.steps is not None else 64
    a.warmup = a.warmup if a.warmup is not None else 8
    configure(a)
    if not a.spare:
        a.spare = SPARE
    if a.impl == "reference":
        return run_reference(a)
    if a.impl == "reference-cuda":
        return run_reference_cuda(a)
    os.environ["TSB_COPY_MODE"] = a.copy_mode
    import torch
    from tierstream_b200 import abi, harness, synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    a.peer = a.tier == "peer" or (a.tier == "auto" and world > 1)
    a.file = a.tier == "file"
    if a.file and (world > 1 or a.workload == "qwen3-235b-a22b-peer"):
        raise SystemExit("--tier file runs the Mixtral- or DeepSeek-shaped workload (the latter with --layers) on one GPU")
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if dist:
            dist.barrier()

    # the peer tier's Qwen3 and DeepSeek shapes write their stores from the generator over a sparse model file; with
    # the file tier the model file holds every byte
    qwen = a.workload in DEVICE_FILLED and not a.file
    # descriptor hashes (the stores' and the landings' checks on the device) for every model written to disk; the
    # Qwen3-shaped stores are written on the device from the generator and checked by the readers' sums instead
    hashed = not qwen
    model = synth.Model(model_path(), LAYERS, UNITS, [PART] * 3, seed=0, top_k=TOP_K, with_hash=hashed)
    if qwen and not a.peer:
        raise SystemExit("%s runs the peer tier only (its experts do not fit pinned RAM)" % a.workload)
    if rank == 0:
        if qwen:
            model.create_sparse()
        else:
            model.write()
            model.hashes()  # kept beside the model file for the other ranks
    barrier()
    peak = h2d_peak(torch) if rank == 0 and not a.peer else None
    read_peak = file_read_peak(model_path(), 3 * PART) if a.file else None
    # one trace per rank: warm-up, the device-timed steps, then one untimed and `steps` timed steps of the e2e leg (a
    # second window of the same routing distribution)
    full = synth.zipf_trace(a.warmup + 2 * a.steps + 1, LAYERS, UNITS, TOP_K, s=ZIPF, seed=1 + rank, rho=RHO)
    ids = full[:a.warmup + a.steps]
    ids2_warm, ids2 = full[a.warmup + a.steps], full[a.warmup + a.steps + 1:]
    inclusive = 0 if a.peer else inclusive_of(a)
    t_open = time.perf_counter()
    setup = None
    if a.peer:
        from tierstream_b200 import peer as peer_mod, runtime
        # the planner's input: this rank's routing counts over a calibration window of its own trace distribution
        cal = synth.zipf_trace(64, LAYERS, UNITS, TOP_K, s=ZIPF, seed=1001 + rank, perm_seed=1 + rank, rho=RHO)
        counts = np.bincount((np.arange(LAYERS)[None, :, None] * UNITS + cal).reshape(-1), minlength=LAYERS * UNITS)
        filler = None
        striped = a.peer_layout == "striped"
        if qwen and striped:
            def filler(store, owner):
                # this rank's stripe of every owned unit written on the device from the model's byte generator, in
                # store order (unit i at base + i * stripe); the first checked against the host generator
                keys = np.nonzero(owner >= 0)[0]
                stripe = peer_mod.stripe_bytes(model.unit_bytes, world)
                lo, n = peer_mod.stripe_range(model.unit_bytes, world, rank)
                if not keys.size or not n:
                    return
                offs = np.array([model.unit_offset(int(k) // UNITS, int(k) % UNITS) + lo for k in keys],
                                dtype=np.uint64)
                s = torch.cuda.Stream()
                fill = abi.load_engine().tse_fill_units_device
                if n == stripe:
                    rc = fill(model.seed, offs.ctypes.data_as(C.POINTER(C.c_uint64)), keys.size, n, store.base,
                              s.cuda_stream)
                else:  # a shorter last stripe: one unit at a time at the store's stride
                    rc = 0
                    for i in range(keys.size):
                        rc = rc or fill(model.seed, offs[i:].ctypes.data_as(C.POINTER(C.c_uint64)), 1, n,
                                        store.base + i * stripe, s.cuda_stream)
                assert rc == 0, "device fill failed: %d" % rc
                s.synchronize()
                k0 = int(keys[0])
                want = model.unit_bytes_of(k0 // UNITS, k0 % UNITS)[lo:lo + n]
                assert np.array_equal(peer_mod.read_device(store.base, n), want), "store fill differs"
        elif qwen:
            def filler(store, owner):
                # every owned unit written on the device from the model's byte generator, in store order; the first
                # one checked against the host generator
                keys = np.nonzero(owner == rank)[0]
                offs = np.array([model.unit_offset(int(k) // UNITS, int(k) % UNITS) for k in keys], dtype=np.uint64)
                if not keys.size:
                    return
                s = torch.cuda.Stream()
                rc = abi.load_engine().tse_fill_units_device(model.seed, offs.ctypes.data_as(C.POINTER(C.c_uint64)),
                                                             keys.size, model.unit_bytes, store.base, s.cuda_stream)
                assert rc == 0, "device fill failed: %d" % rc
                s.synchronize()
                first = peer_mod.read_device(store.base, model.unit_bytes)
                k0 = int(keys[0])
                assert np.array_equal(first, model.unit_bytes_of(k0 // UNITS, k0 % UNITS)), "store fill differs"
        setup = peer_mod.PeerSetup(runtime.Desc(model.desc()), counts, dist, world, rank, local, verify=hashed,
                                   copy=1 if a.peer_copy == "ce" else 0,
                                   collective_device=torch.device("cuda", local) if dist else None, filler=filler,
                                   layout=abi.PEER_STRIPED if striped else abi.PEER_WHOLE_UNITS)
    # verify_hash with descriptor hashes: residents checked at the open, and every unit landed in a slot while decoding
    # hashed on the device against its descriptor hash (the landing check)
    run = harness.DgRun(model, resident_keys=resident_keys(1 + rank), spare_per_layer=a.spare, max_ids=TOP_K,
                        diag=True, test_hooks=False, mode=1, slices=512, wb_defer=a.wb_defer, wb_stream=a.wb_stream,
                        verify=hashed,
                        inclusive=inclusive, peer=setup.tier if setup else None,
                        disk_keys=disk_keys(a, resident_keys(1)) if a.file else (), disk_staging=a.staging,
                        disk_prefetch=1 if a.file and RHO > 0 else 0,
                        disk_queue=a.disk_queue, policy={"lru": 0, "scored": 1, "scored_auto": 2}[a.policy],
                        predict_prev=RHO > 0)
    t_open = time.perf_counter() - t_open
    unit = model.unit_bytes
    # the e2e leg's trace, and every routed unit's expected reader sums in both legs' modes, from the byte generator
    # on the device (outside the timed regions)
    routed = np.unique(np.concatenate([(np.arange(LAYERS)[None, :, None] * UNITS + x).reshape(-1)
                                       for x in (ids[a.warmup:], ids2)]))
    t_exp = time.perf_counter()
    want = {mode: np.zeros(LAYERS * UNITS, dtype=np.uint64) for mode in (0, 1)}
    for mode in (0, 1):
        want[mode][routed] = harness.expected_sums(model, routed, mode)
    t_exp = time.perf_counter() - t_exp
    try:
        for t in range(a.warmup):
            run.step(ids[t])
        run.graph_for(0)  # the e2e leg's graph (positional checksums), captured before any timed region
        # (1) device-timed: ids already in HBM (the whole trace resident), one D2D copy per step into the graph's
        # input buffer, no host copy; each step's reader sums kept on the device for the check after the region
        trace_dev = torch.from_numpy(ids[a.warmup:].reshape(a.steps, -1).copy()).cuda()
        outs_dev = torch.zeros((a.steps, LAYERS * TOP_K), dtype=torch.int64, device="cuda")
        run.stream.wait_stream(torch.cuda.current_stream())
        s0 = run.ctx.stats()
        f0 = json.loads(run.ctx.stats_json())
        j0 = f0["dg"]
        clocks = Clocks(local)
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(run.stream)
        for t in range(a.steps):
            run.ctx.begin()
            with torch.cuda.stream(run.stream):
                run.ids_dev.copy_(trace_dev[t], non_blocking=True)
                run.graph.launch()
                outs_dev[t].copy_(run.out_dev, non_blocking=True)
            run.ctx.end()
            if a.round_every and (t + 1) % a.round_every == 0:
                run.ctx.round()
        e1.record(run.stream)
        e1.synchronize()
        barrier()
        clk = clocks.stop()
        dev_ms = e0.elapsed_time(e1)
        s1 = run.ctx.stats()
        f1 = json.loads(run.ctx.stats_json())
        j1 = f1["dg"]
        layer_path = miss_layer_path(run.ctx, LAYERS)
        c0, c1 = f0["check"], f1["check"]
        check = {"on": bool(c1["on"]), "units_per_token": round((c1["units"] - c0["units"]) / a.steps, 3),
                 "gb_per_token": round((c1["bytes"] - c0["bytes"]) / a.steps / 1e9, 3),
                 "launches_per_token": round((c1["launches"] - c0["launches"]) / a.steps, 3),
                 "merged_per_token": round((c1["merged"] - c0["merged"]) / a.steps, 3),
                 "hold_waits": c1["hold_waits"] - c0["hold_waits"], "mismatches": c1["mismatches"] - c0["mismatches"],
                 "end_wait_ms_per_token": round((c1["end_wait_s"] - c0["end_wait_s"]) * 1e3 / a.steps, 3)}
        peer_units = f1["peer"]["peer_units"] - f0["peer"]["peer_units"]
        self_units = f1["peer"]["self_units"] - f0["peer"]["self_units"]
        peer_bytes = f1["peer"]["peer_bytes"] - f0["peer"]["peer_bytes"]
        self_bytes = f1["peer"]["self_bytes"] - f0["peer"]["self_bytes"]
        units_moved = (s1["fetched"] - s0["fetched"]) + (s1["prefetched"] - s0["prefetched"])
        moved = units_moved * unit
        dma_ms = j1["dma_ms_total"] - j0["dma_ms_total"]
        land_launches = j1["land_launches"] - j0["land_launches"]
        # (2) end to end: the same steps of a second trace window through the ABI with host buffers, the readers
        # computing the positional checksum (the reference GPU tests' check)
        # one untimed step through the e2e path first (its graph's first launch, host buffers), on a token of its own
        run.step(ids2_warm, mode=0)
        s2 = run.ctx.stats()
        outs2 = np.zeros((a.steps, LAYERS, TOP_K), dtype=np.uint64)
        step_ms = []
        import gc
        gc.collect()  # the interpreter's collector off while the host drives the timed tokens (on again after)
        gc.disable()
        try:
            barrier()
            w0 = time.perf_counter()
            for t in range(a.steps):
                ws = time.perf_counter()
                outs2[t] = run.step(ids2[t], mode=0)
                if a.round_every and (t + 1) % a.round_every == 0:
                    run.ctx.round()
                step_ms.append((time.perf_counter() - ws) * 1e3)
            w1 = time.perf_counter()
            barrier()
        finally:
            gc.enable()
        # every routed unit of both legs as its reader saw it, against the generator's sums
        n1, bad1, first1 = harness.check_reads(outs_dev.cpu().numpy().view(np.uint64).reshape(a.steps, LAYERS, TOP_K),
                                               ids[a.warmup:], UNITS, want[1])
        n0, bad0, first0 = harness.check_reads(outs2, ids2, UNITS, want[0])
        s3 = run.ctx.stats()
        moved_e2e = ((s3["fetched"] - s2["fetched"]) + (s3["prefetched"] - s2["prefetched"])) * unit
        e2e_s = w1 - w0
        misses = s1["misses"] - s0["misses"]
        lookups = s1["lookups"] - s0["lookups"]
        dg = {k: s1[k] - s0[k] for k in ("fetched", "prefetched", "prefetch_used", "predicted", "predicted_true",
                                         "bank_serves", "evicted", "evict_short",
                                         "writebacks_done", "collected_mid", "wb_forced", "wb_forced_wait_ns",
                                         "wb_boundary_flushed", "wb_deferred", "wb_cancelled", "resurrected",
                                         "wb_issued_bytes", "covered", "disk_reads", "disk_read_bytes",
                                         "disk_read_ns", "disk_drops", "disk_discards", "disk_overlapped",
                                         "disk_carried", "scored_victims", "score_fallbacks", "round_count",
                                         "round_units", "round_bytes")}
        full = json.loads(run.ctx.stats_json())
        peer_stats, open_stats = full["peer"], full["open"]
    finally:
        run.close()
        if setup:  # every rank's context is closed before any store is unmapped or freed
            barrier()
            setup.close()

    # the device-gated protocol's cost per layer when nothing misses (a small all-resident model, dg_overhead)
    from tierstream_b200 import dg_overhead
    zero_miss = dg_overhead.measure(layers=LAYERS, tokens=100, warmup=10) if rank == 0 else None
    tot = torch.tensor([moved, moved_e2e, dev_ms, e2e_s, dma_ms], dtype=torch.float64, device="cuda")
    ver = torch.tensor([2 * a.steps, n1 + n0, bad1 + bad0], dtype=torch.int64, device="cuda")
    if dist:
        s = tot[[0, 1]].clone()
        m = tot[[2, 3, 4]].clone()
        dist.all_reduce(s, op=dist.ReduceOp.SUM)
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        dist.all_reduce(ver, op=dist.ReduceOp.SUM)
        tot = torch.cat([s, m])
    moved_all, moved_e2e_all, dev_ms_max, e2e_s_max, dma_ms_max = [float(x) for x in tot.cpu()]
    v_tokens, v_units, v_bad = [int(x) for x in ver.cpu()]
    if bad1 or bad0:
        print("rank %d: %d of %d reads differ from the generator (first: timed leg %s, e2e leg %s)" %
              (rank, bad1 + bad0, n1 + n0, first1, first0), file=sys.stderr)
    if rank != 0:
        if dist:
            dist.destroy_process_group()
        return 0
    value = moved_all / (dev_ms_max / 1e3) / 1e9
    e2e = moved_e2e_all / e2e_s_max / 1e9
    achieved = (moved / (dma_ms / 1e3) / 1e9) if dma_ms > 0 else None
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(dev_ms_max / a.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic (seeded random bytes and Zipf routes)",
        "config": {"workload": WORKLOAD, "layers": LAYERS, "experts": UNITS, "part_bytes": PART,
                   "unit_bytes": unit, "top_k": TOP_K, "zipf": ZIPF, "rho": RHO, "residents": RESIDENTS,
                   "predictions": "each layer's routed ids, for the next layer" if RHO > 0 else "none",
                   "spare_slots_per_layer": a.spare, "parallelism": "replicas" if world > 1 else "single",
                   "copy_mode": a.copy_mode,
                   "l2": "inputs larger than L2 (%.0f MB units, %.1f GB arena)" % (
                       unit / 1e6, (RESIDENTS + a.spare * LAYERS + 2 * TOP_K + 1) * unit / 1e9)},
        "tokens_per_s": round(a.steps * world / (dev_ms_max / 1e3), 3),
        "misses_per_token": round(misses / a.steps, 3), "lookups_per_token": round(lookups / a.steps, 3),
        "e2e": {"value": round(e2e, 3), "unit": "GB/s", "h2d_bytes_per_step": LAYERS * TOP_K * 4,
                "d2h_bytes_per_step": LAYERS * TOP_K * 8,
                "tokens_per_s": round(a.steps * world / e2e_s_max, 3),
                "step_ms": {"median": round(statistics.median(step_ms), 3), "min": round(min(step_ms), 3),
                            "max": round(max(step_ms), 3)}},
        "roofline": {"bound": "link", "kernel": "miss service (demand copies + entries + ready on the demand stream)",
                     "achieved": round(achieved, 3) if achieved else None, "peak": round(peak, 3) if peak else None,
                     "unit": "GB/s", "frac": round(achieved / peak, 4) if achieved and peak else None, "traffic": None,
                     "peak_source": "measured in this run: copy-engine pinned->HBM 1 GiB, best of 5 "
                                    "(MEASURED_PEAKS.json has no host-link figure)",
                     "algorithmic_bytes": moved, "device_ms": round(dma_ms, 3),
                     "traffic_note": "the demand copies of 33 MB parts run on the copy engines (peer-tier pulls on "
                                     "the land kernel), whose DRAM bytes ncu does not attribute to one kernel; ncu "
                                     "captures of the land kernel alone show DRAM traffic at or below its algorithmic "
                                     "bytes"},
        "verified": {"tokens": v_tokens, "units": v_units, "mismatches": v_bad, "ranks": world,
                     "how": "every routed unit of every timed token (both legs, every rank) as the engine's reader "
                            "read it through the slot table: word sums in the device-timed leg, positional checksums "
                            "sum(byte x (pos %% 251 + 1)) in the e2e leg, against sums computed on the device from the "
                            "byte generator alone (%.2f s, outside the timed regions)" % t_exp,
                     "stores_checked": bool(a.peer and hashed)},
        "gpu_launches": int(a.steps * (2 + 2 * LAYERS) + land_launches + a.steps * LAYERS +
                            (c1["launches"] - c0["launches"])),
        "dg_zero_miss_us_per_layer": zero_miss["overhead_us_per_layer"],
        "dg_zero_miss": dict(zero_miss, how="rank 0: a %d-layer all-resident model (no token misses), the captured "
                                            "token graph (begin, per layer export -> wait -> reader, end) less the "
                                            "same readers captured alone, per layer; CUDA events, 100 tokens after 10 "
                                            "warm-up" % LAYERS),
        "landing_check": dict(check, how="every unit copied into a slot from host memory (pinned blocks, file "
                                          "staging) hashed on the device (K3, xxh64) against its descriptor hash on a "
                                          "low-priority stream behind the layer's ready word (a copy from a peer store "
                                          "is not: each store was hashed on the device when it was filled); "
                                          "a copy into a slot still being hashed waits for it (hold_waits); each "
                                          "ss_end waits for the previous token's hashes (end_wait)"),
        "clocks": clk, "open_s": round(t_open, 2), "open": open_stats, "dg": dg, "miss_layer_path": layer_path,
        "options": {"wb_defer": a.wb_defer, "wb_stream": a.wb_stream, "spare_slots_per_layer": a.spare,
                    "inclusive_blocks": inclusive, "policy": a.policy, "round_every": a.round_every,
                    "disk_queue": a.disk_queue},
    }
    if a.peer:
        # every expert lives in one rank's store (striped: a stripe of it in every rank's store): a miss is an NVLink
        # pull from a peer or an HBM copy from the rank's own store (striped: both); no pinned RAM is allocated
        line["config"].update({"workload": WORKLOAD if qwen else "mixtral-8x7b-dg-peer",
                               "parallelism": "peer tier x%d" % world,
                               "peer_copy": a.peer_copy, "peer_layout": a.peer_layout})
        line["peer"] = dict(peer_stats, timed_peer_units=peer_units, timed_self_units=self_units,
                            timed_peer_bytes=peer_bytes, timed_self_bytes=self_bytes,
                            checked_units=setup.checked_units)
        # whole units: a missing unit comes from one store, a peer's over NVLink or the rank's own inside HBM, and the
        # peak is the rate of an ideal mover doing both kinds in turn, each at its measured rate; striped: every unit's
        # stripes are pulled together, so the ideal mover overlaps them and is bound by the slower of the two
        hbm_copy = hbm_copy_peak()
        parts_s = (peer_bytes / 770e9, self_bytes / (hbm_copy * 1e9))
        ideal_s = max(parts_s) if striped else sum(parts_s)
        peak_mix = (peer_bytes + self_bytes) / ideal_s / 1e9 if ideal_s > 0 else None
        line["roofline"].update({
            "bound": "nvlink+hbm", "kernel": "miss service from the stores (peer pulls over NVLink + own-store copies)",
            "peak": round(peak_mix, 3) if peak_mix else None,
            "frac": round(achieved / peak_mix, 4) if achieved and peak_mix else None,
            "peak_source": "%s of the peer copy 770 GB/s per direction measured on this pool (MEASURED_PEAKS.json "
                           "has no NVLink figure) for the %.2f GB pulled from peers and the measured HBM copy rate "
                           "(MEASURED_PEAKS.json hbm_gbs / 2 = %.1f GB/s) for the %.2f GB copied from the rank's own "
                           "store, rank 0's timed tokens" % ("the slower (stripes pulled together)" if striped else
                                                             "blend (sum of times)", peer_bytes / 1e9, hbm_copy,
                                                             self_bytes / 1e9)})
    if a.file:
        # a file miss is a synchronous O_DIRECT read into a staging buffer, then its copy to HBM on a copy stream; with
        # several staging buffers the next miss's read runs while the last one's copy lands, so the ideal mover is
        # bound by the slower of the two rates
        rd = dg["disk_read_bytes"] / (dg["disk_read_ns"] / 1e9) / 1e9 if dg["disk_read_ns"] else None
        # with descriptor hashes every file read is hashed on the host as it is read (the reference's read_checked):
        # a read then takes the longer of reading and hashing
        hash_rate = host_hash_rate(unit) if hashed else None
        # an ideal mover serves the file misses at the slowest of read, hash and link, and the misses from pinned
        # blocks at the link, in the proportion of rank 0's timed tokens
        file_rate = min(r for r in (read_peak, hash_rate, peak) if r) if read_peak and peak else None
        file_units = min(dg["disk_reads"], units_moved)
        ideal_s = (file_units * unit / (file_rate * 1e9) + (units_moved - file_units) * unit / (peak * 1e9)
                   if file_rate else 0)
        peak_file = units_moved * unit / ideal_s / 1e9 if ideal_s > 0 else None
        line["config"].update({"workload": WORKLOAD.replace("-peer", "") + "-file", "pinned_per_layer": a.pinned_per_layer,
                               "staging": a.staging, "file_units": LAYERS * UNITS - RESIDENTS -
                               a.pinned_per_layer * LAYERS})
        line["file_tier"] = {"disk_read_gbs": round(rd, 3) if rd else None,
                             "host_hash_gbs": round(hash_rate, 3) if hash_rate else None,
                             "file_read_peak_gbs": round(read_peak, 3) if read_peak else None,
                             "reads_per_token": round(dg["disk_reads"] / a.steps, 3)}
        line["roofline"].update({
            "bound": "file+link", "kernel": "miss service (file read into staging, then the copy, entries and ready)",
            "peak": round(peak_file, 3) if peak_file else None,
            "frac": round(achieved / peak_file, 4) if achieved and peak_file else None,
            "peak_source": "rates measured in this run: a file miss at the slowest of the model file read unit "
                           "after unit as the file tier reads it (O_DIRECT, 8 MiB pieces, 8 reader threads), the host "
                           "xxh64 of one unit on one thread (with descriptor hashes; it overlaps the read) and the "
                           "copy-engine pinned->HBM rate (a read overlaps the previous miss's copy through the staging "
                           "buffers); a miss from a pinned block at that copy rate; blended in the proportion of rank "
                           "0's timed tokens (%d file reads of %d units)" % (file_units, units_moved)})
        a.no_cpu_baseline = True  # the reference arm's sample is the pinned-RAM configuration
    if not a.no_cpu_baseline and world == 1:
        # the reference arm's own measurement (same trace, tokens and warm-up subtraction)
        import oracle
        v_ref, dt_ref = reference_measure(ids, a)
        line["cpu_baseline"] = {"value": round(v_ref, 3), "unit": "GB/s",
                                "cores": int(oracle.ref().oref_copy_threads()), "kind": "reference",
                                "sample": reference_sample_text(a, dt_ref)}
    print(json.dumps(line))
    if dist:
        dist.destroy_process_group()
    return 1 if v_bad else 0


if __name__ == "__main__":
    sys.exit(main())
