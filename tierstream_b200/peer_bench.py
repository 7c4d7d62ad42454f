"""NVLink pull rate of the peer tier's mover (K5), and a planning round's store migration, one process per GPU under
torchrun:

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 -m tierstream_b200.peer_bench

Every rank fills its store (the units it owns of the benchmark's Mixtral-shaped model, owners planned from the ranks'
summed routing counts), the ranks exchange the stores' IPC handles, then rank r copies `--units` units of rank
(r + 1) % N's store into a local buffer, every rank at once (each GPU's link carries one pull in and one out), with
(a) one land-kernel launch (SM loads over NVLink) and (b) the copy engines (cudaMemcpyAsync per part), each timed
with CUDA events on the launching stream after warm-up; then rank 0 alone. Then a re-plan from other routing counts
migrates every rank's store (new stores filled from the current ones: peers over NVLink, its own in HBM), timed on
the host around the copies, max over ranks. Rank 0 prints one JSON line with the per-rank GB/s (max-time over ranks)
against the pool's measured 770 GB/s per direction, and the migration's aggregate GB/s.
"""
import argparse
import ctypes as C
import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

from . import abi, harness, peer, runtime, synth

LAYERS, UNITS, PART = 32, 8, 33030144


def cudart():
    try:
        from cuda.bindings import runtime as rt
    except ImportError:  # older cuda-python
        from cuda import cudart as rt
    return rt


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--units", type=int, default=12)
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    assert world >= 2, "run under torchrun with at least two ranks"
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    setup = None
    try:
        model = synth.Model(os.path.join(harness.model_dir(), "tsb-bench-mixtral-dg.bin"), LAYERS, UNITS, [PART] * 3,
                            seed=0, top_k=2)
        if rank == 0:
            model.write()
        dist.barrier()
        cal = synth.zipf_trace(64, LAYERS, UNITS, 2, s=1.1, seed=1001 + rank)
        counts = np.bincount((np.arange(LAYERS)[None, :, None] * UNITS + cal).reshape(-1), minlength=LAYERS * UNITS)
        setup = peer.PeerSetup(runtime.Desc(model.desc()), counts, dist, world, rank, local, verify=False,
                               collective_device=dev)
        src_rank = (rank + 1) % world
        _, per = peer.store_index(setup.owner, world)
        n = min(a.units, int(per.min()))
        base = setup.tier.bases[src_rank]
        unit = model.unit_bytes
        dst = torch.empty(n * unit, dtype=torch.uint8, device=dev)
        srcs = [base + i * unit + p * PART for i in range(n) for p in range(3)]
        dsts = [dst.data_ptr() + i * unit + p * PART for i in range(n) for p in range(3)]
        s = torch.cuda.Stream()
        lib = abi.load()
        sp = (C.c_void_p * len(srcs))(*srcs)
        dp = (C.c_void_p * len(dsts))(*dsts)
        by = (C.c_uint64 * len(srcs))(*([PART] * len(srcs)))
        rt = cudart()

        def pull_kernel():
            abi.check(lib.tsb_land(sp, dp, by, len(srcs), None, None, None, 0, None, 0, None, 0, s.cuda_stream))

        def pull_ce():
            for x, y in zip(srcs, dsts):
                err = rt.cudaMemcpyAsync(y, x, PART, rt.cudaMemcpyKind.cudaMemcpyDefault, s.cuda_stream)
                assert int(err[0]) == 0, err

        def timed(fn, alone):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ms = []
            for i in range(a.warmup + a.reps):
                dist.barrier()
                if alone and rank != 0:
                    continue
                torch.cuda.synchronize()
                e0.record(s)
                fn()
                e1.record(s)
                e1.synchronize()
                if i >= a.warmup:
                    ms.append(e0.elapsed_time(e1))
            med = float(np.median(ms)) if ms else 0.0
            t = torch.tensor([med], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())

        moved = n * unit
        out = {}
        for name, fn in (("kernel", pull_kernel), ("ce", pull_ce)):
            for alone in (False, True):
                ms = timed(fn, alone)
                out["%s_%s" % (name, "alone" if alone else "all")] = {
                    "ms": round(ms, 4), "gbs_per_rank": round(moved / ms / 1e6, 2),
                    "frac_of_770": round(moved / ms / 1e6 / 770.0, 4)}
        # the bytes pulled equal the owner's source bytes (spot check: first and last unit)
        got = dst.view(n, unit)[[0, n - 1]].cpu().numpy()
        own_keys = np.nonzero(setup.owner == src_rank)[0]
        for row, k in zip(got, own_keys[[0, n - 1]]):
            want = model.unit_bytes_of(int(k) // UNITS, int(k) % UNITS)
            assert np.array_equal(row, want), "rank %d pulled wrong bytes of key %d" % (rank, k)
        # a planning round: other routing counts, new owners, every rank's new store filled from the current ones
        cal2 = synth.zipf_trace(64, LAYERS, UNITS, 2, s=1.1, seed=5001 + rank)
        counts2 = np.bincount((np.arange(LAYERS)[None, :, None] * UNITS + cal2).reshape(-1),
                              minlength=LAYERS * UNITS)
        dist.barrier()
        mig = setup.replan(runtime.Desc(model.desc()), counts2, dist, world, rank, local, collective_device=dev)
        t = torch.tensor([mig["seconds"], float(mig["bytes"]), float(mig["peer_units"] * unit)], dtype=torch.float64,
                         device=dev)
        tmax = t[:1].clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        tsum = t[1:].clone()
        dist.all_reduce(tsum, op=dist.ReduceOp.SUM)
        out["replan_migration"] = {"seconds_max_over_ranks": round(float(tmax.item()), 4),
                                   "bytes_all_ranks": int(tsum[0].item()),
                                   "bytes_from_peers_all_ranks": int(tsum[1].item()),
                                   "gbs_all_ranks": round(float(tsum[0].item()) / float(tmax.item()) / 1e9, 2)}
        if rank == 0:
            print(json.dumps({"bench": "peer pull (K5)", "n_gpus": world, "units_per_rank": n, "unit_bytes": unit,
                              "bytes_per_rank": moved, "peak_gbs_per_direction": 770.0,
                              "peak_source": "peer copy measured on this pool", **out}), flush=True)
        dist.barrier()
    finally:
        if setup:
            setup.close()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
