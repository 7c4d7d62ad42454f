"""The benchmark's workload set-ups, on the CPU: the host-mode workloads' tiers, budgets and routes are BASELINE
configs[0] and [2] as tierstream_b200/host_bench.py states them, their plans are accepted by the planner, and the
directory bench.py --impl reference-cuda hands the reference's driver holds what the driver reads (struct bytes at the
ABI's sizes, the shape, the trace)."""
import ctypes as C
import os
import sys

import numpy as np

from tierstream_b200 import abi, harness, host_bench, runtime, synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_c1_host_is_configs_0():
    w = host_bench.WORKLOADS["c1-host"]
    tiers = host_bench.tiers_of("c1-host")
    assert len(tiers) == 8 * 16
    per_layer = np.array(tiers).reshape(8, 16)
    assert (per_layer[:, :4] == abi.SS_TIER_RESIDENT).all() and (per_layer[:, 4:] == abi.SS_TIER_PINNED).all()
    routes = host_bench.routes_of("c1-host", 64)
    assert routes.shape == (64, 8, 2) and all(len(set(r)) == 2 for r in routes.reshape(-1, 2))
    m = host_bench.model_of("c1-host")
    assert m.unit_bytes == 3 * 131072 and w["ring"] == 4
    b, o = host_bench.budget_options("c1-host", m)
    assert b.ring_slots == 4 and b.dynamic_slots_per_layer == 0 and o.forward_mode == abi.SS_FORWARD_HOST
    assert o.verify_hash == 1


def test_llama3_host_is_configs_2_and_its_plan_is_accepted(tmp_path, monkeypatch):
    m = host_bench.model_of("llama3-70b-host")
    assert m.unit_bytes == 1711308800 and m.layers == 80 and m.units == 1
    tiers = host_bench.tiers_of("llama3-70b-host")
    assert tiers[:35] == [abi.SS_TIER_RESIDENT] * 35 and tiers[35:] == [abi.SS_TIER_PINNED] * 45
    assert 35 * m.unit_bytes <= 60e9  # the 60 GB VRAM budget
    b, o = host_bench.budget_options("llama3-70b-host", m)
    assert b.ring_slots == 2
    desc = runtime.Desc(host_bench.desc_of("llama3-70b-host", m))
    plan = runtime.Plan(desc, b, tiers=tiers)  # the planner accepts it (device and pinned bytes within the budget)
    assert plan.h


def test_reference_cuda_directory_holds_what_the_driver_reads(tmp_path, monkeypatch):
    sys.path.insert(0, ROOT)
    import bench
    m = synth.Model(str(tmp_path / "m.bin"), layers=3, units=4, part_bytes=(4096, 4096, 8192), seed=3, top_k=2)
    setup = harness.DgSetup(m, residents_per_layer=1, max_ids=2, test_hooks=False)
    ids = synth.zipf_trace(5, 3, 4, 2, seed=1)
    want = np.arange(12, dtype=np.uint64)
    d = bench.reference_cuda_dir(m, setup, ids, want, 2)
    try:
        assert os.path.getsize(os.path.join(d, "budget.bin")) == C.sizeof(abi.ss_budget)
        assert os.path.getsize(os.path.join(d, "options.bin")) == C.sizeof(abi.ss_options)
        assert open(os.path.join(d, "meta.txt")).read().split() == ["3", "4", "2"]
        assert np.array_equal(np.fromfile(os.path.join(d, "ids.i32"), dtype=np.int32), ids.reshape(-1))
        assert np.array_equal(np.fromfile(os.path.join(d, "want.u64"), dtype=np.uint64), want)
        assert list(np.fromfile(os.path.join(d, "tiers.u8"), dtype=np.uint8)) == setup.tiers
    finally:
        import shutil
        shutil.rmtree(d, ignore_errors=True)


def test_peer_defaults_follow_the_measurements(monkeypatch):
    """--peer-layout / --peer-copy auto: striped stores with the land kernel for the Mixtral shape, whole units with
    the land kernel for the top-8 shapes, the copy engines for Mixtral's whole units; explicit choices kept."""
    sys.path.insert(0, ROOT)
    import bench
    cases = [([], ("striped", "kernel")), (["--workload", "deepseek-v3-peer"], ("whole", "kernel")),
             (["--workload", "qwen3-235b-a22b-peer"], ("whole", "kernel")), (["--peer-layout", "whole"], ("whole", "ce")),
             (["--peer-layout", "striped", "--peer-copy", "ce"], ("striped", "ce"))]
    for argv, want in cases:
        monkeypatch.setattr(sys, "argv", ["bench.py"] + argv)
        a = bench.args_()
        names = set(bench.QWEN3) | set(bench.DEEPSEEK) | {"LAYERS", "RESIDENTS", "MODEL_FILE"}
        saved = {k: getattr(bench, k) for k in names if hasattr(bench, k)}  # configure sets the module's shape
        try:
            bench.configure(a)
        finally:
            for k, v in saved.items():
                setattr(bench, k, v)
        assert (a.peer_layout, a.peer_copy) == want, argv
