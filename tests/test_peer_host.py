"""The peer tier's host logic, without a GPU: the owner planner's rules, the store index, the two-rank exchange step
(an all-reduce of routing counts over gloo, then the same owners on every rank), and tsb_open_peer's argument checks
(refused before any device call)."""
import ctypes as C
import os

import numpy as np
import pytest

from tierstream_b200 import abi, harness, peer, runtime, synth


def test_equal_counts_deal_keys_round_robin():
    owner = peer.plan_owners(np.ones(10, dtype=np.uint64), 3)
    assert owner.tolist() == [0, 1, 2, 0, 1, 2, 0, 1, 2, 0]


def test_hot_keys_spread_and_loads_balance():
    rng = np.random.default_rng(0)
    counts = (rng.zipf(1.3, size=512) % 10000).astype(np.uint64)
    for world in (2, 4, 8):
        owner = peer.plan_owners(counts, world)
        assert owner.min() == 0 and owner.max() == world - 1
        loads = np.array([counts[owner == r].sum() for r in range(world)], dtype=np.float64)
        # greedy on descending counts: every rank's load within the largest single count of the mean
        assert loads.max() - loads.min() <= counts.max()
        hottest = np.argsort(-counts.astype(np.int64), kind="stable")[:world]
        assert sorted(owner[hottest].tolist()) == list(range(world)), "the hottest keys go to different ranks"


def test_plan_is_deterministic_and_tie_rules():
    counts = np.array([5, 9, 5, 0, 9, 1], dtype=np.uint64)
    a = peer.plan_owners(counts, 2)
    b = peer.plan_owners(counts.copy(), 2)
    assert np.array_equal(a, b)
    # order: 1 (9), 4 (9), 0 (5), 2 (5), 5 (1), 3 (0); loads: r0 9, r1 9 -> 0 to r0 (tie: fewer units equal, lower
    # rank), 2 to r1, 5 to r0 (14 vs 14, units 2 vs 2 -> r0), 3 to r1 (r1 14 < r0 15)
    assert a.tolist() == [0, 0, 1, 1, 1, 0]


def test_capacity_and_overflow_to_pinned():
    counts = np.arange(12, dtype=np.uint64)
    owner = peer.plan_owners(counts, 2, cap_units=[3, 4])
    assert (owner == 0).sum() == 3 and (owner == 1).sum() == 4 and (owner == -1).sum() == 5
    # the unowned keys are the coldest
    assert set(np.nonzero(owner == -1)[0].tolist()) == {0, 1, 2, 3, 4}


def test_store_index_follows_key_order_per_owner():
    owner = np.array([1, 0, 1, -1, 0, 1], dtype=np.int32)
    index, per = peer.store_index(owner, 2)
    assert index.tolist() == [0, 0, 1, -1, 1, 2]
    assert per.tolist() == [2, 3]


def test_bad_plan_arguments():
    lib = abi.load()
    counts = (C.c_uint64 * 4)(1, 2, 3, 4)
    owner = (C.c_int32 * 4)()
    assert lib.tsb_peer_plan(counts, 4, 0, None, owner) == abi.SS_E_INVALID
    bad = np.array([0, 2], dtype=np.int32)
    assert lib.tsb_peer_index(bad.ctypes.data_as(C.POINTER(C.c_int32)), 2, 2, None, None) == abi.SS_E_INVALID
    assert b"not a rank below the world size" in lib.ss_last_error()


def _rank_main(rank, world, port, out_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ids = synth.zipf_trace(20, 4, 16, 2, s=1.1, seed=100 + rank)  # each rank routes its own trace
        local = np.bincount((np.arange(4)[None, :, None] * 16 + ids).reshape(-1), minlength=64)
        counts = peer.all_reduce_counts(local, dist)
        owner = peer.plan_owners(counts, world)
        handles = peer.all_gather_handles(bytes([rank]) * 64, dist, world)
        np.save(os.path.join(out_dir, "r%d.npy" % rank), np.concatenate([counts.astype(np.int64), owner]))
        assert [h[0] for h in handles] == list(range(world))
    finally:
        dist.destroy_process_group()


def test_two_ranks_plan_the_same_owners(tmp_path):
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_rank_main, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn")
    r0, r1 = np.load(tmp_path / "r0.npy"), np.load(tmp_path / "r1.npy")
    assert np.array_equal(r0, r1)
    want = np.zeros(64, dtype=np.int64)
    for r in range(2):
        ids = synth.zipf_trace(20, 4, 16, 2, s=1.1, seed=100 + r)
        want += np.bincount((np.arange(4)[None, :, None] * 16 + ids).reshape(-1), minlength=64)
    assert np.array_equal(r0[:64], want)
    assert np.array_equal(r0[64:], peer.plan_owners(want.astype(np.uint64), 2))


def test_open_peer_refuses_bad_tiers():
    m = synth.Model(os.path.join(harness.model_dir(), "tsb-peer-args.bin"), layers=2, units=4,
                    part_bytes=(256, 256, 256), seed=1)
    desc = runtime.Desc(m.desc())
    lib = abi.load()
    b = abi.budget_defaults()
    o = abi.options_defaults()
    o.forward_mode = abi.SS_FORWARD_DEVICE_GATED
    owner = np.zeros(8, dtype=np.int32)

    def opened(tier):
        h = C.c_void_p()
        t = tier.struct()
        return lib.tsb_open_peer(desc.h, C.byref(b), None, C.byref(o), C.byref(t), C.byref(h))

    assert opened(peer.Tier(2, 2, owner, [0, 0])) == abi.SS_E_INVALID  # rank outside the world
    assert b"rank outside" in lib.ss_last_error()
    assert opened(peer.Tier(2, 0, owner[:6], [0, 0])) == abi.SS_E_INVALID  # fewer keys than gated units
    assert b"gated units" in lib.ss_last_error()
    assert opened(peer.Tier(1, 0, owner, [0])) == abi.SS_E_INVALID  # rank 0 owns units but has no store
    assert b"store_base is null" in lib.ss_last_error()
    t = peer.Tier(1, 0, owner, [0x1000], copy=2)
    assert opened(t) == abi.SS_E_INVALID


def test_stripe_geometry():
    """The striped layout's stripes: ceil(unit / world) rounded up to 256 bytes, covering the unit once in rank order,
    the last ones shorter or empty; the benchmarked expert sizes cut into equal stripes."""
    for unit, world in [(8192, 2), (8192, 3), (99090432, 8), (44040192, 8), (1000, 8), (100, 3), (256, 1)]:
        s = peer.stripe_bytes(unit, world)
        assert s % 256 == 0 and s * world >= unit and s - 256 < -(-unit // world)
        ranges = [peer.stripe_range(unit, world, r) for r in range(world)]
        assert sum(n for _, n in ranges) == unit
        assert all(lo == r * s for r, (lo, _) in enumerate(ranges))
        lens = [n for _, n in ranges]
        assert lens == sorted(lens, reverse=True)  # full stripes, then at most one short one, then empty ones
    assert peer.stripe_bytes(99090432, 8) == 99090432 // 8  # the Mixtral-shaped expert
    assert peer.stripe_bytes(44040192, 8) == 44040192 // 8  # the DeepSeek-shaped expert
    assert [peer.stripe_range(1000, 8, r)[1] for r in range(8)] == [256, 256, 256, 232, 0, 0, 0, 0]
    assert abi.load().tsb_peer_stripe_bytes(1000, 0) == 0


def test_striped_entry_points_refuse_bad_arguments():
    m = synth.Model(os.path.join(harness.model_dir(), "tsb-peer-args.bin"), layers=2, units=4,
                    part_bytes=(256, 256, 256), seed=1)
    desc = runtime.Desc(m.desc())
    lib = abi.load()
    owner = np.zeros(8, dtype=np.int32)
    op = owner.ctypes.data_as(C.POINTER(C.c_int32))
    h = C.c_void_p()
    assert lib.tsb_peer_store_create_striped(desc.h, op, 8, 2, 2, 0, 1, C.byref(h)) == abi.SS_E_INVALID
    assert b"rank below it" in lib.ss_last_error()
    assert lib.tsb_peer_store_create_striped(desc.h, op, 8, 0, 0, 0, 1, C.byref(h)) == abi.SS_E_INVALID
    assert lib.tsb_peer_store_create_striped(desc.h, op, 7, 0, 2, 0, 1, C.byref(h)) == abi.SS_E_INVALID
    assert lib.tsb_peer_store_create_striped(None, op, 8, 0, 2, 0, 1, C.byref(h)) == abi.SS_E_INVALID
    t = peer.Tier(2, 0, owner, [0x1000, 0x2000], layout=2).struct()
    assert lib.tsb_peer_tier_verify(desc.h, C.byref(t), 0, None) == abi.SS_E_INVALID
    assert b"layout must be" in lib.ss_last_error()
    b = abi.budget_defaults()
    o = abi.options_defaults()
    o.forward_mode = abi.SS_FORWARD_DEVICE_GATED
    t = peer.Tier(2, 0, owner, [0x1000, 0], layout=abi.PEER_STRIPED).struct()  # rank 1 holds stripes, no store
    assert lib.tsb_open_peer(desc.h, C.byref(b), None, C.byref(o), C.byref(t), C.byref(h)) == abi.SS_E_INVALID
    assert b"holds a stripe" in lib.ss_last_error()


def test_replan_entry_points_refuse_bad_arguments():
    lib = abi.load()
    t = peer.Tier(1, 0, np.zeros(4, dtype=np.int32), [0x1000]).struct()
    assert lib.tsb_dg_peer_retier(None, C.byref(t)) == abi.SS_E_INVALID
    owner = (C.c_int32 * 4)()
    bases = (C.c_void_p * 1)()
    assert lib.tsb_peer_store_migrate(None, owner, bases, 4, 1, None, None, None, None) == abi.SS_E_INVALID
    assert b"null argument" in lib.ss_last_error()


def _rank_dies(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        counts = peer.all_reduce_counts(np.ones(8, dtype=np.int64), dist)
        if rank == 1:
            raise SystemExit(3)  # the rank leaves between the steps, before the handle exchange
        try:
            peer.all_gather_handles(bytes(64), dist, world)
            outcome = "returned"
        except Exception as e:  # the survivor learns of it from the collective's timeout, not a hang
            outcome = "raised: " + type(e).__name__
        with open(os.path.join(out_dir, "r%d.txt" % rank), "w") as f:
            f.write("%s %d" % (outcome, int(counts.sum())))
    finally:
        if rank == 0:
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def test_a_rank_that_leaves_fails_the_exchange_with_an_error(tmp_path):
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.start_processes(_rank_dies, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn", join=False)
    ctx.processes[1].join(60)
    ctx.processes[0].join(60)
    assert ctx.processes[1].exitcode == 3
    text = (tmp_path / "r0.txt").read_text()
    assert text.startswith("raised:") and text.endswith(" 16"), text


def _pieces(parts, world, rank):
    lib = abi.load()
    pb = (C.c_uint64 * len(parts))(*parts)
    cap = world + len(parts) + 4
    out = np.zeros((cap, 5), dtype=np.uint64)
    n = C.c_uint32()
    assert lib.tsb_test_peer_pieces(pb, len(parts), world, rank, out.ctypes.data_as(C.POINTER(C.c_uint64)), cap,
                                    C.byref(n)) == abi.SS_OK
    assert n.value <= cap
    return out[:n.value]


@pytest.mark.parametrize("seed", range(40))
def test_striped_miss_copies_cover_the_unit(seed):
    """The copies a striped miss issues (the mover's own split, tsb_test_peer_pieces): every byte of every part
    exactly once, each from the stripe that holds it and inside it, the stripes in rotation from the next rank to this
    rank's own, at most world + parts - 1 copies."""
    r = np.random.default_rng(3000 + seed)
    parts = [int(r.integers(1, 40)) * 256 + (int(r.integers(0, 256)) if seed % 4 == 3 else 0)
             for _ in range(int(r.integers(1, 5)))]
    unit = sum(parts)
    offset = np.cumsum([0] + parts[:-1])
    for world in (1, 2, 3, 5, 8):
        s = peer.stripe_bytes(unit, world)
        for rank in range(world):
            cp = _pieces(parts, world, rank)
            assert len(cp) <= world + len(parts) - 1
            covered = [np.zeros(p, dtype=np.int32) for p in parts]
            order = []
            for src, in_stripe, part, in_part, n in (tuple(int(v) for v in row) for row in cp):
                assert n > 0 and in_stripe + n <= peer.stripe_range(unit, world, src)[1]
                assert src * s + in_stripe == offset[part] + in_part  # the same unit bytes on both sides
                covered[part][in_part:in_part + n] += 1
                if not order or order[-1] != src:
                    order.append(src)
            assert all((c == 1).all() for c in covered), "a byte copied twice or never"
            stripes = [q for q in range(world) if peer.stripe_range(unit, world, q)[1] > 0]
            want = [(rank + j) % world for j in range(1, world + 1) if (rank + j) % world in stripes]
            assert order == want, (order, want)
