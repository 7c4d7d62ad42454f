"""The peer tier on the GPU: misses on owned units are copied from the owners' stores, every unit the engine reads has
the source bytes, and the slot table after every token equals the reference DgCore's on the same trace with the
owned units treated as pinned-RAM homes (deterministic schedule). One GPU emulates two ranks (both stores in its
HBM, the store addresses handed over directly); with two GPUs, two processes exchange CUDA IPC handles after an
NCCL all-reduce of their routing counts."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import oracle  # noqa: E402
from tierstream_b200 import harness, peer, runtime, synth  # noqa: E402


def expected_sums(model, orc):
    out = np.zeros(model.layers * model.units, dtype=np.uint64)
    buf = np.empty(model.unit_bytes, dtype=np.uint8)
    for L in range(model.layers):
        for u in range(model.units):
            orc.orc_fill_bytes(model.seed, model.unit_offset(L, u), model.unit_bytes, buf.ctypes.data)
            out[L * model.units + u] = orc.orc_checksum(buf.ctypes.data, model.unit_bytes)
    return out


def replay_cfg_for(run, model, tokens):
    P = model.layers * model.units - len(run.resident_keys)
    return runtime.replay_config([model.units] * model.layers, list(model.part_bytes),
                                 persistent_slots=len(run.resident_keys) + model.layers, bank_slots=run.n_ids,
                                 blocks=P + model.layers, spare_target=model.layers, order=run.resident_keys,
                                 tokens=tokens, n_ids=run.n_ids)


def route_counts(model, ids):
    keys = np.arange(model.layers)[None, :, None] * model.units + ids
    return np.bincount(keys.reshape(-1), minlength=model.layers * model.units).astype(np.uint64)


@pytest.fixture(scope="module")
def model():
    m = synth.Model(os.path.join(harness.model_dir(), "tsb-test-peer.bin"), layers=6, units=16,
                    part_bytes=(2048, 2048, 4096), seed=5, top_k=2, with_hash=True)
    m.write()
    return m


def check_run(run, m, ids, want, ref_tables):
    for t in range(ids.shape[0]):
        got = run.step(ids[t])
        keys = np.arange(m.layers)[:, None] * m.units + ids[t]
        assert np.array_equal(got, want[keys]), "token %d read wrong bytes" % t
        assert np.array_equal(run.ctx.table(run.keys), ref_tables[t]), "slot table differs after token %d" % t


@pytest.mark.parametrize("copy", [0, 1])
@pytest.mark.parametrize("mixed", [False, True])
def test_emulated_two_ranks(model, orc, monkeypatch, copy, mixed):
    monkeypatch.setenv("TSB_DG_DETERMINISTIC", "1")
    m = model
    ids = synth.zipf_trace(40, m.layers, m.units, 2, s=1.0, seed=21)
    counts = route_counts(m, ids[:10])
    keys = m.layers * m.units
    owner = peer.plan_owners(counts, 2, cap_units=[keys // 4, keys // 4] if mixed else None)
    assert ((owner < 0).any()) == mixed
    desc = runtime.Desc(m.desc())
    stores = [peer.Store(desc, owner, r, 0, verify=True) for r in range(2)]
    tier = peer.Tier(2, 0, owner, [s.base for s in stores], copy=copy)
    run = harness.DgRun(m, residents_per_layer=3, max_ids=2, verify=True, peer=tier)
    try:
        open_table = run.ctx.table(run.keys).copy()
        want = expected_sums(m, orc)
        t_ref, s_ref = oracle.ref_replay(replay_cfg_for(run, m, ids.shape[0]), ids)
        check_run(run, m, ids, want, t_ref)
        st = run.ctx.stats()
        assert st["misses"] == s_ref[-1][2] and st["fetched"] == s_ref[-1][4] and st["evicted"] == s_ref[-1][10]
        import json
        pj = json.loads(run.ctx.stats_json())["peer"]
        assert pj["world"] == 2 and pj["all_owned"] == (0 if mixed else 1)
        assert pj["peer_units"] > 0 and pj["self_units"] > 0
        if not mixed:
            assert pj["peer_units"] + pj["self_units"] == st["fetched"] + st["prefetched"]
        run.ctx.check()
        for L in range(m.layers):
            for u in range(m.units):
                run.ctx.check_unit(L, u)
        run.ctx.reset_open()  # moves through the staging unit take their bytes from the stores
        assert np.array_equal(run.ctx.table(run.keys), open_table)
        for L in range(m.layers):
            for u in range(m.units):
                run.ctx.check_unit(L, u)
    finally:
        run.close()
        for s in stores:
            s.close()


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("copy", [0, 1])
@pytest.mark.parametrize("mixed", [False, True])
def test_striped_emulated_ranks(model, orc, monkeypatch, world, copy, mixed):
    """The striped layout on one GPU: `world` stores, each holding one stripe of every owned unit (world = 3 gives
    2,816-byte stripes whose edges fall inside the 2,048 / 2,048 / 4,096-byte parts, the last stripe 2,560 bytes).
    The ranks' shares of the tier check (tsb_peer_tier_verify) cover every owned unit once; the last rank decodes,
    reading the source bytes, with the slot table after every token equal to the reference replay; every owned
    unit's pulls took one stripe from each store."""
    from tierstream_b200 import abi
    monkeypatch.setenv("TSB_DG_DETERMINISTIC", "1")
    m = model
    ids = synth.zipf_trace(40, m.layers, m.units, 2, s=1.0, seed=22)
    keys = m.layers * m.units
    owner = peer.plan_owners(route_counts(m, ids[:10]), world,
                             cap_units=[keys // (2 * world)] * world if mixed else None)
    assert ((owner < 0).any()) == mixed
    owned = int((owner >= 0).sum())
    desc = runtime.Desc(m.desc())
    stores = [peer.Store(desc, owner, r, 0, layout=abi.PEER_STRIPED, world=world) for r in range(world)]
    stripe = peer.stripe_bytes(m.unit_bytes, world)
    assert stripe == -(-(-(-m.unit_bytes // world)) // 256) * 256
    assert all(s.bytes == owned * stripe for s in stores)
    bases = [s.base for s in stores]
    checked = [peer.verify_tier(desc, peer.Tier(world, r, owner, bases, copy, abi.PEER_STRIPED), 0)
               for r in range(world)]
    assert sum(checked) == owned and max(checked) - min(checked) <= 1
    k0 = int(np.nonzero(owner >= 0)[0][0])
    lo, n = peer.stripe_range(m.unit_bytes, world, world - 1)
    assert np.array_equal(peer.read_device(stores[-1].base, n),
                          m.unit_bytes_of(k0 // m.units, k0 % m.units)[lo:lo + n])
    rank = world - 1
    tier = peer.Tier(world, rank, owner, bases, copy=copy, layout=abi.PEER_STRIPED)
    run = harness.DgRun(m, residents_per_layer=3, max_ids=2, verify=True, peer=tier)
    try:
        open_table = run.ctx.table(run.keys).copy()
        t_ref, s_ref = oracle.ref_replay(replay_cfg_for(run, m, ids.shape[0]), ids)
        check_run(run, m, ids, expected_sums(m, orc), t_ref)
        st = run.ctx.stats()
        assert st["misses"] == s_ref[-1][2] and st["fetched"] == s_ref[-1][4]
        import json
        pj = json.loads(run.ctx.stats_json())["peer"]
        assert pj["layout"] == "striped" and pj["world"] == world and pj["self_units"] == 0
        assert pj["peer_units"] > 0 and pj["self_bytes"] == pj["peer_units"] * n
        assert pj["peer_bytes"] + pj["self_bytes"] == pj["peer_units"] * m.unit_bytes
        if not mixed:
            assert pj["peer_units"] == st["fetched"] + st["prefetched"]
        run.ctx.check()
        for L in range(m.layers):
            for u in range(m.units):
                run.ctx.check_unit(L, u)
        run.ctx.reset_open()  # residents taken from the stores again, stripe by stripe
        assert np.array_equal(run.ctx.table(run.keys), open_table)
        for L in range(m.layers):
            for u in range(m.units):
                run.ctx.check_unit(L, u)
    finally:
        run.close()
        for s in stores:
            s.close()


def test_striped_tier_check_finds_a_changed_byte(model):
    """One byte of one stripe changed in its store: the share of the tier check that gathers that unit reports
    SS_E_HASH, the other share passes; a striped store refuses a migration and a per-store check."""
    from tierstream_b200 import abi
    m = model
    owner = peer.plan_owners(np.ones(m.layers * m.units, dtype=np.uint64), 2)
    desc = runtime.Desc(m.desc())
    stores = [peer.Store(desc, owner, r, 0, layout=abi.PEER_STRIPED, world=2) for r in range(2)]
    bases = [s.base for s in stores]
    try:
        for r in range(2):
            peer.verify_tier(desc, peer.Tier(2, r, owner, bases, 0, abi.PEER_STRIPED), 0)

        class _View:  # stripe 1 of owned unit 0 (position 0: rank 0's share), byte 5
            __cuda_array_interface__ = {"shape": (16,), "typestr": "|u1", "data": (bases[1], False), "version": 3}

        v = torch.as_tensor(_View(), device="cuda")
        v[5] ^= 0x5A
        torch.cuda.synchronize()
        with pytest.raises(abi.TsError) as e:
            peer.verify_tier(desc, peer.Tier(2, 0, owner, bases, 0, abi.PEER_STRIPED), 0)
        assert e.value.status == abi.SS_E_HASH
        assert peer.verify_tier(desc, peer.Tier(2, 1, owner, bases, 0, abi.PEER_STRIPED), 0) > 0
        s = torch.cuda.Stream()
        dst = peer.Store(desc, owner, 0, 0, fill=False, layout=abi.PEER_STRIPED, world=2)
        with pytest.raises(abi.TsError) as e:
            dst.migrate_from(owner, bases, s.cuda_stream)
        assert e.value.status == abi.SS_E_UNSUPPORTED
        dst.close()
    finally:
        for s in stores:
            s.close()


def test_replan_migrates_the_stores_mid_decode(model, orc, monkeypatch):
    """A planning round between tokens: new owners from other counts, new stores filled from the current ones
    (tsb_peer_store_migrate), the context switched to them (tsb_dg_peer_retier), the old stores freed. The decode
    goes on reading the source bytes, and the tables keep equal to the reference replay of the whole trace (the
    owners never enter the cache's decisions)."""
    import torch as T
    monkeypatch.setenv("TSB_DG_DETERMINISTIC", "1")
    m = model
    ids = synth.zipf_trace(30, m.layers, m.units, 2, s=1.0, seed=31)
    a = peer.plan_owners(route_counts(m, ids[:10]), 2)
    b = peer.plan_owners(route_counts(m, synth.zipf_trace(10, m.layers, m.units, 2, s=1.0, seed=99)), 2)
    assert (a != b).sum() > 10
    desc = runtime.Desc(m.desc())
    old = [peer.Store(desc, a, r, 0, verify=True) for r in range(2)]
    run = harness.DgRun(m, residents_per_layer=3, max_ids=2, peer=peer.Tier(2, 0, a, [x.base for x in old]))
    new = []
    try:
        want = expected_sums(m, orc)
        t_ref, _ = oracle.ref_replay(replay_cfg_for(run, m, ids.shape[0]), ids)
        check_run(run, m, ids[:15], want, t_ref[:15])
        s = T.cuda.Stream()
        for r in range(2):
            st = peer.Store(desc, b, r, 0, fill=False)
            units, peer_units, nbytes = st.migrate_from(a, [x.base for x in old], s.cuda_stream)
            assert units == (b == r).sum() and peer_units == ((b == r) & (a != r)).sum()
            assert nbytes == units * m.unit_bytes
            new.append(st)
        run.ctx.retier(peer.Tier(2, 0, b, [x.base for x in new]))
        for x in old:
            x.close()
        for t in range(15, 30):
            got = run.step(ids[t])
            keys = np.arange(m.layers)[:, None] * m.units + ids[t]
            assert np.array_equal(got, want[keys]), "token %d read wrong bytes after the re-plan" % t
            assert np.array_equal(run.ctx.table(run.keys), t_ref[t]), "slot table differs after token %d" % t
        for L in range(m.layers):
            for u in range(m.units):
                run.ctx.check_unit(L, u)
    finally:
        run.close()
        for x in old + new:
            x.close()


def _two_gpu_rank(rank, world, port, path, out_dir, layout):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["TSB_DG_DETERMINISTIC"] = "1"
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    setup = run = None
    try:
        m = synth.Model(path, layers=6, units=16, part_bytes=(2048, 2048, 4096), seed=5, top_k=2, with_hash=True)
        ids = synth.zipf_trace(30, m.layers, m.units, 2, s=1.0, seed=40 + rank)
        desc = runtime.Desc(m.desc())
        setup = peer.PeerSetup(desc, route_counts(m, ids[:10]), dist, world, rank, rank, verify=True, copy=0,
                               collective_device=torch.device("cuda", rank), layout=layout)
        if layout:  # striped: the ranks' shares of the tier check gathered every unit over NVLink
            assert setup.checked_units == m.layers * m.units // world
        run = harness.DgRun(m, residents_per_layer=3, max_ids=2, peer=setup.tier)
        got = [run.step(ids[t]) for t in range(15)]
        # a planning round mid-decode: other counts, new owners, stores migrated over NVLink (striped: kept), the
        # context switched
        mig = setup.replan(desc, route_counts(m, synth.zipf_trace(10, m.layers, m.units, 2, s=1.0, seed=70 + rank)),
                           dist, world, rank, rank, ctx=run.ctx, collective_device=torch.device("cuda", rank))
        assert mig["units"] == (0 if layout else (setup.owner == rank).sum())
        got += [run.step(ids[t]) for t in range(15, ids.shape[0])]
        got = np.stack(got)
        tables = np.stack([run.ctx.table(run.keys)])  # final table only; per-token parity is checked below
        np.savez(os.path.join(out_dir, "r%d.npz" % rank), got=got, owner=setup.owner, table=tables[0],
                 resident=np.array(run.resident_keys))
        run.close()
        run = None
        dist.barrier()
    finally:
        if run:
            run.close()
        if setup:
            dist.barrier()
            setup.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("layout", [0, 1], ids=["whole", "striped"])
def test_two_gpus_exchange_and_pull(model, orc, tmp_path, layout):
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_two_gpu_rank, args=(2, port, model.path, str(tmp_path), layout), nprocs=2,
                       start_method="spawn")
    want = expected_sums(model, orc)
    r = [np.load(tmp_path / ("r%d.npz" % i)) for i in range(2)]
    assert np.array_equal(r[0]["owner"], r[1]["owner"])
    for rank in range(2):
        ids = synth.zipf_trace(30, model.layers, model.units, 2, s=1.0, seed=40 + rank)
        keys = np.arange(model.layers)[None, :, None] * model.units + ids
        assert np.array_equal(r[rank]["got"], want[keys]), "rank %d read wrong bytes" % rank
        cfg = runtime.replay_config([model.units] * model.layers, list(model.part_bytes),
                                    persistent_slots=len(r[rank]["resident"]) + model.layers, bank_slots=2,
                                    blocks=model.layers * model.units - len(r[rank]["resident"]) + model.layers,
                                    spare_target=model.layers, order=list(r[rank]["resident"]), tokens=30, n_ids=2)
        t_ref, _ = oracle.ref_replay(cfg, ids)
        assert np.array_equal(r[rank]["table"], t_ref[-1]), "rank %d slot table differs" % rank


def test_allocated_stores_written_on_the_device(model, orc, monkeypatch):
    """Stores the library only allocates (tsb_peer_store_alloc), written by the caller: here by the model's byte
    generator on the device (the benchmark's way to fill stores larger than host RAM). The decode then reads the
    source bytes and the tables equal the reference replay, as with stores filled from the file."""
    import ctypes as C

    from tierstream_b200 import abi
    monkeypatch.setenv("TSB_DG_DETERMINISTIC", "1")
    m = model
    ids = synth.zipf_trace(20, m.layers, m.units, 2, s=1.0, seed=23)
    owner = peer.plan_owners(route_counts(m, ids[:8]), 2)
    desc = runtime.Desc(m.desc())
    stores = [peer.Store(desc, owner, r, 0, fill=False) for r in range(2)]
    eng = abi.load_engine()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())  # after the inputs torch made on its own stream
    for r, st in enumerate(stores):
        keys = np.nonzero(owner == r)[0]
        offs = np.array([m.unit_offset(int(k) // m.units, int(k) % m.units) for k in keys], dtype=np.uint64)
        assert eng.tse_fill_units_device(m.seed, offs.ctypes.data_as(C.POINTER(C.c_uint64)), keys.size, m.unit_bytes,
                                         st.base, s.cuda_stream) == 0
    s.synchronize()
    k0 = int(np.nonzero(owner == 1)[0][0])
    assert np.array_equal(peer.read_device(stores[1].base, m.unit_bytes),
                          m.unit_bytes_of(k0 // m.units, k0 % m.units))
    run = harness.DgRun(m, residents_per_layer=3, max_ids=2, peer=peer.Tier(2, 0, owner, [x.base for x in stores]))
    try:
        t_ref, _ = oracle.ref_replay(replay_cfg_for(run, m, ids.shape[0]), ids)
        check_run(run, m, ids, expected_sums(m, orc), t_ref)
    finally:
        run.close()
        for x in stores:
            x.close()
