"""The slot cache under the device's concurrency, on the CPU (tsb_test_dg_async_replay): the same seeded configurations
as the table-parity suites (two tiers with write-backs, predictions and inclusive shares; the file tier with reads in
flight, the opt-in policies, rounds and scored eviction; kept-resident layers; a reset mid-trace), driven with copy
streams as worker threads that run their work in order after random delays, events that complete when their stream
reaches them, reads that land late, and an engine thread that exports, waits and reads as the device does. Every unit
the engine reads through the device table has its own bytes, and the mover saw no hazard: no host write into a block a
pending copy uses, no host read of a block a pending copy writes, no two moves of a wave on one slot, no engine read of
a slot a pending copy writes, no copy on a block whose file read had not ended."""
import ctypes as C

import numpy as np
import pytest

from tierstream_b200 import abi

from test_dg_disk_replay import make_disk_case
from test_dg_queue_replay import random_queue_case
from test_dg_replay import make_case
from test_dg_replay_fuzz import random_case

RACES = ["host write into a busy block", "host read of a block being written", "moves of a wave on one slot",
         "engine read of a slot being written", "copy on a block being read"]


def unit_sums(src, keys, unit):
    w = (np.arange(unit, dtype=np.uint64) % 251 + 1)
    return (src.reshape(keys, unit).astype(np.uint64) * w).sum(axis=1)


def run_async(cfg, ids, preds, seed, delay_us, mutation=0):
    n_units = [cfg.n_units[i] for i in range(cfg.n_gated)]
    keys = sum(n_units)
    unit = sum(cfg.part_bytes[i] for i in range(cfg.n_parts))
    src = np.random.default_rng(seed).integers(0, 256, size=keys * unit, dtype=np.uint8)
    cfg.move_bytes = 1
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    p = np.ascontiguousarray(preds, dtype=np.int32) if preds is not None else None
    reads = np.zeros((cfg.tokens, cfg.n_gated, cfg.n_ids), dtype=np.uint64)
    races = np.zeros(5, dtype=np.uint64)
    st = abi.load().tsb_test_dg_async_replay(C.byref(cfg), ids.ctypes.data, p.ctypes.data if p is not None else None,
                                             src.ctypes.data, seed, delay_us, mutation,
                                             reads.ctypes.data_as(C.POINTER(C.c_uint64)),
                                             races.ctypes.data_as(C.POINTER(C.c_uint64)))
    assert st == abi.SS_OK, abi.load().ss_last_error().decode()
    want = unit_sums(src, keys, unit)
    base = np.concatenate([[0], np.cumsum(n_units)])
    for t in range(cfg.tokens):
        for g in range(cfg.n_gated):
            for i in range(cfg.n_ids):
                u = int(ids[t, g, i])
                if 0 <= u < n_units[g] and reads[t, g, i]:
                    assert reads[t, g, i] == want[base[g] + u], "token %d layer %d id %d read wrong bytes" % (t, g, i)
    assert races.tolist() == [0] * 5, dict(zip(RACES, races.tolist()))
    return reads


def every_routed_read(cfg, ids, reads, held=()):
    """Every routed id of an exported layer was read (a held layer is read without an export)."""
    for t in range(cfg.tokens):
        for g in range(cfg.n_gated):
            if (t, g) in held:
                continue
            for i in range(cfg.n_ids):
                if 0 <= int(ids[t, g, i]) < cfg.n_units[g]:
                    assert reads[t, g, i] != 0, "token %d layer %d id %d: no entry when read" % (t, g, i)


@pytest.mark.parametrize("seed", range(24))
def test_two_tiers_under_concurrency(seed):
    kw = random_case(seed)
    cfg, ids, preds = make_case(**kw)
    reads = run_async(cfg, ids, preds, 7000 + seed, int(np.random.default_rng(seed).choice([0, 30, 120])))
    every_routed_read(cfg, ids, reads)


@pytest.mark.parametrize("seed", range(24))
def test_file_tier_with_reads_in_flight_under_concurrency(seed):
    kw = random_queue_case(seed)
    cfg, ids, preds = make_disk_case(**kw)
    try:
        reads = run_async(cfg, ids, preds, 8000 + seed, int(np.random.default_rng(seed).choice([0, 40, 150])))
    except AssertionError as e:
        if "capacity" in str(e).lower() or "no free slot" in str(e).lower():
            pytest.skip("a configuration the cache refuses: %s" % e)
        raise
    every_routed_read(cfg, ids, reads)


@pytest.mark.parametrize("seed", range(16))
def test_landings_and_bank_keep_under_concurrency(seed):
    """Landing blocks (predictions of file units read ahead, promoted by demands, expired by layer or TTL) and bank
    keep (bank-served file reads into the pinned blocks that become their homes), with reads landing late: every
    routed unit's bytes are its own and no hazard is seen."""
    r = np.random.default_rng(9100 + seed)
    G, U = int(r.integers(2, 6)), int(r.choice([8, 16]))
    B = int(r.choice([2, 4]))
    kw = dict(G=G, U=U, R=1, pinned=int(r.integers(0, U // 2)), D=int(r.integers(1, 3)), B=B, S=int(r.integers(2, 5)),
              Q=int(r.integers(0, G + 1)), tokens=25, s=float(r.choice([0.8, 1.2])), seed=int(r.integers(0, 1000)),
              n_pred=int(r.integers(1, B + 1)), landing_blocks=int(r.integers(1, 12)),
              landing_ttl=int(r.choice([0, 1, 3])), disk_queue=int(r.integers(2, 5)),
              bank_keep=int(r.integers(0, 3)), wb_defer=int(r.integers(0, 2)))
    cfg, ids, preds = make_disk_case(**kw)
    reads = run_async(cfg, ids, preds, 9500 + seed, int(r.choice([0, 40, 150])))
    every_routed_read(cfg, ids, reads)


@pytest.mark.parametrize("seed", range(12))
def test_every_file_tier_option_together_under_concurrency(seed):
    """Landings, bank keep, clean evict, reverts, strict admission, scoring and rounds at once, with reads in flight
    landing late: every routed unit's bytes are its own and no hazard is seen."""
    r = np.random.default_rng(9900 + seed)
    G, U = int(r.integers(3, 6)), int(r.choice([8, 16]))
    B = int(r.choice([2, 4]))
    kw = dict(G=G, U=U, R=1, pinned=int(r.integers(1, U // 2)), D=2, B=B, S=int(r.integers(2, 5)), Q=int(r.integers(1, G + 1)),
              tokens=25, s=float(r.choice([0.8, 1.2])), seed=int(r.integers(0, 1000)), n_pred=int(r.integers(1, B + 1)),
              disk_prefetch=int(r.integers(0, 2)), landing_blocks=int(r.integers(1, 8)),
              landing_ttl=int(r.choice([0, 2])), disk_queue=int(r.integers(2, 5)), bank_keep=int(r.integers(1, 3)),
              clean_evict=1, pf_revert=int(r.integers(0, 2)), pf_strict=int(r.integers(0, 2)),
              policy=int(r.integers(0, 3)), round_every=int(r.choice([0, 4])), wb_defer=int(r.integers(0, 2)))
    cfg, ids, preds = make_disk_case(**kw)
    try:
        reads = run_async(cfg, ids, preds, 9950 + seed, int(r.choice([0, 40, 150])))
    except AssertionError as e:
        if "capacity" in str(e).lower() or "no free slot" in str(e).lower():
            pytest.skip("a configuration the cache refuses: %s" % e)
        raise
    every_routed_read(cfg, ids, reads)


@pytest.mark.parametrize("reset_at", [7, 15])
def test_reset_mid_trace_under_concurrency(reset_at):
    cfg, ids, preds = make_disk_case(G=5, U=16, R=3, pinned=5, D=2, B=3, Q=12, S=3, tokens=30, s=0.9, seed=5,
                                     n_pred=2, disk_prefetch=1, disk_queue=4)
    cfg.reset_at = reset_at
    reads = run_async(cfg, ids, preds, 99, 80)
    every_routed_read(cfg, ids, reads)


def test_scored_rounds_and_policies_under_concurrency():
    cfg, ids, preds = make_disk_case(G=6, U=16, R=2, pinned=6, D=2, B=2, Q=14, S=4, tokens=40, s=1.0, seed=17,
                                     n_pred=2, disk_prefetch=1, disk_queue=3, policy=1, round_every=4, clean_evict=1,
                                     pf_revert=1)
    reads = run_async(cfg, ids, preds, 123, 100)
    every_routed_read(cfg, ids, reads)


@pytest.mark.parametrize("seed", range(16))
def test_kept_resident_layers_under_concurrency(seed):
    from test_dg_resident_replay import events
    r = np.random.default_rng(61_000 + seed)
    G, U, D = int(r.integers(2, 6)), int(r.choice([8, 16])), int(r.integers(2, 5))
    tokens = int(r.integers(15, 35))
    ev = events(G, U, seed, n=int(r.integers(1, 5)), max_ids=min(3, D), tokens=tokens)
    kw = dict(G=G, U=U, B=int(r.integers(1, 4)), R=int(r.integers(3, 5)), D=D, tokens=tokens,
              seed=int(r.integers(1, 10 ** 6)), wb_defer=int(r.integers(0, 2)), s=float(r.uniform(0.7, 1.3)),
              resident_events=ev)
    if seed % 2:
        kw.update(pinned=int(r.integers(0, U - kw["R"])), S=2, Q=D * G + 2, disk_queue=int(r.integers(1, 4)))
    else:
        kw["Q"] = D * G + 2
    cfg, ids, preds = (make_disk_case if seed % 2 else make_case)(**kw)
    try:
        reads = run_async(cfg, ids, preds, 9000 + seed, 60)
    except AssertionError as e:
        if "persistent slots" in str(e) or "capacity" in str(e).lower():
            pytest.skip("a hold the cache refuses: %s" % e)
        raise
    held, now = set(), {}
    for t in range(tokens):
        for g, ids_ in now.items():
            if ids_:
                held.add((t, g))
        for (te, g, u) in ev:
            if te == t:
                now[g] = u
    every_routed_read(cfg, ids, reads, held)


def perfect_predictions_case(k, disk):
    """Predictions that are the next layer's own routes, so every prefetch is used: the window where a prefetched
    unit's entry could be seen before its bytes, and demands that must wait for the prefetch bringing their unit."""
    if disk:
        cfg, ids, _ = make_disk_case(G=5, U=16, R=2, pinned=8, D=4, B=2, Q=24, S=3, tokens=25, s=0.8, seed=40 + k,
                                     n_pred=2, disk_prefetch=1, disk_queue=3, prefetch_per_layer=4,
                                     prefetch_per_token=40)
    else:
        cfg, ids, _ = make_case(G=5, U=16, R=2, D=4, B=2, Q=24, tokens=25, s=0.8, seed=40 + k, n_pred=2,
                                prefetch_per_layer=4, prefetch_per_token=40)
    preds = np.zeros_like(ids)
    preds[:, :-1, :] = ids[:, 1:, :]
    return cfg, ids, preds


@pytest.mark.parametrize("mutation", [1, 2])
@pytest.mark.parametrize("disk", [0, 1])
def test_planted_ordering_faults_are_caught(mutation, disk):
    """The cache's test mutations: an entry published before its unit's bytes, a demand that does not wait for the
    prefetch bringing its unit. Each is caught (wrong bytes read, a unit without an entry when read, a hazard, or a
    failed replay) in at least 3 of these 10 runs (measured: 6-8 of 10 for the first, 10 of 10 for the second; the
    faults are timing windows); the same runs without the mutation are clean."""
    caught = 0
    runs = 10
    for k in range(runs):
        cfg, ids, preds = perfect_predictions_case(k, disk)
        try:
            reads = run_async(cfg, ids, preds, 500 + k, 200, mutation)
            every_routed_read(cfg, ids, reads)
        except AssertionError:
            caught += 1
    assert caught >= 3, "mutation %d caught in %d of %d runs" % (mutation, caught, runs)
    for k in range(3):
        cfg, ids, preds = perfect_predictions_case(k, disk)
        every_routed_read(cfg, ids, run_async(cfg, ids, preds, 500 + k, 200))
