"""The device-gated layout ss_open takes (slots, banks, blocks, spare and file units, staging buffers, the resolved
read depth and score weights, the residents) against the reference's own dg_layout on the same descriptor, tiers,
budget and options, on the CPU: every number is identical, or both refuse with the same status. Options this build
refuses as unsupported (window priors) are left out; host read-ahead, which both refuse with
SS_E_INVALID in this mode, is tests/test_open_refusals.py's."""
import ctypes as C
import os

import numpy as np
import pytest

import oracle
from tierstream_b200 import abi, runtime, synth

N_OUT = 27


def ours(desc_json, tiers, b, o):
    desc = runtime.Desc(desc_json)
    try:
        plan = runtime.Plan(desc, b, tiers=tiers)
    except Exception:
        return "plan", None, None
    out = np.zeros(N_OUT, dtype=np.uint64)
    res = np.zeros(4096, dtype=np.uint32)
    st = abi.load().tsb_test_dg_layout(desc.h, plan.h, C.byref(o), out.ctypes.data_as(C.POINTER(C.c_uint64)), N_OUT,
                                       res.ctypes.data, res.size)
    return st, out, res[:int(out[22])] if st == abi.SS_OK else None


def reference(desc_json, tiers, b, o):
    t = np.asarray(tiers, dtype=np.uint8)
    out = np.zeros(N_OUT, dtype=np.uint64)
    res = np.zeros(4096, dtype=np.uint32)
    err = C.create_string_buffer(512)
    raw = desc_json.encode()
    st = oracle.ref().oref_dg_layout(raw, len(raw), t.ctypes.data, t.size, C.byref(b), C.byref(o), out.ctypes.data,
                                     N_OUT, res.ctypes.data, res.size, err, 512)
    return st, out, res[:int(out[22])] if st == 0 else None, err.value


def random_case(seed, tmp):
    r = np.random.default_rng(70_000 + seed)
    G, U = int(r.integers(1, 6)), int(r.choice([2, 4, 8, 16]))
    parts = [256 * int(x) for x in r.integers(1, 9, size=int(r.integers(1, 4)))]
    m = synth.Model(os.path.join(tmp, "l%d.bin" % seed), layers=G, units=U, part_bytes=parts, seed=seed,
                    with_hash=bool(r.random() < 0.5))
    desc_json = m.desc()
    tiers = []
    disk_ok = r.random() < 0.5
    for g in range(G):
        for u in range(U):
            x = r.random()
            tiers.append(abi.SS_TIER_RESIDENT if x < 0.3 else abi.SS_TIER_DISK if (disk_ok and x > 0.75)
                         else abi.SS_TIER_PINNED)
    unit = sum(parts)
    hs = (unit + 4095) // 4096 * 4096
    b = abi.budget_defaults()
    b.tier_mode = abi.SS_TIER_MODE_EXCLUSIVE
    B = int(r.integers(1, 5))
    b.dynamic_slots_per_layer = int(r.integers(0, 4))
    b.ring_slots = 2 * B + 1 - int(r.random() < 0.1)
    b.host_spare_units = int(r.integers(0, 12))
    n_res = tiers.count(abi.SS_TIER_RESIDENT)
    b.device_bytes = (n_res + b.dynamic_slots_per_layer * G + 2 * B + 2) * unit + (64 << 20)
    b.margin_gib = 1.0 / 1024
    b.margin_fraction = 0.0
    b.host_pinned_bytes = (G * U + b.host_spare_units + 12) * hs + (64 << 20)
    o = abi.options_defaults()
    o.forward_mode = abi.SS_FORWARD_DEVICE_GATED
    o.pin_planned = 0
    o.dg_max_ids = B
    if r.random() < 0.3:
        o.dg_spare_slots = int(r.integers(0, 6))
    if r.random() < 0.3:
        o.dg_inclusive_blocks = int(r.integers(0, 6))
    if disk_ok and r.random() < 0.8:
        o.dg_disk_tier = 1
        o.dg_disk_staging = int(r.choice([0, 0, 1, 3, 9]))
        o.dg_disk_queue = int(r.choice([0, 1, 2, 5, 0xFFFFFFFF]))
        o.dg_disk_prefetch = int(r.random() < 0.5)
    if r.random() < 0.3:
        o.policy = int(r.integers(1, 3))
        if r.random() < 0.5:
            w = sorted(int(x) for x in r.integers(0, 1001, size=2))
            o.dg_score_w_trans, o.dg_score_w_freq, o.dg_score_w_recency = w[0], w[1] - w[0], 1000 - w[1]
    for f in ("dg_no_admit", "dg_clean_evict", "dg_pf_revert_unused", "dg_pf_strict_admit"):
        if r.random() < 0.15:
            setattr(o, f, 1)
    if r.random() < 0.2:
        o.dg_bank_keep = int(r.integers(1, 3))
    if r.random() < 0.15:  # (refused by both without the file tier or with a queue other than AUTO)
        o.dg_disk_queue_adapt = 1
    if r.random() < 0.2:  # landing blocks (refused by both without the file tier or with a queue of 1)
        o.dg_landing_blocks = int(r.choice([1, 4, 64, 4097]))
        if r.random() < 0.5:
            o.dg_landing_ttl = int(r.choice([0, 3, 1025]))
        if r.random() < 0.3:
            o.dg_landing_max_queued = int(r.choice([0, 2, 65]))
        if r.random() < 0.3:
            o.dg_landing_chunk = int(r.choice([0, 8192, 5000, 0xFFFFFFFF]))
    return desc_json, tiers, b, o


@pytest.mark.parametrize("seed", range(150))
def test_layout_matches_reference(ref, tmp_path, seed):
    desc_json, tiers, b, o = random_case(seed, str(tmp_path))
    st, out, res = ours(desc_json, tiers, b, o)
    if st == "plan":
        pytest.skip("the plan itself is refused")
    r_st, r_out, r_res, r_err = reference(desc_json, tiers, b, o)
    assert st == r_st, "status %d vs the reference's %d (%s): %s" % (st, r_st, r_err, abi.load().ss_last_error())
    if st == abi.SS_OK:
        assert np.array_equal(out, r_out), "layout %s vs %s" % (out.tolist(), r_out.tolist())
        assert np.array_equal(res, r_res)


def test_bank_keep_values(ref, tmp_path):
    """dg_bank_keep 0, 1 and 2 open (the same layout as the reference's); 3 is refused by both with SS_E_INVALID."""
    for seed in range(150):
        desc_json, tiers, b, o = random_case(seed, str(tmp_path))
        st, _, _ = ours(desc_json, tiers, b, o)
        if st == abi.SS_OK:
            break
    for v, want in ((0, abi.SS_OK), (1, abi.SS_OK), (2, abi.SS_OK), (3, abi.SS_E_INVALID)):
        o.dg_bank_keep = v
        st, out, _ = ours(desc_json, tiers, b, o)
        r_st, r_out, _, r_err = reference(desc_json, tiers, b, o)
        assert st == r_st == want, (v, st, r_st, r_err)
        if st == abi.SS_OK:
            assert np.array_equal(out, r_out)
    assert b"dg_bank_keep" in abi.load().ss_last_error()


def test_landing_values(ref, tmp_path):
    """Landing blocks on a file-tier case with reads in flight: every count, TTL, queue and chunk setting gives the
    reference's layout (the blocks charged to the host budget), or both refuse with the same status."""
    for seed in range(150):
        desc_json, tiers, b, o = random_case(seed, str(tmp_path))
        if abi.SS_TIER_DISK not in tiers:
            continue
        o.dg_disk_tier, o.dg_disk_queue, o.dg_disk_queue_adapt = 1, 3, 0
        o.dg_landing_blocks = o.dg_landing_ttl = o.dg_landing_max_queued = o.dg_landing_chunk = 0
        if ours(desc_json, tiers, b, o)[0] == abi.SS_OK:
            break
    seen = set()
    for blocks, ttl, queued, chunk, queue in ((1, 0, 0, 0, 3), (8, 2, 4, 8192, 3), (64, 1024, 64, 0xFFFFFFFF, 3),
                                              (4, 0, 0, 0, 1), (0, 1, 0, 0, 3), (4096, 0, 0, 4096, 3),
                                              (100000, 0, 0, 0, 3)):
        o.dg_landing_blocks, o.dg_landing_ttl, o.dg_landing_max_queued, o.dg_landing_chunk = blocks, ttl, queued, chunk
        o.dg_disk_queue = queue
        st, out, _ = ours(desc_json, tiers, b, o)
        r_st, r_out, _, r_err = reference(desc_json, tiers, b, o)
        assert st == r_st, (blocks, ttl, queued, chunk, queue, st, r_st, r_err)
        if st == abi.SS_OK:
            assert np.array_equal(out, r_out), (blocks, out.tolist(), r_out.tolist())
        seen.add(st)
    assert abi.SS_OK in seen and abi.SS_E_INVALID in seen


def test_layout_cases_are_mostly_accepted(ref, tmp_path):
    acc = 0
    for seed in range(150):
        st, _, _ = ours(*random_case(seed, str(tmp_path)))
        acc += st == abi.SS_OK
    assert acc >= 50, acc
