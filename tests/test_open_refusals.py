"""Open-time refusals of the read-ahead option, on the CPU: the host forward mode refuses readahead_units above 64
with SS_E_INVALID before any device work (src/stream_ctx.cpp:212), and the device-gated layout refuses any
read-ahead with SS_E_INVALID, as the reference's dg_layout does (src/dg_layout.cpp:194)."""
import ctypes as C
import json

import numpy as np

import oracle
from tierstream_b200 import abi, runtime

DESC = {"schema": "strix-stream/desc-v1", "engine": "t", "unit_align": 256,
        "sources": [{"path": "/nonexistent/x.bin", "align": 4096}], "order": "ranked", "tiers": "pinned|disk",
        "layers": [{"index": 0, "kind": "moe", "n_units": 4, "top_k": 1,
                    "parts": [{"name": "a", "format": "x-t", "source": 0, "offset": 0, "stride": 4096,
                               "bytes": 4096}]}]}


def budget():
    b = abi.budget_defaults()
    b.device_bytes = 1 << 30
    b.host_pinned_bytes = 1 << 30
    b.margin_gib = 1.0 / 1024
    return b


def test_host_mode_refuses_more_than_64_read_ahead_buffers():
    desc = runtime.Desc(json.dumps(DESC))
    b = budget()
    plan = runtime.Plan(desc, b, tiers=[abi.SS_TIER_DISK] * 4)
    o = abi.options_defaults()
    o.forward_mode = abi.SS_FORWARD_HOST
    o.readahead_units = 65
    h = C.c_void_p()
    assert abi.load().ss_open(desc.h, C.byref(b), plan.h, C.byref(o), C.byref(h)) == abi.SS_E_INVALID
    assert b"readahead_units must be <= 64" in abi.load().ss_last_error()


def test_device_gated_layout_refuses_read_ahead_like_the_reference(ref):
    desc_json = json.dumps(DESC)
    desc = runtime.Desc(desc_json)
    b = budget()
    b.tier_mode = abi.SS_TIER_MODE_EXCLUSIVE
    b.dynamic_slots_per_layer = 1
    b.ring_slots = 3
    b.host_spare_units = 1
    tiers = [abi.SS_TIER_RESIDENT, abi.SS_TIER_PINNED, abi.SS_TIER_PINNED, abi.SS_TIER_PINNED]
    plan = runtime.Plan(desc, b, tiers=tiers)
    o = abi.options_defaults()
    o.forward_mode = abi.SS_FORWARD_DEVICE_GATED
    o.pin_planned = 0
    o.dg_max_ids = 1
    o.readahead_units = 2
    out = np.zeros(23, dtype=np.uint64)
    res = np.zeros(16, dtype=np.uint32)
    st = abi.load().tsb_test_dg_layout(desc.h, plan.h, C.byref(o), out.ctypes.data_as(C.POINTER(C.c_uint64)), 23,
                                       res.ctypes.data, res.size)
    ours = abi.load().ss_last_error()
    t = np.asarray(tiers, dtype=np.uint8)
    err = C.create_string_buffer(512)
    raw = desc_json.encode()
    st_ref = oracle.ref().oref_dg_layout(raw, len(raw), t.ctypes.data, t.size, C.byref(b), C.byref(o),
                                         out.ctypes.data, 23, res.ctypes.data, res.size, err, 512)
    assert st == st_ref == abi.SS_E_INVALID
    assert b"readahead_units must be 0" in ours and b"readahead_units must be 0" in err.value
