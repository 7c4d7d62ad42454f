"""The descriptor parser and the planner against the reference's own (its capi.cpp, desc.cpp and plan.cpp compiled
from its sources) on the CPU: random desc-v1 descriptors (every layer kind, parts, sources, orders, tier sets, hashes,
benefits, fixed bytes, broken ones too) and budgets, through the same C ABI calls. The descriptor's status, its JSON
and every layer's units and unit bytes are equal; ss_plan_make (budget and benefits), ss_plan_from_tiers (given
tiers) and ss_plan_from_json (a plan JSON of tier letters, broken now and then) give the same status, the same tier
for every unit, the same totals and the same plan JSON."""
import ctypes as C
import json

import numpy as np
import pytest

import oracle
from tierstream_b200 import abi


def random_desc(r, broken):
    align = int(r.choice([256, 4096]))
    n_src = int(r.integers(1, 3))
    layers = []
    for i in range(int(r.integers(1, 7))):
        kind = str(r.choice(["dense", "moe", "moe", "blob"]))
        L = {"index": i, "kind": kind, "fixed_bytes": int(r.integers(0, 1 << 20))}
        if kind != "dense":
            n = 1 if kind == "blob" else int(r.integers(1, 12))
            if kind == "moe":
                L["n_units"] = n
                L["top_k"] = int(r.integers(1, n + 1))
            parts, off = [], int(r.integers(0, 4)) * 4096
            for p in range(int(r.integers(1, 4))):
                b = int(r.integers(1, 64)) * 256
                parts.append({"name": "p%d" % p, "format": "x-test", "source": int(r.integers(0, n_src)),
                              "offset": off, "stride": b, "bytes": b})
                off += b * n
            L["parts"] = parts
            if r.random() < 0.4:
                L["hash"] = ["%016x" % int(x) for x in r.integers(0, 1 << 62, size=n)]
            if r.random() < 0.3:
                L["benefit"] = [float(x) for x in r.uniform(0.1, 5.0, size=n)]
            if r.random() < 0.1:
                L["streamable"] = False
        layers.append(L)
    d = {"schema": "strix-stream/desc-v1", "engine": "t", "unit_align": align,
         "sources": [{"path": "/nonexistent/s%d.bin" % k, "align": 4096} for k in range(n_src)],
         "order": str(r.choice(["ranked", "prefix"])), "tiers": str(r.choice(["pinned", "pinned|disk", "disk"])),
         "layers": layers}
    if r.random() < 0.3:
        d["host_fixed"] = [{"name": "kv", "bytes": int(r.integers(0, 1 << 22))}]
    if r.random() < 0.3:
        d["workspace_bytes_per_row"] = int(r.integers(0, 1 << 20))
    if broken:
        what = int(r.integers(0, 6))
        if what == 0:
            d["bogus"] = 1
        elif what == 1:
            layers[0]["kind"] = "expert"
        elif what == 2:
            layers[-1]["index"] = 9
        elif what == 3:
            d["schema"] = "strix-stream/desc-v0"
        elif what == 4 and "parts" in layers[-1]:
            layers[-1]["unit_bytes"] = 7
        else:
            d["order"] = "random"
    return d


def random_budget(r, d):
    b = abi.budget_defaults()
    unit_total = sum(sum(p["bytes"] for p in L.get("parts", [])) * L.get("n_units", 1) for L in d["layers"])
    b.device_bytes = int(r.integers(0, 2 * unit_total + (8 << 20) + 1))
    b.host_pinned_bytes = int(r.integers(0, 2 * unit_total + (8 << 20) + 1))
    b.workspace_bytes = int(r.integers(0, 1 << 20))
    b.margin_gib = float(r.choice([0.0, 1.0 / 1024, 0.001]))
    b.margin_fraction = float(r.choice([0.0, 0.01, 0.03]))
    b.dynamic_slots_per_layer = int(r.integers(0, 3))
    b.ring_slots = int(r.integers(0, 6))
    b.tier_mode = int(r.integers(0, 2))
    b.pinned_backing = int(r.random() < 0.2)
    b.host_spare_units = int(r.integers(0, 8))
    return b


def ours(text, b, benefit, tiers, mode):
    lib = abi.load()
    h = C.c_void_p()
    raw = text.encode()
    st = lib.ss_desc_from_json(raw, len(raw), C.byref(h))
    if st != abi.SS_OK:
        return dict(desc_status=st)
    p, n = C.c_void_p(), C.c_size_t()
    abi.check(lib.ss_desc_to_json(h, C.byref(p), C.byref(n)))
    desc_json = abi.take_text(p, n.value)
    layers = [(lib.ss_desc_layer_units(h, l), lib.ss_desc_unit_bytes(h, l)) for l in range(lib.ss_desc_n_layers(h))]
    base = 0  # every unit's global index and the total, from the layers' units
    for l, (units, _) in enumerate(layers):
        for u in (0, units - 1, units, -1):
            assert lib.ss_desc_unit_index(h, l, u) == (base + u if 0 <= u < units else -1)
        base += units
    assert lib.ss_desc_total_units(h) == base
    assert lib.ss_desc_unit_index(h, len(layers), 0) == -1
    plan = C.c_void_p()
    if mode == 0:
        bb = (C.c_double * max(1, len(benefit)))(*benefit) if benefit is not None else None
        st = lib.ss_plan_make(h, C.byref(b), bb, len(benefit) if benefit is not None else 0, C.byref(plan))
    elif mode == 2:
        st = lib.ss_plan_from_json(h, C.byref(b), bytes(tiers), len(tiers), C.byref(plan))
    else:
        t = (C.c_uint8 * max(1, len(tiers)))(*tiers)
        st = lib.ss_plan_from_tiers(h, C.byref(b), t, len(tiers), C.byref(plan))
    out = dict(desc_status=0, desc_json=desc_json, layers=layers, plan_status=st)
    if st == abi.SS_OK:
        out["tiers"] = [lib.ss_plan_unit_tier(plan, l, u) for l in range(len(layers)) for u in range(layers[l][0])]
        tot = abi.ss_plan_totals()
        lib.ss_plan_get_totals(plan, C.byref(tot))
        out["totals"] = [getattr(tot, f) for f, _ in tot._fields_]
        abi.check(lib.ss_plan_to_json(plan, C.byref(p), C.byref(n)))
        out["plan_json"] = abi.take_text(p, n.value)
        lib.ss_plan_free(plan)
    lib.ss_desc_free(h)
    return out


def reference(text, b, benefit, tiers, mode):
    raw = text.encode()
    cap = 4096
    tiers_out = np.zeros(cap, dtype=np.uint8)
    tot = abi.ss_plan_totals()
    js = C.create_string_buffer(1 << 20)
    ds = C.create_string_buffer(1 << 20)
    lay = np.zeros(64, dtype=np.uint64)
    dst = C.c_int()
    err = C.create_string_buffer(512)
    bb = np.asarray(benefit if benefit is not None else [0.0], dtype=np.float64)
    tt = np.frombuffer(bytes(tiers), dtype=np.uint8) if mode == 2 and tiers else \
        np.asarray(tiers if tiers else [0], dtype=np.uint8)
    st = oracle.ref().oref_plan(raw, len(raw), C.byref(b), bb.ctypes.data if benefit is not None else None,
                                len(benefit) if benefit is not None else 0, tt.ctypes.data, len(tiers), mode,
                                tiers_out.ctypes.data, cap, C.byref(tot), js, len(js), ds, len(ds), lay.ctypes.data,
                                lay.size, C.byref(dst), err, 512)
    if dst.value != 0:
        return dict(desc_status=dst.value)
    out = dict(desc_status=0, desc_json=ds.value.decode(), plan_status=st)
    n_layers = len(json.loads(text)["layers"])
    out["layers"] = [(int(lay[2 * i]), int(lay[2 * i + 1])) for i in range(n_layers)]
    if st == 0:
        total = sum(u for u, _ in out["layers"])
        out["tiers"] = tiers_out[:total].tolist()
        out["totals"] = [getattr(tot, f) for f, _ in tot._fields_]
        out["plan_json"] = js.value.decode()
    return out


def plan_json(r, d):
    """A plan JSON for ss_plan_from_json: per layer one letter per unit (R P D X B); one in six broken (a wrong
    length, a bad letter, a missing layer, no "tiers")."""
    per = [L.get("n_units", 1 if L["kind"] == "blob" else 0) for L in d["layers"]]
    layers = ["".join(r.choice(list("RPPDB"), size=n)) for n in per]
    if r.random() < 1 / 6:
        what = int(r.integers(0, 4))
        if what == 0 and any(per):
            i = next(k for k, n in enumerate(per) if n)
            layers[i] = layers[i][:-1]
        elif what == 1 and any(per):
            i = next(k for k, n in enumerate(per) if n)
            layers[i] = "Q" + layers[i][1:]
        elif what == 2:
            layers = layers[:-1]
        else:
            return json.dumps({"plan": layers})
    return json.dumps({"tiers": layers})


@pytest.mark.parametrize("seed", range(200))
def test_descriptor_and_plan_match_reference(ref, seed):
    r = np.random.default_rng(80_000 + seed)
    d = random_desc(r, broken=r.random() < 0.15)
    text = json.dumps(d)
    b = random_budget(r, d)
    total = sum(L.get("n_units", 1 if L["kind"] == "blob" else 0) for L in d["layers"])
    mode = int(r.integers(0, 3))
    benefit = [float(x) for x in r.uniform(0, 3, size=total)] if (mode == 0 and r.random() < 0.5) else None
    tiers = [int(x) for x in r.choice([0, 1, 1, 2], size=total)] if mode == 1 else []
    if mode == 2:
        tiers = plan_json(r, d).encode()
    a, e = ours(text, b, benefit, tiers, mode), reference(text, b, benefit, tiers, mode)
    assert a["desc_status"] == e["desc_status"], (a, e)
    if a["desc_status"]:
        return
    assert json.loads(a["desc_json"]) == json.loads(e["desc_json"])
    assert a["layers"] == e["layers"]
    assert a["plan_status"] == e["plan_status"], (a.get("plan_status"), e.get("plan_status"))
    if a["plan_status"] == 0:
        assert a["tiers"] == e["tiers"]
        assert a["totals"] == e["totals"]
        assert json.loads(a["plan_json"]) == json.loads(e["plan_json"])
