"""Scored eviction's profile on the CPU: this library's SHA-256 (FIPS 180-4, written here) equals hashlib's on every
padding case; the profile identity of a descriptor's gated layers is the reference format's (sha256 of the layer
indices, unit counts, unit bytes and per-unit xxh64 lists); a well-formed TSSCPRF1 profile loads with its counts, and
each broken rule (magic, version, layer and unit counts, provenance length, size, identity, checksum) is refused with
SS_E_INVALID naming it; a descriptor without unit hashes cannot bind a profile."""
import ctypes as C
import hashlib
import json
import struct

import numpy as np
import pytest

from tierstream_b200 import abi, runtime, synth


def sha(data):
    out = (C.c_uint8 * 32)()
    buf = np.frombuffer(data, dtype=np.uint8) if data else np.zeros(1, dtype=np.uint8)
    abi.check(abi.load().tsb_test_sha256(buf.ctypes.data, len(data), out))
    return bytes(out)


def test_sha256_matches_hashlib():
    rng = np.random.default_rng(4)
    for n in list(range(0, 200)) + [1000, 4095, 4096, 65537, 1 << 20]:
        data = rng.integers(0, 256, size=n, dtype=np.uint8).tobytes()
        assert sha(data) == hashlib.sha256(data).digest(), n
    assert sha(b"abc").hex() == hashlib.sha256(b"abc").hexdigest()


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    return synth.Model(str(tmp_path_factory.mktemp("prof") / "m.bin"), layers=3, units=5, part_bytes=(256, 512),
                       seed=7, with_hash=True)


def identity_of(desc_json):
    d = json.loads(desc_json)
    gated = [l for l in d["layers"] if l.get("n_units", 0) > 0]
    b = struct.pack("<I", len(gated))
    for l in gated:
        b += struct.pack("<IIQ", l["index"], l["n_units"], sum(p["bytes"] for p in l["parts"]))
        b += b"".join(struct.pack("<Q", int(h, 16)) for h in l["hash"])
    return hashlib.sha256(b).digest(), [l["n_units"] for l in gated]


def profile_bytes(units, identity, cells, prov=b"fitted offline", version=1, magic=b"TSSCPRF1"):
    b = magic + struct.pack("<II", version, len(units)) + b"".join(struct.pack("<I", u) for u in units)
    b += identity + struct.pack("<I", len(prov)) + prov
    b += b"".join(np.asarray(c, dtype="<u4").tobytes() for c in cells)
    return b + hashlib.sha256(b).digest()


def check(desc, prof, cap=0):
    ident = (C.c_uint8 * 32)()
    cells = np.zeros(max(cap, 1), dtype=np.uint32)
    buf = np.frombuffer(prof, dtype=np.uint8) if prof else None
    st = abi.load().tsb_test_score_profile(desc.h, buf.ctypes.data if buf is not None else None,
                                           len(prof) if prof else 0, ident, cells.ctypes.data, cap)
    return st, bytes(ident), cells[:cap]


def test_identity_and_a_good_profile(model):
    text = model.desc()
    desc = runtime.Desc(text)
    want_id, units = identity_of(text)
    st, ident, _ = check(desc, None)
    assert st == abi.SS_OK and ident == want_id
    rng = np.random.default_rng(1)
    cells = [rng.integers(0, 1 << 32, size=(u, u), dtype=np.uint64).astype(np.uint32) for u in units]
    st, _, got = check(desc, profile_bytes(units, want_id, cells), cap=sum(u * u for u in units))
    assert st == abi.SS_OK
    assert np.array_equal(got, np.concatenate([c.reshape(-1) for c in cells]))


@pytest.mark.parametrize("what,mutate,msg", [
    ("magic", lambda u, i, c: profile_bytes(u, i, c, magic=b"TSSCPRF2"), b"bad magic"),
    ("version", lambda u, i, c: profile_bytes(u, i, c, version=2), b"unsupported version"),
    ("n_gated", lambda u, i, c: profile_bytes(u[:-1], i, c[:-1]), b"n_gated"),
    ("units", lambda u, i, c: profile_bytes([u[0] + 1] + u[1:], i, [np.zeros((u[0] + 1, u[0] + 1))] + c[1:]),
     b"units of gated layer 0"),
    ("provenance", lambda u, i, c: profile_bytes(u, i, c, prov=b"x" * 4097), b"provenance longer"),
    ("size", lambda u, i, c: profile_bytes(u, i, c)[:-1], b"size"),
    ("identity", lambda u, i, c: profile_bytes(u, bytes(32), c), b"identity mismatch"),
    ("checksum", lambda u, i, c: profile_bytes(u, i, c)[:-1] + b"\0", b"checksum mismatch"),
])
def test_broken_profiles_are_refused(model, what, mutate, msg):
    text = model.desc()
    desc = runtime.Desc(text)
    ident, units = identity_of(text)
    cells = [np.ones((u, u), dtype=np.uint32) for u in units]
    st, _, _ = check(desc, mutate(units, ident, cells))
    assert st == abi.SS_E_INVALID, what
    assert msg in abi.load().ss_last_error(), (what, abi.load().ss_last_error())


def test_descriptor_without_hashes_cannot_bind(tmp_path):
    m = synth.Model(str(tmp_path / "n.bin"), layers=2, units=3, part_bytes=(256,), seed=1, with_hash=False)
    st, _, _ = check(runtime.Desc(m.desc()), None)
    assert st == abi.SS_E_INVALID and b"per-unit hashes" in abi.load().ss_last_error()
