"""The drop-in boundary: libtierstream.so exports every function include/*.h declares (ss_*, ts_*, ss_test_*, tsb_*),
and every versioned struct has the reference header's size and field offsets (tests/golden/abi_layout.json, generated
from the reference's include/strix_stream/ss.h by tests/golden/gen_abi_layout.py)."""
import json
import os
import re
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = ["include/strix_stream/ss.h", "include/strix_stream/ss_test.h", "include/tierstream/ts.h",
           "include/tierstream/tsb.h"]


def declared():
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", " ", open(os.path.join(ROOT, h)).read(), flags=re.S)
        for m in re.finditer(r"(?:SS|TS)_API\s+[^;(]*?\b((?:ss|ts|tsb)_\w+)\s*\(", text):
            names.add(m.group(1))
    return names


def exported():
    out = subprocess.run(["nm", "-D", "--defined-only", os.path.join(ROOT, "tierstream_b200", "libtierstream.so")],
                         capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_every_declared_function_is_exported():
    d, e = declared(), exported()
    assert len(d) > 300
    missing = sorted(d - e)
    assert not missing, "declared but not exported: %s" % missing


def test_ts_names_pair_with_ss_names():
    d = declared()
    for n in d:
        if n.startswith("ts_"):
            assert "ss_" + n[3:] in d


def test_ts_names_are_aliases_of_ss_functions(lib):
    """Every exported ts_* function is its ss_* function's own entry point (a linker alias), not a wrapper."""
    import ctypes as C
    addr = lambda n: C.cast(getattr(lib, n), C.c_void_p).value  # noqa: E731
    ts_names = sorted(n for n in exported() if n.startswith("ts_"))
    assert len(ts_names) > 150
    for n in ts_names:
        assert addr(n) == addr("ss_" + n[3:]), n


def test_generated_ts_files_are_current():
    """include/tierstream/ts.h and the alias script are what include/tierstream/gen_ts.py makes of ss.h."""
    r = subprocess.run(["python", os.path.join(ROOT, "include", "tierstream", "gen_ts.py"), "--check"],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


def test_library_loads_and_reports(lib):
    assert lib.ss_abi_version() == 1
    assert lib.tsb_cuda_arch() == 100


def _layout_with(include_dir):
    golden = json.load(open(os.path.join(ROOT, "tests", "golden", "abi_layout.json")))
    src = ['#include <stdio.h>', '#include <stddef.h>', '#include "strix_stream/ss.h"', "int main(void) {"]
    for struct, fields in golden.items():
        src.append('printf("%s __sizeof__ %%zu\\n", sizeof(%s));' % (struct, struct))
        for f in fields["fields"]:
            src.append('printf("%s %s %%zu\\n", offsetof(%s, %s));' % (struct, f, struct, f))
    src.append("return 0; }")
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "l.c")
        open(c, "w").write("\n".join(src))
        subprocess.run(["gcc", "-std=c11", "-I", include_dir, c, "-o", os.path.join(d, "l")], check=True)
        out = subprocess.run([os.path.join(d, "l")], capture_output=True, text=True, check=True).stdout
    got = {}
    for line in out.splitlines():
        s, f, v = line.split()
        got.setdefault(s, {})[f] = int(v)
    return golden, got


def test_struct_layouts_match_reference_header():
    golden, got = _layout_with(os.path.join(ROOT, "include"))
    for struct, g in golden.items():
        assert got[struct]["__sizeof__"] == g["size"], struct
        for f, off in g["fields"].items():
            assert got[struct][f] == off, "%s.%s" % (struct, f)


def test_round_defaults_and_cancel_without_a_context():
    """ss_dg_round_defaults fills the reference's defaults; ss_dg_round_cancel refuses a missing context."""
    import ctypes as C
    from tierstream_b200 import abi
    lib = abi.load()
    p = abi.ss_dg_round_params()
    lib.ss_dg_round_defaults_sized(C.byref(p), C.sizeof(p))
    assert (p.struct_size, p.flags, p.budget_bytes, p.max_units) == (C.sizeof(p), 0, 0, 96)
    assert abs(p.hysteresis - 1.25) < 1e-7 and abs(p.decay - 0.85) < 1e-7
    assert lib.ss_dg_round_cancel(None) == abi.SS_E_INVALID


def test_struct_defaults_match_the_reference(ref):
    """ss_options_defaults_sized and ss_budget_defaults_sized fill every byte as the reference's own do (its capi.cpp,
    compiled), at the full size and at a caller's older, shorter size (the tail left as the caller had it), except one
    field: ss_options.backend defaults to SS_BACKEND_CUDA here, the only backend this build has, where the reference
    defaults to its CPU backend (capi.cpp:111), so that defaults open a context on this build."""
    import ctypes as C
    import oracle
    from tierstream_b200 import abi
    lib = abi.load()
    for size_o, size_b in ((C.sizeof(abi.ss_options), C.sizeof(abi.ss_budget)), (80, 48)):
        ours_o = (C.c_uint8 * C.sizeof(abi.ss_options))(*([0xA5] * C.sizeof(abi.ss_options)))
        ours_b = (C.c_uint8 * C.sizeof(abi.ss_budget))(*([0xA5] * C.sizeof(abi.ss_budget)))
        ref_o = (C.c_uint8 * C.sizeof(abi.ss_options))(*([0xA5] * C.sizeof(abi.ss_options)))
        ref_b = (C.c_uint8 * C.sizeof(abi.ss_budget))(*([0xA5] * C.sizeof(abi.ss_budget)))
        lib.ss_options_defaults_sized(C.cast(ours_o, C.POINTER(abi.ss_options)), size_o)
        lib.ss_budget_defaults_sized(C.cast(ours_b, C.POINTER(abi.ss_budget)), size_b)
        oracle.ref().oref_defaults(C.cast(ref_o, C.c_void_p), size_o, C.cast(ref_b, C.c_void_p), size_b)
        off = abi.ss_options.backend.offset
        assert ours_o[off] == abi.SS_BACKEND_CUDA and ref_o[off] == 0  # SS_BACKEND_CPU
        ref_o[off] = abi.SS_BACKEND_CUDA
        assert bytes(ours_o) == bytes(ref_o), "ss_options defaults differ at size %d" % size_o
        assert bytes(ours_b) == bytes(ref_b), "ss_budget defaults differ at size %d" % size_b
