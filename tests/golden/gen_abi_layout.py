"""Writes tests/golden/abi_layout.json: the size and every field offset of the ABI's versioned structs, compiled
against the reference's own include/strix_stream/ss.h (run where the reference checkout exists, with its include
directory as the argument; default: ../reference/include beside this repository)."""
import json
import os
import re
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
STRUCTS = ["ss_budget", "ss_options", "ss_plan_totals", "ss_layer_stats", "ss_group", "ss_layer_view",
           "ss_exclusive_stats", "ss_snapshot_info", "ss_dg_part", "ss_dg_device_view", "ss_dg_unit",
           "ss_dg_layer_timeline", "ss_dg_boundary_timeline", "ss_dg_stats", "ss_file_identity",
           "ss_dg_round_params", "ss_dg_round_result"]


def fields_of(header, struct):
    text = re.sub(r"/\*.*?\*/", " ", open(header).read(), flags=re.S)
    m = re.search(r"typedef struct %s \{(.*?)\} %s;" % (struct, struct), text, flags=re.S)
    body = m.group(1)
    names = []
    for decl in body.split(";"):
        decl = decl.strip()
        if not decl:
            continue
        decl = re.sub(r"\[[^\]]*\]", "", decl)
        parts = decl.split(",")
        first = parts[0].split()
        names.append(first[-1].lstrip("*"))
        for p in parts[1:]:
            names.append(p.strip().lstrip("*"))
    return names


def main(include_dir):
    header = os.path.join(include_dir, "strix_stream", "ss.h")
    spec = {s: fields_of(header, s) for s in STRUCTS}
    src = ['#include <stdio.h>', '#include <stddef.h>', '#include "strix_stream/ss.h"', "int main(void) {"]
    for s, fs in spec.items():
        src.append('printf("%s __sizeof__ %%zu\\n", sizeof(%s));' % (s, s))
        for f in fs:
            src.append('printf("%s %s %%zu\\n", offsetof(%s, %s));' % (s, f, s, f))
    src.append("return 0; }")
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "l.c")
        open(c, "w").write("\n".join(src))
        subprocess.run(["gcc", "-std=c11", "-I", include_dir, c, "-o", os.path.join(d, "l")], check=True)
        out = subprocess.run([os.path.join(d, "l")], capture_output=True, text=True, check=True).stdout
    golden = {}
    for line in out.splitlines():
        s, f, v = line.split()
        g = golden.setdefault(s, {"size": 0, "fields": {}})
        if f == "__sizeof__":
            g["size"] = int(v)
        else:
            g["fields"][f] = int(v)
    json.dump(golden, open(os.path.join(HERE, "abi_layout.json"), "w"), indent=1, sort_keys=True)
    print("wrote", len(golden), "structs")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else
         os.path.join(os.path.dirname(os.path.dirname(HERE)), "..", "reference", "include"))
