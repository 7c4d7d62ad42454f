"""Builds the in-tree native libraries: tierstream_b200/libtierstream.so and libtsb_engine.so (nvcc + g++ for
sm_100a, tierstream_b200/csrc/Makefile), and the checkers under oracle/ (oracle/Makefile)."""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _make(directory, extra=()):
    jobs = str(max(1, min(16, os.cpu_count() or 1)))
    subprocess.run(["make", "-j", jobs, *extra], cwd=directory, check=True)


def build(oracle=True):
    _make(os.path.join(HERE, "csrc"))
    if oracle:
        # the reference checkout beside this repository, when present, for the reference harness
        ref = os.path.normpath(os.path.join(ROOT, "..", "reference"))
        extra = ["REF=" + ref] if os.path.isdir(os.path.join(ref, "src")) else ["REF=/nonexistent"]
        _make(os.path.join(ROOT, "oracle"), extra)


if __name__ == "__main__":
    build(oracle="--no-oracle" not in sys.argv)
