"""Synthetic models and route traces for the tests and the benchmark (seeded, no dataset).

Bytes: one file per model, byte i = the reference fixtures' generator (tests/fixture.hpp:16-22 there) with
file_id = the config's seed, written by libtsb_engine.so's multi-threaded filler. Layout: one packed record per unit,
the parts (gate / up / down) back to back; descriptor part p of layer L: offset = L x units x record + p-th part
offset, stride = record bytes. Routes: per (token, layer) top_k distinct ids, uniform or Zipf(s) over a per-layer
seeded permutation of the experts (P(rank r) ~ r^-s), drawn by rejection, optionally reusing the previous layer's ids
with probability rho (layer-to-layer correlation).
"""
import ctypes as C
import json
import os

import numpy as np

from . import abi


class Model:
    """A synthetic gated MoE model on disk and its descriptor."""

    def __init__(self, path, layers, units, part_bytes, seed=0, top_k=2, with_hash=False, base=0):
        self.path = path
        self.layers = int(layers)
        self.units = int(units)
        self.part_bytes = [int(b) for b in part_bytes]
        self.unit_bytes = sum(self.part_bytes)
        self.seed = int(seed)
        self.top_k = int(top_k)
        self.base = int(base)
        self.file_bytes = self.base + self.layers * self.units * self.unit_bytes
        self.with_hash = with_hash
        self._hashes = None

    def unit_offset(self, layer, unit):
        return self.base + (layer * self.units + unit) * self.unit_bytes

    def write(self, threads=None):
        """Writes the model file (skipped when a file of the right size exists)."""
        if os.path.exists(self.path) and os.path.getsize(self.path) == self.file_bytes:
            return
        eng = abi.load_engine()
        threads = threads or max(1, min(16, os.cpu_count() or 1))
        chunk = 1 << 28
        buf = np.empty(min(chunk, self.file_bytes), dtype=np.uint8)
        tmp = "%s.%d.tmp" % (self.path, os.getpid())  # (processes writing the same model each write their own)
        with open(tmp, "wb") as f:
            pos = 0
            while pos < self.file_bytes:
                n = min(chunk, self.file_bytes - pos)
                eng.tse_fill_bytes(self.seed, pos, n, buf.ctypes.data, threads)
                f.write(memoryview(buf)[:n])
                pos += n
        os.replace(tmp, self.path)

    def create_sparse(self):
        """A model file of the right size whose bytes are never read (the peer tier's stores are filled on the device
        from the same generator): a sparse file, no data written."""
        if not (os.path.exists(self.path) and os.path.getsize(self.path) == self.file_bytes):
            with open(self.path, "wb") as f:
                f.truncate(self.file_bytes)

    def unit_bytes_of(self, layer, unit):
        """The unit's engine bytes (its parts back to back) as numpy uint8."""
        out = np.empty(self.unit_bytes, dtype=np.uint8)
        abi.load_engine().tse_fill_bytes(self.seed, self.unit_offset(layer, unit), self.unit_bytes,
                                         out.ctypes.data, 4)
        return out

    def hashes(self, threads=None):
        """xxh64 of every unit (layer-major), by the library's host xxh64: from the model file when it is written (a
        pool of threads, each reading and hashing whole units; the result is kept beside the file as <path>.xxh64 and
        reused while it is newer than the file), else from the byte generator."""
        if self._hashes is not None:
            return self._hashes
        n = self.layers * self.units
        lib = abi.load()
        side = self.path + ".xxh64"
        written = os.path.exists(self.path) and os.path.getsize(self.path) == self.file_bytes
        if written and os.path.exists(side) and os.path.getsize(side) == 8 * n and \
                os.path.getmtime(side) >= os.path.getmtime(self.path):
            self._hashes = [int(x) for x in np.fromfile(side, dtype=np.uint64)]
            return self._hashes
        if not written:
            h = []
            for L in range(self.layers):
                for u in range(self.units):
                    b = self.unit_bytes_of(L, u)
                    h.append(int(lib.tsb_xxh64(b.ctypes.data, b.size, 0)))
            self._hashes = h
            return h
        from concurrent.futures import ThreadPoolExecutor
        out = np.zeros(n, dtype=np.uint64)

        def one(k):
            buf = np.empty(self.unit_bytes, dtype=np.uint8)
            with open(self.path, "rb", buffering=0) as f:
                f.seek(self.unit_offset(k // self.units, k % self.units))
                got = f.readinto(memoryview(buf))
            assert got == self.unit_bytes, "short read of %s" % self.path
            out[k] = lib.tsb_xxh64(buf.ctypes.data, buf.size, 0)

        with ThreadPoolExecutor(threads or max(1, min(16, os.cpu_count() or 1))) as ex:
            list(ex.map(one, range(n)))
        tmp = side + ".%d.tmp" % os.getpid()
        out.tofile(tmp)
        os.replace(tmp, side)
        self._hashes = [int(x) for x in out]
        return self._hashes

    def desc(self, tiers="pinned", order="ranked", engine="tsb-synth"):
        layers = []
        names = ["gate", "up", "down", "extra"]
        for L in range(self.layers):
            parts, off = [], 0
            for p, b in enumerate(self.part_bytes):
                parts.append({"name": names[p], "format": "x-synthetic", "source": 0,
                              "offset": self.base + L * self.units * self.unit_bytes + off,
                              "stride": self.unit_bytes, "bytes": b})
                off += b
            layer = {"index": L, "kind": "moe", "n_units": self.units, "top_k": self.top_k, "parts": parts}
            if self.with_hash:
                hs = self.hashes()[L * self.units:(L + 1) * self.units]
                layer["hash"] = ["%016x" % v for v in hs]
            layers.append(layer)
        return json.dumps({"schema": "strix-stream/desc-v1", "engine": engine, "unit_align": 256,
                           "sources": [{"path": self.path, "align": 4096}], "order": order, "tiers": tiers,
                           "layers": layers})


def zipf_trace(tokens, layers, units, top_k, s=1.1, seed=1, rho=0.0, uniform=False, perm_seed=None):
    """int32 [tokens][layers][top_k] routed ids (distinct within a row). perm_seed: the per-layer popularity
    permutations from that seed instead of `seed` (another sample of the same routing distribution)."""
    rng = np.random.default_rng(seed)
    perms = [rng.permutation(units) for _ in range(layers)]
    if perm_seed is not None:
        prng = np.random.default_rng(perm_seed)
        perms = [prng.permutation(units) for _ in range(layers)]
    if uniform:
        p = np.full(units, 1.0 / units)
    else:
        w = np.arange(1, units + 1, dtype=np.float64) ** (-float(s))
        p = w / w.sum()
    out = np.empty((tokens, layers, top_k), dtype=np.int32)
    for t in range(tokens):
        prev = None
        for L in range(layers):
            if prev is not None and rho > 0 and rng.random() < rho:
                out[t, L] = prev
                continue
            chosen = []
            while len(chosen) < top_k:
                r = int(rng.choice(units, p=p))
                e = int(perms[L][r])
                if e not in chosen:
                    chosen.append(e)
            out[t, L] = chosen
            prev = out[t, L].copy()
    return out


def popularity_order(layers, units, s=1.1, seed=1):
    """Per layer, expert ids from most to least popular under zipf_trace's permutation (for ranked residents)."""
    rng = np.random.default_rng(seed)
    return [list(map(int, rng.permutation(units))) for _ in range(layers)]
