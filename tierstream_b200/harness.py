"""Drives a device-gated context the way an engine does (tests, smoke and bench.py): a synthetic model on disk, its
descriptor and plan, ss_open, then per token ss_begin / one captured graph (begin, per layer export -> wait -> reader,
end) / ss_end, with the token's routed ids copied from pinned host memory into the device buffer the graph reads.
Everything that moves a byte is the library (libtierstream.so); torch only provides device memory and streams.
"""
import ctypes as C
import os

import numpy as np
import torch

from . import abi, runtime, synth


class DgSetup:
    """What DgRun opens: the descriptor, the plan (tiers: resident_keys, disk_keys, the rest pinned), the budget and the
    options, built without a device (a CPU test checks the layout they give, tsb_test_dg_layout)."""

    def __init__(self, model, residents_per_layer=None, resident_keys=None, spare_per_layer=1, max_ids=2,
                 host_spare_units=None, diag=False, test_hooks=True, wb_defer=1, wb_stream=1, verify=False,
                 timeout_ms=10000, device_bytes=None, resident_order=None, inclusive=0, disk_keys=(), disk_staging=0,
                 disk_prefetch=0, disk_queue=0, policy=0, weights=None, profile=None, bank_keep=0,
                 disk_queue_adapt=0, landing_blocks=0, landing_ttl=0):
        G, U = model.layers, model.units
        tiers = [abi.SS_TIER_PINNED] * (G * U)
        if resident_keys is None:
            resident_keys = []
            for g in range(G):
                order = resident_order[g] if resident_order else list(range(U))
                resident_keys += [g * U + e for e in order[:residents_per_layer]]
        for k in resident_keys:
            tiers[k] = abi.SS_TIER_RESIDENT
        for k in disk_keys:  # the file tier: these units live in their files only
            tiers[k] = abi.SS_TIER_DISK
        self.tiers = tiers
        self.resident_keys = list(resident_keys)
        self.disk_keys = list(disk_keys)
        b = abi.budget_defaults()
        unit = model.unit_bytes
        slots = len(resident_keys) + spare_per_layer * G + 2 * max_ids + 1
        b.device_bytes = device_bytes or (slots * unit + (4 << 30))
        b.margin_gib = 1.0 / 1024
        b.margin_fraction = 0.0
        b.tier_mode = abi.SS_TIER_MODE_EXCLUSIVE
        b.dynamic_slots_per_layer = spare_per_layer
        b.ring_slots = 2 * max_ids + 1
        b.host_spare_units = host_spare_units if host_spare_units is not None else spare_per_layer * G + inclusive
        hs = (unit + 4095) // 4096 * 4096
        b.host_pinned_bytes = (G * U - len(resident_keys) - len(self.disk_keys) + b.host_spare_units + 2 +
                               ((disk_staging or 8) + landing_blocks if self.disk_keys else 0)) * hs + (64 << 20)
        self.desc = runtime.Desc(model.desc())
        self.plan = runtime.Plan(self.desc, b, tiers=tiers)
        o = abi.options_defaults()
        o.forward_mode = abi.SS_FORWARD_DEVICE_GATED
        o.pin_planned = 0
        o.dg_max_ids = max_ids
        o.dg_test_hooks = 1 if test_hooks else 0
        o.dg_diag = 1 if diag else 0
        o.dg_wb_defer = wb_defer
        o.dg_wb_stream = wb_stream
        o.verify_hash = 1 if verify else 0
        o.dg_wait_timeout_ms = timeout_ms
        o.dg_inclusive_blocks = inclusive
        o.policy = policy  # scored eviction: SS_POLICY_SCORED / SCORED_AUTO, weights out of 1000, a profile's bytes
        if weights:
            o.dg_score_w_trans, o.dg_score_w_freq, o.dg_score_w_recency = weights
        if profile is not None:
            self._profile = C.create_string_buffer(bytes(profile), len(profile))
            o.dg_score_profile = C.addressof(self._profile)
            o.dg_score_profile_len = len(profile)
        if self.disk_keys:
            o.dg_disk_tier = 1
            o.dg_disk_staging = disk_staging
            o.dg_disk_prefetch = disk_prefetch
            o.dg_disk_queue = disk_queue
            o.dg_bank_keep = bank_keep  # bank-served file reads kept in pinned blocks (1: recency front, 2: middle)
            o.dg_disk_queue_adapt = disk_queue_adapt  # (with disk_queue SS_DG_DISK_QUEUE_AUTO)
            o.dg_landing_blocks, o.dg_landing_ttl = landing_blocks, landing_ttl  # (predictions land file units)
        self.budget, self.options = b, o


class DgRun:
    """A device-gated context and its engine stand-in's token graph. predict_prev: each layer's routed ids are also
    its prediction of the next layer's (ss_dg_enqueue_predict reads the export's own id buffer on the device: the
    predictor of traces whose layers repeat their predecessor's experts); n_pred > 0 instead predicts from ids the host
    gives each step."""

    def __init__(self, model, n_pred=0, slices=64, mode=0, with_reader=True, peer=None, max_ids=2, predict_prev=False,
                 **setup):
        self.model = model
        G, U = model.layers, model.units
        if predict_prev:
            n_pred = max_ids
        self.G, self.U, self.n_ids, self.n_pred, self.mode = G, U, max_ids, n_pred, mode
        s = DgSetup(model, max_ids=max_ids, **setup)
        self.setup = s
        self.desc, self.plan, o = s.desc, s.plan, s.options
        self.resident_keys, self.disk_keys = s.resident_keys, s.disk_keys
        o.device = torch.cuda.current_device()  # the context lives on the engine's device
        self.ctx = runtime.DgContext(self.desc, self.plan, o, peer=peer)
        self.stream = torch.cuda.Stream()
        self.ids_pin = torch.zeros(G * max_ids, dtype=torch.int32).pin_memory()
        self.ids_dev = torch.zeros(G * max_ids, dtype=torch.int32, device="cuda")
        self.pred_pin = torch.zeros(max(1, G * n_pred), dtype=torch.int32).pin_memory()
        self.pred_dev = torch.zeros(max(1, G * n_pred), dtype=torch.int32, device="cuda")
        self.out_dev = torch.zeros(G * max_ids, dtype=torch.int64, device="cuda")
        self.out_pin = torch.zeros(G * max_ids, dtype=torch.int64).pin_memory()
        self.stream.wait_stream(torch.cuda.current_stream())  # the zero fills above ran on torch's stream
        pred_ptr = (self.ids_dev if predict_prev else self.pred_dev).data_ptr() if n_pred else 0
        self.graph = runtime.TokenGraph(self.ctx, G, self.ids_dev.data_ptr(), max_ids, self.out_dev.data_ptr(),
                                        self.stream.cuda_stream, slices=slices, mode=mode, pred_dev=pred_ptr,
                                        n_pred=n_pred, with_reader=with_reader)
        self.keys = G * U
        self.graphs = {(mode, None): self.graph}
        self._graph_args = dict(slices=slices, pred_dev=pred_ptr, n_pred=n_pred, with_reader=with_reader)

    def graph_for(self, mode, held=None):
        """The token graph whose readers check in `mode` (0: positional checksum, 1: word sum), captured on first use
        on the same context, buffers and stream; held: per gated layer, held resident (not exported, read directly)."""
        key = (mode, tuple(bool(h) for h in held) if held is not None and any(held) else None)
        if key not in self.graphs:
            self.graphs[key] = runtime.TokenGraph(self.ctx, self.G, self.ids_dev.data_ptr(), self.n_ids,
                                                  self.out_dev.data_ptr(), self.stream.cuda_stream, mode=mode,
                                                  held=key[1], **self._graph_args)
        return self.graphs[key]

    def step(self, ids, preds=None, sync=True, mode=None, held=None):
        """One token: routed ids [G][max_ids] (and predictions [G][n_pred]); returns the readers' checksums (in `mode`,
        default the graph's of the open). held: the layers held by ss_dg_make_resident (their ids must be held units)."""
        graph = self.graph if mode is None and held is None else self.graph_for(self.mode if mode is None else mode,
                                                                                held)
        self.ids_pin.numpy()[:] = np.asarray(ids, dtype=np.int32).reshape(-1)
        if preds is not None:
            self.pred_pin.numpy()[:self.G * self.n_pred] = np.asarray(preds, dtype=np.int32).reshape(-1)
        self.ctx.begin()
        with torch.cuda.stream(self.stream):
            self.ids_dev.copy_(self.ids_pin, non_blocking=True)
            if preds is not None:
                self.pred_dev.copy_(self.pred_pin, non_blocking=True)
            graph.launch()
            self.out_pin.copy_(self.out_dev, non_blocking=True)
        if sync:
            self.stream.synchronize()
        self.ctx.end()
        return self.out_pin.numpy().reshape(self.G, self.n_ids).astype(np.uint64)

    def close(self):
        for g in getattr(self, "graphs", {}).values():
            g.close()
        self.graphs = {}
        if getattr(self, "graph", None):
            self.graph.close()
        if getattr(self, "ctx", None):
            self.ctx.close()


def model_dir():
    for d in ("/dev/shm", "/tmp"):
        if os.path.isdir(d) and os.access(d, os.W_OK):
            return d
    return "."


def expected_sums(model, keys, mode, slices=64):
    """The reader's checksum of each unit keys[i] (key = layer x units + unit), computed on the current device from
    the model's byte generator alone (libtsb_engine.so tse_expect_sums: no copy the runtime made is read); uint64."""
    keys = np.asarray(keys, dtype=np.int64).reshape(-1)
    out = np.zeros(keys.size, dtype=np.uint64)
    if not keys.size:
        return out
    offs = np.array([model.unit_offset(int(k) // model.units, int(k) % model.units) for k in keys], dtype=np.uint64)
    offs_dev = torch.from_numpy(offs.view(np.int64)).cuda()
    res = torch.zeros(keys.size, dtype=torch.int64, device="cuda")
    s = torch.cuda.current_stream()
    rc = abi.load_engine().tse_expect_sums(model.seed, offs_dev.data_ptr(), keys.size, model.unit_bytes, mode,
                                           res.data_ptr(), slices, s.cuda_stream)
    if rc != 0:
        raise RuntimeError("tse_expect_sums failed: %d" % rc)
    out[:] = res.cpu().numpy().view(np.uint64)
    return out


def check_reads(outs, ids, units, want):
    """Compares reader outputs outs[t][g][k] with want[key] for key = g x units + ids[t][g][k]: (units checked,
    mismatches, the first mismatch as (token, layer, k) or None)."""
    outs = np.asarray(outs, dtype=np.uint64)
    ids = np.asarray(ids, dtype=np.int64)
    keys = np.arange(ids.shape[1])[None, :, None] * units + ids
    bad = outs != want[keys]
    first = tuple(int(x) for x in np.argwhere(bad)[0]) if bad.any() else None
    return int(bad.size), int(bad.sum()), first
