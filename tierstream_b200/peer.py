"""The peer tier from Python (the library does the work; torch.distributed is only the plumbing between the ranks).

One process per GPU. Each rank counts its own routes per gated key; the counts are summed over the ranks by one
all-reduce (NCCL on GPUs, gloo on CPU) -- the tier's only collective; every rank then plans the same owners
(tsb_peer_plan), fills its own store from the descriptor's sources (tsb_peer_store_create), and the ranks exchange
their stores' CUDA IPC handles (an all-gather of 64-byte handles) and map each other's stores. A device-gated context
opened with the resulting Tier (runtime.DgContext(..., peer=tier)) copies each miss on an owned unit from its owner's
store: over NVLink for a peer, inside HBM for its own. With layout=abi.PEER_STRIPED every rank's store holds one
stripe of every owned unit instead (tsb_peer_store_create_striped), a miss reads a stripe from each GPU, and the
stores are checked against the descriptor's hashes once mapped (tsb_peer_tier_verify), each rank gathering its share
of the units.
"""
import ctypes as C

import numpy as np

from . import abi


def plan_owners(counts, world, cap_units=None):
    """owner[keys] from routing counts already summed over the ranks (tsb_peer_plan)."""
    counts = np.ascontiguousarray(counts, dtype=np.uint64)
    keys = counts.size
    owner = np.empty(keys, dtype=np.int32)
    cap = None
    if cap_units is not None:
        cap = np.ascontiguousarray(np.broadcast_to(np.asarray(cap_units, dtype=np.uint64), (world,)))
    abi.check(abi.load().tsb_peer_plan(counts.ctypes.data_as(C.POINTER(C.c_uint64)), keys, world,
                                       cap.ctypes.data_as(C.POINTER(C.c_uint64)) if cap is not None else None,
                                       owner.ctypes.data_as(C.POINTER(C.c_int32))))
    return owner


def store_index(owner, world):
    """(index[keys], units_per_rank[world]) of an owner map (tsb_peer_index)."""
    owner = np.ascontiguousarray(owner, dtype=np.int32)
    index = np.empty(owner.size, dtype=np.int64)
    per = np.empty(world, dtype=np.uint64)
    abi.check(abi.load().tsb_peer_index(owner.ctypes.data_as(C.POINTER(C.c_int32)), owner.size, world,
                                        index.ctypes.data_as(C.POINTER(C.c_int64)),
                                        per.ctypes.data_as(C.POINTER(C.c_uint64))))
    return index, per


def stripe_bytes(unit_bytes, world):
    """The striped layout's stripe size (tsb_peer_stripe_bytes)."""
    return int(abi.load().tsb_peer_stripe_bytes(unit_bytes, world))


def stripe_range(unit_bytes, world, r):
    """(offset, bytes) of stripe r of a unit in the striped layout."""
    s = stripe_bytes(unit_bytes, world)
    lo = r * s
    return lo, max(0, min(s, unit_bytes - lo))


class Store:
    """This rank's store: the units it owns, in its GPU's HBM (tsb_peer_store_create), or with
    layout=abi.PEER_STRIPED its stripe of every owned unit (tsb_peer_store_create_striped)."""

    def __init__(self, desc, owner, rank, device=0, verify=True, fill=True, layout=abi.PEER_WHOLE_UNITS, world=1):
        """fill = False: allocated only (tsb_peer_store_alloc); the caller writes every unit (or stripe). A striped
        store is never checked here (verify ignored): check the tier once mapped (verify_tier)."""
        owner = np.ascontiguousarray(owner, dtype=np.int32)
        self.h = C.c_void_p()
        self.layout = layout
        op = owner.ctypes.data_as(C.POINTER(C.c_int32))
        if layout == abi.PEER_STRIPED:
            abi.check(abi.load().tsb_peer_store_create_striped(desc.h, op, owner.size, rank, world, device,
                                                               1 if fill else 0, C.byref(self.h)))
        elif fill:
            abi.check(abi.load().tsb_peer_store_create(desc.h, op, owner.size, rank, device, 1 if verify else 0,
                                                       C.byref(self.h)))
        else:
            abi.check(abi.load().tsb_peer_store_alloc(desc.h, op, owner.size, rank, device, C.byref(self.h)))
        self.base = abi.load().tsb_peer_store_base(self.h) or 0
        self.bytes = int(abi.load().tsb_peer_store_bytes(self.h))

    def handle(self):
        """The store's CUDA IPC handle (64 bytes), or 64 zero bytes for an empty store."""
        if not self.base:
            return bytes(abi.PEER_HANDLE_BYTES)
        buf = (C.c_uint8 * abi.PEER_HANDLE_BYTES)()
        abi.check(abi.load().tsb_peer_store_export(self.h, buf))
        return bytes(buf)

    def migrate_from(self, old_owner, old_bases, stream):
        """Fills this store (allocated for its new owners) from where its units live now (tsb_peer_store_migrate):
        (units, units from peers, bytes)."""
        old_owner = np.ascontiguousarray(old_owner, dtype=np.int32)
        bases = (C.c_void_p * len(old_bases))(*[b or None for b in old_bases])
        u, pu, by = C.c_uint64(), C.c_uint64(), C.c_uint64()
        abi.check(abi.load().tsb_peer_store_migrate(self.h, old_owner.ctypes.data_as(C.POINTER(C.c_int32)),
                                                    C.cast(bases, C.POINTER(C.c_void_p)), old_owner.size,
                                                    len(old_bases), stream, C.byref(u), C.byref(pu), C.byref(by)))
        return u.value, pu.value, by.value

    def close(self):
        if getattr(self, "h", None):
            abi.load().tsb_peer_store_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


def read_device(ptr, nbytes):
    """nbytes of device memory at ptr (an address on the current device) as a host numpy array."""
    import torch

    class _View:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}

    return torch.as_tensor(_View(), device="cuda").cpu().numpy()


def map_store(handle, device):
    """Maps another process's store on `device`; returns its address here (0 for an empty store's handle)."""
    if not any(handle):
        return 0
    buf = (C.c_uint8 * abi.PEER_HANDLE_BYTES).from_buffer_copy(handle)
    base = C.c_void_p()
    abi.check(abi.load().tsb_peer_map(buf, device, C.byref(base)))
    return base.value or 0


def unmap_store(base):
    if base:
        abi.check(abi.load().tsb_peer_unmap(C.c_void_p(base)))


class Tier:
    """The owners and each rank's store address as seen from this process: the tsb_peer_tier of tsb_open_peer."""

    def __init__(self, world, rank, owner, bases, copy=0, layout=abi.PEER_WHOLE_UNITS):
        self.world, self.rank, self.copy, self.layout = world, rank, copy, layout
        self.owner = np.ascontiguousarray(owner, dtype=np.int32)
        self.bases = (C.c_void_p * world)(*[b or None for b in bases])

    def struct(self):
        t = abi.tsb_peer_tier()
        t.struct_size = C.sizeof(t)
        t.world, t.rank, t.keys = self.world, self.rank, self.owner.size
        t.owner = self.owner.ctypes.data_as(C.POINTER(C.c_int32))
        t.store_base = C.cast(self.bases, C.POINTER(C.c_void_p))
        t.copy = self.copy
        t.layout = self.layout
        return t


def verify_tier(desc, tier, device):
    """This rank's share of the tier checked against the descriptor's hashes (tsb_peer_tier_verify): the units
    checked; raises on a mismatch."""
    t = tier.struct()
    n = C.c_uint64()
    abi.check(abi.load().tsb_peer_tier_verify(desc.h, C.byref(t), device, C.byref(n)))
    return n.value


def all_reduce_counts(counts, dist, device=None):
    """The tier's one collective: routing counts summed over the ranks (int64 on the GPU over NCCL, CPU over gloo)."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(counts, dtype=np.int64))
    if device is not None:
        t = t.to(device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.cpu().numpy().astype(np.uint64)


def all_gather_handles(handle, dist, world, device=None):
    import torch
    mine = torch.frombuffer(bytearray(handle), dtype=torch.uint8)
    if device is not None:
        mine = mine.to(device)
    out = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(out, mine)
    return [bytes(o.cpu().numpy().tobytes()) for o in out]


class PeerSetup:
    """Everything a rank holds for the tier: its store, the mapped peer stores and the Tier to open with.
    Close it after the context that uses it."""

    def __init__(self, desc, local_counts, dist, world, rank, device, cap_units=None, verify=True, copy=0,
                 collective_device=None, filler=None, layout=abi.PEER_WHOLE_UNITS):
        """filler(store, owner): writes the rank's store itself (the store is then only allocated by the library).
        layout=abi.PEER_STRIPED: striped stores; with verify, every rank checks its share of the units once all
        stores are mapped (tsb_peer_tier_verify), before the closing barrier."""
        if dist is None:  # one rank: nothing to exchange
            assert world == 1 and rank == 0
            self.counts = np.ascontiguousarray(local_counts, dtype=np.uint64)
        else:
            self.counts = all_reduce_counts(local_counts, dist, collective_device)
        self.owner = plan_owners(self.counts, world, cap_units)
        self.layout = layout
        self.checked_units = 0
        self.store = Store(desc, self.owner, rank, device, verify, fill=filler is None, layout=layout, world=world)
        if filler is not None:
            filler(self.store, self.owner)
        handles = ([self.store.handle()] if dist is None else
                   all_gather_handles(self.store.handle(), dist, world, collective_device))
        self.mapped = []
        bases = []
        for r in range(world):
            if r == rank:
                bases.append(self.store.base)
            else:
                b = map_store(handles[r], device)
                self.mapped.append(b)
                bases.append(b)
        self.tier = Tier(world, rank, self.owner, bases, copy, layout)
        if layout == abi.PEER_STRIPED and verify:
            if dist is not None:
                dist.barrier()  # every store written before any rank gathers from it
            self.checked_units = verify_tier(desc, self.tier, device)
        if dist is not None:
            dist.barrier()

    def replan(self, desc, local_counts, dist, world, rank, device, ctx=None, cap_units=None, collective_device=None):
        """A planning round: the ranks' fresh routing counts summed (one all-reduce), the owners planned again, every
        rank's new store filled from the current stores (peers over NVLink, its own in HBM), the new stores'
        handles exchanged, and `ctx` (if given) switched to the new tier between tokens; the old stores are released
        once every rank switched. Returns {units, peer_units, bytes, seconds} of this rank's migration."""
        import time

        import torch
        counts = local_counts if dist is None else all_reduce_counts(local_counts, dist, collective_device)
        new_owner = plan_owners(counts, world, cap_units)
        if self.layout == abi.PEER_STRIPED:
            # striped stores do not depend on the owners: the same owned units keep the same stores
            if not np.array_equal(new_owner >= 0, self.owner >= 0):
                raise ValueError("a striped tier's re-plan must keep the same owned units")
            tier = Tier(world, rank, new_owner, [self.tier.bases[r] for r in range(world)], self.tier.copy,
                        self.layout)
            if ctx is not None:
                ctx.retier(tier)
            self.tier, self.owner, self.counts = tier, new_owner, counts
            return {"units": 0, "peer_units": 0, "bytes": 0, "seconds": 0.0}
        old_owner, old_bases = self.owner, [self.tier.bases[r] for r in range(world)]
        store = Store(desc, new_owner, rank, device, verify=False, fill=False)
        s = torch.cuda.Stream(device=device)
        t0 = time.perf_counter()
        units, peer_units, nbytes = store.migrate_from(old_owner, old_bases, s.cuda_stream)
        seconds = time.perf_counter() - t0
        if dist is not None:
            dist.barrier()  # every rank is done reading the old stores
        handles = ([store.handle()] if dist is None else
                   all_gather_handles(store.handle(), dist, world, collective_device))
        mapped, bases = [], []
        for r in range(world):
            if r == rank:
                bases.append(store.base)
            else:
                b = map_store(handles[r], device)
                mapped.append(b)
                bases.append(b)
        tier = Tier(world, rank, new_owner, bases, self.tier.copy)
        if ctx is not None:
            ctx.retier(tier)
        if dist is not None:
            dist.barrier()  # every context reads the new stores only
        self.close()
        self.store, self.mapped, self.tier, self.owner, self.counts = store, mapped, tier, new_owner, counts
        return {"units": units, "peer_units": peer_units, "bytes": nbytes, "seconds": seconds}

    def close(self):
        for b in getattr(self, "mapped", []):
            unmap_store(b)
        self.mapped = []
        if getattr(self, "store", None):
            self.store.close()
            self.store = None
