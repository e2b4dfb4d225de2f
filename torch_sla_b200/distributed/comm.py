"""NCCL communicators of the row-sharded kernels.

The kernels drive NCCL themselves (grouped send/recv for the halo on a side
stream, small allreduces on the compute stream), so each process group gets
two communicators of its own -- one per stream, so their operations never
interleave differently on different ranks. The unique ids travel through
the caller's torch.distributed group. On one node the shard CG runs instead
on peer-memory exchange buffers (sla_p2p_create), which use NCCL only to
trade their IPC handles.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from .. import _lib as L

_COMMS: dict = {}
_P2P: list = []  # peer-memory handles, released (collectively) by destroy_all


class Communicators:
    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.halo = self._make()
        self.reduce = self._make()

    def _make(self):
        lib = L.lib()
        uid = (ctypes.c_ubyte * 128)()
        if self.rank == 0:
            L.check("sla_comm_unique_id", lib.sla_comm_unique_id(uid))
        obj = [bytes(uid)]
        src = dist.get_global_rank(self.group, 0) if self.group is not None else 0
        dist.broadcast_object_list(obj, src=src, group=self.group)
        raw = (ctypes.c_ubyte * 128).from_buffer_copy(obj[0])
        handle = ctypes.c_void_p()
        L.check("sla_comm_init", lib.sla_comm_init(ctypes.byref(handle), self.world, raw,
                                                   self.rank))
        return handle

    def destroy(self):
        for h in (self.halo, self.reduce):
            if h:
                L.lib().sla_comm_destroy(h)
        self.halo = self.reduce = None


def communicators(group=None) -> Communicators:
    """Per (process group, device) communicators, created on first use by
    every rank of the group together."""
    key = (id(group), torch.cuda.current_device())
    c = _COMMS.get(key)
    if c is None:
        c = Communicators(group)
        _COMMS[key] = c
    return c


def register_p2p(handle) -> None:
    _P2P.append(handle)


def destroy_all() -> None:
    """Release the peer-memory exchange buffers and the communicators, on
    every rank together (call before destroy_process_group)."""
    for h in _P2P:
        if h:
            L.lib().sla_p2p_destroy(h)
    _P2P.clear()
    for c in list(_COMMS.values()):
        c.destroy()
    _COMMS.clear()
