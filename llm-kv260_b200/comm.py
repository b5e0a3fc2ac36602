"""Python face of include/b200_comm.h: the rank-ordered all-reduce, all-gather
and greedy candidate exchange over NVLink peer memory.

The window handles are exchanged with torch.distributed (any backend); the
data path is this library's kernels, not NCCL.
"""

from __future__ import annotations

import ctypes

from .capi import B200Error, check, lib
from .engine import dev_ptr


class OrderedAllReduce:
    """One rank's communicator (b200_comm_t)."""

    def __init__(self, rank: int, world: int, device: int, max_floats: int, group=None):
        import torch.distributed as dist
        self.rank, self.world, self.device = rank, world, device
        h = ctypes.c_void_p()
        check(lib().b200_comm_create(ctypes.byref(h), rank, world, device, max_floats), "b200_comm_create")
        self.h = h
        self.stream = 0
        nbytes = lib().b200_comm_handle_bytes()
        mine = (ctypes.c_uint8 * nbytes)()
        check(lib().b200_comm_export(self.h, mine), "b200_comm_export")
        blobs = [None] * world
        dist.all_gather_object(blobs, bytes(mine), group=group)
        allh = (ctypes.c_uint8 * (nbytes * world)).from_buffer_copy(b"".join(blobs))
        check(lib().b200_comm_import(self.h, allh), "b200_comm_import")
        if group is not None or dist.is_initialized():
            dist.barrier(group=group)

    def bind(self, engine) -> None:
        """Run the collectives on this engine's stream."""
        self.stream = engine.stream

    def allreduce_ordered(self, t) -> None:
        check(lib().b200_allreduce_sum(self.h, dev_ptr(t), t.numel(), ctypes.c_void_p(self.stream)),
              "b200_allreduce_sum")

    def allgather(self, inp, out, nbytes: int) -> None:
        check(lib().b200_allgather(self.h, dev_ptr(inp), dev_ptr(out), nbytes, ctypes.c_void_p(self.stream)),
              "b200_allgather")

    def pick(self, inp, out) -> None:
        check(lib().b200_allgather_pick(self.h, dev_ptr(inp), dev_ptr(out), ctypes.c_void_p(self.stream)),
              "b200_allgather_pick")

    def status(self) -> int:
        s = ctypes.c_uint(0)
        check(lib().b200_comm_status(self.h, ctypes.byref(s)), "b200_comm_status")
        return int(s.value)

    def close(self) -> None:
        if self.h:
            lib().b200_comm_destroy(self.h)
            self.h = None


__all__ = ["OrderedAllReduce", "B200Error"]
