"""Peer-memory all-reduce for tensor-parallel decode (``spx_ar_*`` /
``spx_op_allreduce``, csrc/k_allreduce.cu).

One communicator per rank: two data slots that the row-parallel GEMM writes
its partial sum into, and a flag array; handles are exchanged once through
torch.distributed, after which an all-reduce is a single kernel that signals
its peers, waits (bounded) for theirs and sums the slots over NVLink.  It has
no counterpart in the reference; it replaces NCCL for the small messages of
decode steps and can be captured in a CUDA graph (epochs live on the device).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import check
from .graph import DeviceTensor, Graph


def _all_gather_bytes(mine: bytes, device: int, world: int, group) -> bytes:
    import torch
    import torch.distributed as dist
    dev = torch.device("cuda", device)
    t = torch.tensor(np.frombuffer(mine, np.uint8).copy(), device=dev)
    every = torch.empty(world * len(mine), dtype=torch.uint8, device=dev)
    dist.all_gather_into_tensor(every, t, group=group)
    return every.cpu().numpy().tobytes()


class PeerAllReduce:
    def __init__(self, device: int, rank: int, world: int, max_bytes: int, group=None,
                 exchange=None):
        """`exchange(mine: bytes) -> bytes` returns every rank's handle in rank
        order; by default an all-gather over torch.distributed (`group`)."""
        self._l = _lib.lib()
        self.rank, self.world = rank, world
        self.max_bytes = int((max_bytes + 15) // 16 * 16)
        h = ctypes.c_void_p()
        check(self._l.spx_ar_create(device, rank, world, self.max_bytes, ctypes.byref(h)))
        self.h = h
        hs = int(self._l.spx_ar_handle_size())
        buf = (ctypes.c_char * hs)()
        check(self._l.spx_ar_handle(h, buf, hs))
        if exchange is None:
            exchange = lambda mine: _all_gather_bytes(mine, device, world, group)  # noqa: E731
        handles = exchange(bytes(buf))
        if len(handles) != world * hs:
            raise ValueError(f"handle exchange returned {len(handles)} bytes, "
                             f"expected {world} x {hs}")
        check(self._l.spx_ar_open(h, handles))
        self.slots = [int(self._l.spx_ar_slot(h, s)) for s in (0, 1)]

    def slot(self, s: int, shape, graph: Graph) -> DeviceTensor:
        return DeviceTensor(self.slots[s], tuple(shape), np.dtype(np.float32), graph)

    def allreduce(self, graph: Graph, slot: int, out: DeviceTensor, n: int) -> None:
        check(self._l.spx_op_allreduce(graph.h, self.h, slot, ctypes.c_void_p(out.ptr), n))

    def reset(self) -> None:
        """Zeroes this rank's flags and epochs after a timed-out all-reduce;
        every rank calls it between two barriers."""
        check(self._l.spx_ar_reset(self.h))

    def close(self) -> None:
        if self.h:
            self._l.spx_ar_destroy(self.h)
            self.h = None
