"""Peer-memory communicator of one rank (include/thvm_sm100.h sm100_peer_* /
sm100_comm_*): every GPU of the box holds one comm buffer, mapped into the
other ranks' processes through CUDA IPC; the library's kernels exchange the
decode step's partial sums and argmax candidates through them with stores
over NVLink.  torch.distributed carries only the host-side exchange of the
64-byte IPC handles at set-up."""
from __future__ import annotations

import ctypes

from . import _lib as L


class PeerComm:
    def __init__(self, rank: int, world: int, cols: int, group=None):
        import torch.distributed as dist
        self.lib, self.rank, self.world, self.dist, self.group = L.lib(), rank, world, dist, group
        nbytes = int(self.lib.sm100_comm_bytes(cols))
        if nbytes == 0:
            raise ValueError(f"comm buffer: {cols} columns")
        own, handle = ctypes.c_void_p(), (ctypes.c_char * 64)()
        L.check(self.lib.sm100_peer_alloc(nbytes, ctypes.byref(own), handle), "peer_alloc")
        self.own = own.value
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.opened = []
        ptrs = []
        for r, h in enumerate(handles):
            if r == rank:
                ptrs.append(self.own)
                continue
            p = ctypes.c_void_p()
            L.check(self.lib.sm100_peer_open(ctypes.create_string_buffer(h, 64), ctypes.byref(p)), "peer_open")
            self.opened.append(p.value)
            ptrs.append(p.value)
        L.check(self.lib.sm100_comm_set_peers(self.own, (ctypes.c_void_p * world)(*ptrs), world), "comm_set_peers")
        dist.barrier(group=group)   # every table is written before any rank's first exchange

    def allreduce_rmsnorm(self, h, g, y, rows: int, cols: int, eps: float, stream, zero_rest: bool = False):
        L.check(self.lib.sm100_comm_allreduce_rmsnorm(h, g, y, self.own, self.rank, self.world, rows, cols, eps,
                                                      int(zero_rest), stream), "comm_allreduce_rmsnorm")

    def allreduce_layernorm(self, h, g, b, y, rows: int, cols: int, eps: float, stream):
        L.check(self.lib.sm100_comm_allreduce_layernorm(h, g, b, y, self.own, self.rank, self.world, rows, cols, eps,
                                                        stream), "comm_allreduce_layernorm")

    def pick(self, val, idx, rows: int, tok, stream):
        L.check(self.lib.sm100_comm_pick(val, idx, self.own, self.rank, self.world, rows, tok, stream), "comm_pick")

    def status(self) -> int:
        return int(self.lib.sm100_comm_status())

    def close(self):
        """After every rank's last exchange: unmap the peers, free the buffer."""
        if self.own is None:
            return
        self.dist.barrier(group=self.group)
        for p in self.opened:
            self.lib.sm100_peer_close(p)
        self.dist.barrier(group=self.group)
        self.lib.sm100_peer_free(self.own)
        self.own, self.opened = None, []
