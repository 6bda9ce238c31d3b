"""Peer-memory collectives for one-process-per-GPU jobs (the j4b_peer_* C ABI).

Each rank allocates one buffer with `j4b_peer_alloc`, the 64-byte CUDA IPC handles are exchanged
with `torch.distributed.all_gather_object`, every rank maps the others' buffers and builds a
group. The engine's collectives then move data with plain loads and stores over NVLink:
`allgather_matvec` (a row-sharded quantMatvec whose epilogue stores into every rank's buffer)
and `allreduce` (rank-ordered sum, identical on every rank).
"""
from __future__ import annotations

import ctypes

from . import _lib
from ._lib import call

GATHER_CHANNEL = 0
ALLREDUCE_CHANNEL = 1


class PeerGroup:
    def __init__(self, device: int, rank: int, world: int, nbytes: int = 1 << 30, call=call):
        """Collective over the ranks of the default process group. `call` is the C-ABI caller
        (replaceable for tests of the exchange without a GPU). The buffer holds 16 channels of
        two parity halves of 8-byte flagged words: the default 1 GiB takes a gathered output or
        an all-reduce of up to 4M floats per channel (batch 16 x 14336 rows x 8 ranks is 1.8M)."""
        import torch.distributed as dist
        if world > 8:
            raise ValueError("peer groups hold at most 8 ranks")
        self.device, self.rank, self.world, self.nbytes = device, rank, world, nbytes
        self.bases = []
        local = ctypes.c_uint64(0)
        handle = ctypes.create_string_buffer(64)
        call("j4b_peer_alloc", device, nbytes, ctypes.byref(local), handle)
        self.local = local.value
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle.raw))
        self.remote = []
        bases = (ctypes.c_uint64 * world)()
        for r in range(world):
            if r == rank:
                bases[r] = self.local
                continue
            ptr = ctypes.c_uint64(0)
            call("j4b_peer_open", device, ctypes.create_string_buffer(handles[r], 64), ctypes.byref(ptr))
            self.remote.append(ptr.value)
            bases[r] = ptr.value
        g = ctypes.c_void_p()
        call("j4b_peer_group_create", device, world, rank, bases, nbytes, ctypes.byref(g))
        self.handle = g
        self.bases = list(bases)
        dist.barrier()

    def allgather_matvec(self, w, x_ptr: int, y_all_ptr: int, batch: int, stream: int, add_ptr: int = 0):
        call("j4b_quant_matvec_allgather", ctypes.c_void_p(w.handle), x_ptr, add_ptr, y_all_ptr, batch,
             self.handle, GATHER_CHANNEL, stream)

    def allgather_matvec_host(self, w, x_host, y_all_host, batch: int, stream: int):
        """The same with host tensors (j4b_quant_matvec_allgather_host): x_host [batch, cols] and
        y_all_host [batch, rows * world], f32 CPU tensors (pinned ones are used in place)."""
        call("j4b_quant_matvec_allgather_host", ctypes.c_void_p(w.handle), x_host.data_ptr(), batch,
             y_all_host.data_ptr(), self.handle, GATHER_CHANNEL, stream)

    def allgather_matvec_host_plan(self, w, x_host, y_all_host, batch: int, stream: int):
        """allgather_matvec_host recorded once as a replayable plan (j4b_quant_matvec_host_plan);
        every rank records and runs its plans in the same order."""
        from .backend import QuantPlan
        return QuantPlan.make(w, x_host, y_all_host, batch, self.handle, GATHER_CHANNEL, stream)

    def allreduce(self, src_ptr: int, n: int, out_ptr: int, stream: int):
        call("j4b_peer_allreduce", self.handle, ALLREDUCE_CHANNEL, src_ptr, n, out_ptr, stream)

    def status(self) -> int:
        v = ctypes.c_int(0)
        call("j4b_peer_status", self.handle, ctypes.byref(v))
        return v.value

    def close(self):
        """Collective: every rank closes after the others are done with its buffer."""
        import torch
        import torch.distributed as dist
        if self.handle is None:
            return
        torch.cuda.synchronize()
        dist.barrier()
        for p in self.remote:
            _lib.load().j4b_peer_close(p)
        dist.barrier()
        _lib.load().j4b_peer_group_free(self.handle)
        _lib.load().j4b_peer_free(self.local)
        self.handle = None
