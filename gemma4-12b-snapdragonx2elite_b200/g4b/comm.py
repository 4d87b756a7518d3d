"""The tensor-parallel decode's cross-GPU reductions over NVLink peer memory,
set up through CUDA IPC: the exchange buffers of the in-chain all-reduce
(g4b_gemv_chain_create_tp) and the stand-alone one-kernel all-reduce
(g4b_allreduce_f32).

Every rank allocates one exchange buffer with the library (cudaMalloc, so the
IPC handle covers exactly that buffer), exports its handle, gathers the
others' through torch.distributed, and maps them.  The collectives are then
ordinary kernels; they are captured into CUDA graphs like any kernel.
`close()` unmaps and frees; call it before destroy_process_group.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import torch
import torch.distributed as dist

from . import _lib as L


class PeerBuffers:
    """One exchange buffer per rank (zero-filled device memory from the
    library), every rank's mapped into every process through CUDA IPC.
    `ptrs` is a device int64 tensor of the world buffer addresses (this rank's
    own at [rank]).  `close()` unmaps and frees; call it before
    destroy_process_group."""

    def __init__(self, nbytes: int, device: torch.device, group=None):
        self.lib = L.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.nbytes = int(nbytes)
        if self.nbytes <= 0:
            raise ValueError("PeerBuffers: nbytes must be positive")
        own = C.c_void_p()
        L.check("g4b_comm_alloc", self.lib.g4b_comm_alloc(self.nbytes, C.byref(own)))
        self.own = own.value
        handle = (C.c_uint8 * 64)()
        L.check("g4b_ipc_handle", self.lib.g4b_ipc_handle(self.own, handle))
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device)
        allh = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(allh, mine, group=group)
        self.opened = []
        ptrs = []
        for r, h in enumerate(allh):
            if r == self.rank:
                ptrs.append(self.own)
                continue
            hb = (C.c_uint8 * 64)(*h.cpu().tolist())
            p = C.c_void_p()
            L.check("g4b_ipc_open", self.lib.g4b_ipc_open(hb, C.byref(p)))
            self.opened.append(p.value)
            ptrs.append(p.value)
        self.ptrs = torch.tensor(ptrs, dtype=torch.int64, device=device)
        dist.barrier(group=group)

    def close(self) -> None:
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self.opened:
            self.lib.g4b_ipc_close(p)
        self.opened = []
        if self.own:
            self.lib.g4b_comm_free(self.own)
            self.own = None


class PeerAllReduce:
    def __init__(self, n: int, device: torch.device, group=None):
        self.lib = L.load()
        self.n = n
        world = dist.get_world_size(group)
        nbytes = int(self.lib.g4b_allreduce_buffer_bytes(world, n))
        if nbytes == 0:
            raise ValueError(f"PeerAllReduce: unsupported world={world} or n={n}")
        self.bufs = PeerBuffers(nbytes, device, group)
        self.world = self.bufs.world
        self.rank = self.bufs.rank
        self.ptrs = self.bufs.ptrs
        self.counter = torch.zeros(1, dtype=torch.int32, device=device)

    def __call__(self, t: torch.Tensor, out: Optional[torch.Tensor] = None,
                 stream: Optional[torch.cuda.Stream] = None, pdl: bool = False) -> torch.Tensor:
        """Sum of t over the ranks, in place unless `out` is given (f32, n elements).
        pdl: launch with programmatic dependent launch (the kernel may start
        while its predecessor runs, and lets its successor start early)."""
        if t.dtype != torch.float32 or t.numel() != self.n or not t.is_contiguous():
            raise ValueError("PeerAllReduce: f32 contiguous tensor of n elements expected")
        y = t if out is None else out
        s = stream if stream is not None else torch.cuda.current_stream(t.device)
        L.check("g4b_allreduce_f32", self.lib.g4b_allreduce_f32(
            t.data_ptr(), y.data_ptr(), self.n, self.rank, self.world, self.ptrs.data_ptr(),
            self.counter.data_ptr(), 1 if pdl else 0, s.cuda_stream))
        return y

    def close(self) -> None:
        self.bufs.close()
