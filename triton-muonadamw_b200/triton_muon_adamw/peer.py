"""Gradient buffers every rank of the node reads directly (CUDA IPC over NVLink).

The sharded step with ``reduce_grads`` consumes un-reduced data-parallel
gradients: each rank's gradients live in one ``PeerArena`` (a device
allocation of the same size and layout on every rank), every rank maps all
the others' arenas, and the AdamW and Muon-prep kernels sum the copies of
each element they own straight from peer memory (``mad_grad_reduce``).  That
is the reduce-scatter of the gradients fused into the optimizer's first
kernels: no NCCL reduce-scatter, no reduced-gradient buffer.

Rank r's copy of the byte at address ``a`` of this rank's arena is at
``a + delta[r]``; ``delta[own rank] == 0``.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib


class _DeviceBytes:
    """``__cuda_array_interface__`` of a raw device allocation, for a zero-copy torch view."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerArena:
    """One IPC-shared device allocation per rank of ``process_group``, all mapped on every rank.

    Collective: every rank constructs it with the same ``nbytes``.  ``tensor``
    is this rank's arena as a uint8 CUDA tensor (zero-filled at allocation).
    Call :meth:`close` on every rank, after the last kernel that reads it.
    """

    def __init__(self, nbytes: int, device: torch.device, process_group):
        lib = _lib.load()
        self.pg = process_group
        self.rank = dist.get_rank(process_group)
        self.world = dist.get_world_size(process_group)
        if self.world > _lib.MAX_RANKS:
            raise ValueError(f"gradient reduction supports at most {_lib.MAX_RANKS} ranks, got {self.world}")
        self.nbytes = max(256, int(nbytes))
        with torch.cuda.device(device):
            ptr = ctypes.c_void_p()
            handle = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)()
            _lib.check(lib.mad_ipc_alloc(self.nbytes, ctypes.byref(ptr), handle), "mad_ipc_alloc")
            self.ptr = ptr.value
            mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device)
            handles = [torch.empty_like(mine) for _ in range(self.world)]
            dist.all_gather(handles, mine, group=process_group)
            self.peer_ptrs = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.peer_ptrs.append(self.ptr)
                    continue
                hb = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)(*h.cpu().tolist())
                peer = ctypes.c_void_p()
                _lib.check(lib.mad_ipc_open(hb, ctypes.byref(peer)), f"mad_ipc_open (rank {r})")
                self.peer_ptrs.append(peer.value)
        self.tensor = torch.as_tensor(_DeviceBytes(self.ptr, self.nbytes), device=device)
        self.closed = False

    def spec(self, scale: float) -> _lib.GradReduce:
        """The kernels' reduction descriptor: every rank's copy, rank order, times ``scale``."""
        red = _lib.GradReduce()
        red.n_ranks = self.world
        red.scale = scale
        for r, p in enumerate(self.peer_ptrs):
            red.delta[r] = p - self.ptr
        return red

    def close(self) -> None:
        """Unmap the peers' arenas, wait for every rank to do the same, free this rank's (collective)."""
        if self.closed:
            return
        lib = _lib.load()
        torch.cuda.synchronize()
        for r, p in enumerate(self.peer_ptrs):
            if r != self.rank:
                _lib.check(lib.mad_ipc_close(p), "mad_ipc_close")
        dist.barrier(group=self.pg)
        self.tensor = None
        _lib.check(lib.mad_ipc_free(self.ptr), "mad_ipc_free")
        self.closed = True
