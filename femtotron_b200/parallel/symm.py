"""Symmetric device buffers over one process group (one process per GPU, one node).

Each rank allocates ``nbytes`` with cudaMalloc (native ``symm_alloc``), exports a CUDA IPC
handle, gathers every peer's handle over the group and opens it, so ``peer_ptr(r, off)`` is a
device address of rank r's buffer usable by this process's copy engines and kernels over
NVLink.  All ranks lay out the same objects at the same offsets, which is what makes the
buffer symmetric.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from femtotron_b200.ops.ext import native

_ALIGN = 256


def align(n: int, a: int = _ALIGN) -> int:
    return (n + a - 1) // a * a


class SymmetricHeap:
    def __init__(self, group, ranks, nbytes: int, device: torch.device):
        self.group = group
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        self.device = device
        self.nbytes = align(max(int(nbytes), _ALIGN))
        C = native()
        self.local = C.symm_alloc(self.nbytes, device.index)
        self._opened: list[int] = []
        handle = C.ipc_handle(self.local).tolist()
        handles = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(handles, handle, group=group)
        else:
            handles = [handle]
        self.peer_base: list[int] = []
        for r in range(self.world):
            if r == self.rank:
                self.peer_base.append(self.local.data_ptr())
            else:
                p = C.ipc_open(torch.tensor(handles[r], dtype=torch.uint8), device.index)
                self._opened.append(p)
                self.peer_base.append(p)

    def view(self, offset: int, numel: int, dtype: torch.dtype) -> torch.Tensor:
        es = torch.tensor([], dtype=dtype).element_size()
        if offset % es or offset + numel * es > self.nbytes:
            raise ValueError("symmetric view out of range or misaligned")
        return self.local[offset:offset + numel * es].view(dtype)

    def peer_ptr(self, r: int, offset: int) -> int:
        return self.peer_base[r] + offset

    def close(self) -> None:
        C = native()
        for p in self._opened:
            C.ipc_close(p)
        self._opened.clear()


class SymmetricAllocator:
    """Bump allocator laying out named regions at the same offsets on every rank."""

    def __init__(self):
        self.offsets: dict[str, int] = {}
        self.size = 0

    def reserve(self, name: str, nbytes: int) -> int:
        off = align(self.size)
        self.offsets[name] = off
        self.size = off + nbytes
        return off
