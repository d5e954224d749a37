"""In-switch (NVLS) all-reduce over one process group of one node.

``NVLSAllReduce(group, nbytes, device)`` builds a multicast buffer of at least ``nbytes`` per
GPU (``csrc/nvls.cu``): rank 0 creates the multicast object and sends its POSIX file
descriptor to every peer over an abstract Unix socket (``socket.send_fds``), whose name the
group broadcasts; every rank adds its device, binds its own physical copy and maps a unicast
and a multicast address.  ``all_reduce_(t, average)`` copies ``t`` into the local copy, then a
bounded barrier (``multimem.red`` + a wait with a time limit), the in-switch reduction of this
rank's slice (``multimem.ld_reduce`` with fp32 accumulation, ``multimem.st`` of the result to
every copy), a second barrier, and the copy back.  Each GPU sends and receives about one copy of
the data over NVLink instead of the two of a ring all-reduce.

Used by the data-parallel gradient buckets (``parallel/data_parallel/ddp.py``) when
``FT_NVLS=1`` (the default on GPUs that support multicast); the reference all-reduces with NCCL
(femtotron/parallel/data_parallel/ddp.py:43-61).  ``close()`` tears the buffer down on every
rank together; call it before the process group is destroyed.
"""
from __future__ import annotations

import os
import socket
import uuid

import torch
import torch.distributed as dist

from femtotron_b200.ops.ext import error_flag, native

FLAG_BYTES = 256
TIMEOUT_MS = int(os.environ.get("FT_COMM_TIMEOUT_MS", "30000"))
BARRIER_CODE = 280


def nvls_available(device: torch.device) -> bool:
    if device.type != "cuda" or os.environ.get("FT_NVLS", "1") == "0":
        return False
    try:
        return bool(native().nvls_supported(device.index))
    except Exception:
        return False


def share_fd(group, fd: int | None, timeout_s: float = 120.0) -> int | None:
    """Give rank 0's open file descriptor `fd` to every other rank of `group` (one node): rank 0
    listens on an abstract Unix socket whose name the group broadcasts, and sends the
    descriptor to each peer that connects (SCM_RIGHTS via ``socket.send_fds``).  Rank 0 passes
    its descriptor and gets None back (it keeps its own); the others pass None and get their
    own duplicate, which they close when done."""
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    name = [None]
    srv = None
    if rank == 0:
        if fd is None:
            raise ValueError("share_fd: rank 0 must pass the descriptor")
        name = ["\0femtotron_fd_%d_%s" % (os.getpid(), uuid.uuid4().hex)]
        srv = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        srv.settimeout(timeout_s)
        srv.bind(name[0])
        srv.listen(max(1, world))
    dist.broadcast_object_list(name, src=dist.get_global_rank(group, 0), group=group)
    if rank == 0:
        try:
            for _ in range(world - 1):
                conn, _ = srv.accept()
                with conn:
                    socket.send_fds(conn, [b"fd"], [fd])
        finally:
            srv.close()
        return None
    s = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
    s.settimeout(timeout_s)
    try:
        s.connect(name[0])
        _, fds, _, _ = socket.recv_fds(s, 16, 1)
    finally:
        s.close()
    if len(fds) != 1:
        raise RuntimeError("share_fd: no descriptor received")
    return fds[0]


class NVLSAllReduce:
    def __init__(self, group, nbytes: int, device: torch.device):
        C = native()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device
        if not C.nvls_supported(device.index):
            raise RuntimeError("NVLS multicast is not supported on this device")
        self.size = int(C.nvls_round_size(device.index, self.world, int(nbytes) + FLAG_BYTES))
        self.data_bytes = self.size - FLAG_BYTES
        self.flag_off = self.data_bytes
        self.id = self._open(C)
        C.nvls_add_device(self.id)
        dist.barrier(group=group)
        self.uc, self.mc = C.nvls_bind_map(self.id)
        torch.cuda.synchronize(device)     # the cleared counter is in place before any barrier
        dist.barrier(group=group)
        self.buf = C.tensor_at(self.uc, self.data_bytes, torch.uint8, device.index)
        self.epoch = 0
        self.closed = False

    def _open(self, C) -> int:
        """Create (rank 0) or import (the others) the multicast object."""
        if self.rank == 0:
            hid = C.nvls_create(self.device.index, self.world, self.size)
            fd = C.nvls_export_fd(hid)
            try:
                share_fd(self.group, fd)
            finally:
                os.close(fd)
            return hid
        fd = share_fd(self.group, None)
        try:
            return C.nvls_import(self.device.index, self.world, self.size, fd)
        finally:
            os.close(fd)

    def _barrier(self) -> None:
        self.epoch += 1
        native().nvls_barrier(self.uc, self.mc, self.flag_off, self.epoch * self.world,
                              error_flag(self.device), BARRIER_CODE, TIMEOUT_MS)

    def all_reduce_(self, t: torch.Tensor, average: bool = False) -> torch.Tensor:
        """In-place sum (or mean) of `t` (fp32 or bf16, contiguous) over the group, on the
        current stream."""
        if t.dtype not in (torch.float32, torch.bfloat16) or not t.is_contiguous():
            raise ValueError("NVLS all-reduce: contiguous fp32 or bf16 tensors")
        n = t.numel() * t.element_size()
        if n > self.data_bytes:
            raise ValueError(f"NVLS all-reduce: {n} bytes exceed the buffer ({self.data_bytes})")
        nr = (n + 15) // 16 * 16
        view = self.buf[:n].view(t.dtype)
        view.copy_(t.reshape(-1))
        self._barrier()                      # every rank's contribution is in place
        native().nvls_reduce_slice(self.mc, nr, self.rank, self.world, t.dtype == torch.float32,
                                   1.0 / self.world if average else 1.0)
        self._barrier()                      # every slice's result is in every copy
        t.view(-1).copy_(view)
        return t

    def all_reduce_many_(self, ts: list, average: bool = False) -> None:
        """In-place sum (or mean) of several same-dtype tensors, packed back to back in the
        buffer (one barrier pair and one reduction for all of them)."""
        if not ts:
            return
        dt = ts[0].dtype
        if dt not in (torch.float32, torch.bfloat16) or any(t.dtype != dt for t in ts):
            raise ValueError("NVLS all-reduce: tensors of one dtype, fp32 or bf16")
        es = ts[0].element_size()
        n = sum(t.numel() for t in ts) * es
        if n > self.data_bytes:
            raise ValueError(f"NVLS all-reduce: {n} bytes exceed the buffer ({self.data_bytes})")
        flat = self.buf[:n].view(dt)
        off = 0
        for t in ts:
            flat[off:off + t.numel()].copy_(t.reshape(-1))
            off += t.numel()
        self._barrier()
        native().nvls_reduce_slice(self.mc, (n + 15) // 16 * 16, self.rank, self.world,
                                   dt == torch.float32, 1.0 / self.world if average else 1.0)
        self._barrier()
        off = 0
        for t in ts:
            t.view(-1).copy_(flat[off:off + t.numel()])
            off += t.numel()

    def close(self) -> None:
        if self.closed:
            return
        self.closed = True
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        native().nvls_close(self.id)
        dist.barrier(group=self.group)
