"""ZeRO-3 unit: the parameters of one module (usually a decoder block) packed into one flat
buffer that is sharded over the data-parallel group.

State per unit (the roles of the reference's ParamGroupCluster,
femtotron/sharding/param_group_cluster.py:28-418, with a B200-oriented implementation):
  flat_param_shard  bf16 [shard]   this rank's slice of the packed parameters
  master            fp32 [shard]   optimizer master; ``param_views[name]`` are its slices
  compute_views     bf16 views of flat_param_shard matching param_views (the fused AdamW
                    writes the updated bf16 values there directly)
  flat_grad_shard   fp32 [shard]   reduced gradient of this rank's slice, accumulated over
                    micro-batches

Two modes:
  * dp_size == 1 ("direct"): parameters stay permanently as views of flat_param_shard and
    their fp32 ``main_grad`` are views of flat_grad_shard, so the wgrad GEMMs accumulate
    straight into the optimizer's gradient: no gather, no scatter, no copies.
  * dp_size > 1: ``unshard`` all-gathers the packed parameters (optionally prefetched on a
    communication stream), ``reshard`` drops them; during a unit's backward the gradients
    go to a bf16 buffer that ``reduce_scatter_grads`` reduces (AVG) into flat_grad_shard on
    the communication stream.

With a symmetric heap (CUDA, dp > 1) the packed parameter shard and the bf16 gradient buffer
live in IPC-shared memory: the all-gather is copy-engine pulls of every peer's shard, and the
reduce-scatter is the native P2P kernel (publish an epoch flag to every peer after the unit's
backward; a kernel on the communication stream waits for all peers' flags, reads its slice of
every peer's buffer over NVLink and writes the fp32 shard, averaging and accumulating in the
same pass).  The reference does both with NCCL collectives
(femtotron/sharding/param_group_cluster.py:248-252, :321-324).
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from .cluster_sharding_spec import compute_cluster_layout

import os

# FT_ZERO3_DEBUG_NOCOPY=1 skips the parameter transfer of every gather (wrong numerics; used
# only to separate the cost of the transfer from the cost of its bookkeeping)
_DEBUG_NOCOPY = os.environ.get("FT_ZERO3_DEBUG_NOCOPY") == "1"
# bound of the in-kernel wait for the peers' gradient flags (a peer that late has failed)
P2P_TIMEOUT_MS = int(os.environ.get("FT_P2P_TIMEOUT_MS", "20000"))


class ParamGroupCluster:
    def __init__(self, name: str, module: nn.Module, param_groups: list, dp_group,
                 master_dtype: torch.dtype, comm_stream: torch.cuda.Stream | None = None,
                 symm=None, symm_grad=None):
        if not param_groups:
            raise ValueError(f"cluster {name}: empty param_groups")
        for pg in param_groups:
            if pg.cluster is not None:
                raise RuntimeError(f"cluster {name}: ParamGroup {pg.name} already claimed")
        if len({pg.compute.device for pg in param_groups}) != 1:
            raise ValueError(f"cluster {name}: parameters on different devices")
        self.name = name
        self.module = module
        self.param_groups = param_groups
        self.dp_group = dp_group
        self.dp_rank = dist.get_rank(dp_group) if dp_group is not None else 0
        self.dp_size = dist.get_world_size(dp_group) if dp_group is not None else 1
        self.master_dtype = master_dtype
        first = param_groups[0].compute
        self.device = first.device
        self.compute_dtype = first.dtype
        self.comm_stream = comm_stream
        self.layouts, self.shard_size, self.pad_size = compute_cluster_layout(
            [pg.compute.numel() for pg in param_groups], [pg.compute.shape for pg in param_groups],
            [pg.compute.dtype for pg in param_groups], self.dp_rank, self.dp_size,
            align=self.SYMM_ALIGN if symm is not None else 1)
        self.total_numel = sum(l.numel for l in self.layouts)
        self.padded_size = self.shard_size * self.dp_size
        self.direct = self.dp_size == 1
        # (SymmetricHeap, byte offset): flat_param_shard lives in symmetric memory and the
        # all-gather is a set of copy-engine pulls of every peer's shard (no SMs used)
        self.symm = symm
        # (gradient buffer byte offset, flag array byte offset) in the same heap: P2P
        # reduce-scatter instead of NCCL
        self.symm_grad = symm_grad if symm is not None else None
        self._rs_epoch = 0
        # reduce-scatter flavour over the symmetric gradient buffer: "ce" (copy engines pull
        # the peers' slices after a stream-side flag wait, then a local reduce kernel) or
        # "p2p" (one kernel that waits for the flags and loads the peers' slices itself)
        self.rs_mode = "ce"
        self.rs_stream = None
        # dtype of the unsharded gradient buffer the backward accumulates into (dp > 1);
        # fp32 lets the weight-gradient GEMMs accumulate through the TMA reduce-add epilogue
        # and keeps micro-batch accumulation exact; the strategy may choose bf16 to save memory
        self.grad_dtype = self.compute_dtype

        self.flat_param_shard = self._initialize_flat_param_shard()
        self.master = self.flat_param_shard.to(master_dtype)
        self.param_views: dict[str, torch.Tensor] = {}
        self.compute_views: dict[str, torch.Tensor] = {}
        for pg, l in zip(param_groups, self.layouts):
            if l.has_local_view:
                self.param_views[pg.name] = self.master.narrow(0, l.local_offset, l.local_numel).detach().requires_grad_(True)
                self.compute_views[pg.name] = self.flat_param_shard.narrow(0, l.local_offset, l.local_numel)
        self.flat_grad_shard = torch.zeros(self.shard_size, dtype=torch.float32, device=self.device)
        # dp > 1: the first reduce-scatter of a step overwrites instead of adding
        self._grad_fresh = not self.direct
        self._full_buffer: torch.Tensor | None = None
        self._prefetch: tuple[torch.Tensor, torch.cuda.Event] | None = None
        self._grad_buffer: torch.Tensor | None = None
        self.in_backward = False
        self.opt_config = dict(param_groups[0].opt_config)
        self._take_over_param_groups()

    # ------------------------------------------------------------------ construction
    def _initialize_flat_param_shard(self) -> torch.Tensor:
        full = torch.zeros(self.padded_size, dtype=self.compute_dtype, device=self.device)
        for pg, l in zip(self.param_groups, self.layouts):
            full[l.global_offset:l.global_end].copy_(pg.compute.data.reshape(-1))
        s = self.dp_rank * self.shard_size
        if self.symm is not None:
            heap, off = self.symm
            shard = heap.view(off, self.shard_size, self.compute_dtype)
            shard.copy_(full[s:s + self.shard_size])
            return shard
        return full[s:s + self.shard_size].clone()

    # shard size granularity (elements) when the unit lives in symmetric memory
    SYMM_ALIGN = 64

    @staticmethod
    def shard_numel(param_groups, dp_size: int, align: int = 1) -> int:
        total = sum(pg.compute.numel() for pg in param_groups)
        unit = dp_size * max(1, align)
        return (total + unit - 1) // unit * max(1, align)

    def _gather_into(self, buf: torch.Tensor) -> None:
        """All-gather the packed parameters into `buf` on the current stream."""
        if _DEBUG_NOCOPY:   # timing diagnostic only: bookkeeping without the transfer
            return
        if self.symm is None:
            dist.all_gather_into_tensor(buf, self.flat_param_shard, group=self.dp_group)
            return
        from femtotron_b200.ops.ext import native
        heap, off = self.symm
        nb = self.shard_size * buf.element_size()
        base = buf.data_ptr()
        native().copy_from_ptrs([base + r * nb for r in range(self.dp_size)],
                                [heap.peer_ptr(r, off) for r in range(self.dp_size)],
                                [nb] * self.dp_size)

    def _take_over_param_groups(self) -> None:
        for pg in self.param_groups:
            pg.master = None
            pg.master_spec = None
            pg.cluster = self
        if self.direct:
            for pg, l in zip(self.param_groups, self.layouts):
                pg.compute.data = self.flat_param_shard[l.global_offset:l.global_end].view(l.original_shape)
                pg.compute.main_grad = self.flat_grad_shard[l.global_offset:l.global_end].view(l.original_shape)
        else:
            for pg in self.param_groups:
                pg.compute.data = torch.empty(0, dtype=pg.compute.dtype, device=pg.compute.device)

    # ------------------------------------------------------------------ parameters
    def prefetch(self) -> None:
        """Start the all-gather of the packed parameters on the communication stream."""
        if self.direct or self._full_buffer is not None or self._prefetch is not None:
            return
        if self.comm_stream is None or not self.device.type == "cuda":
            return
        cur = torch.cuda.current_stream(self.device)
        self.comm_stream.wait_stream(cur)
        with torch.cuda.stream(self.comm_stream):
            buf = torch.empty(self.padded_size, dtype=self.compute_dtype, device=self.device)
            self._gather_into(buf)
            ev = torch.cuda.Event()
            ev.record(self.comm_stream)
        self._prefetch = (buf, ev)

    def unshard(self) -> None:
        if self.direct or self._full_buffer is not None:
            return
        from femtotron_b200.utils.comm_timing import TIMER
        if self._prefetch is not None:
            buf, ev = self._prefetch
            self._prefetch = None
            cur = torch.cuda.current_stream(self.device)
            with TIMER.wait("param_gather"):
                cur.wait_event(ev)
            buf.record_stream(cur)
        else:
            buf = torch.empty(self.padded_size, dtype=self.compute_dtype, device=self.device)
            with TIMER.wait("param_gather_inline"):
                self._gather_into(buf)
        self._full_buffer = buf
        for pg, l in zip(self.param_groups, self.layouts):
            pg.compute.data = buf[l.global_offset:l.global_end].view(l.original_shape)

    def reshard(self) -> None:
        if self.direct or self._full_buffer is None:
            return
        for pg in self.param_groups:
            pg.compute.data = torch.empty(0, dtype=pg.compute.dtype, device=pg.compute.device)
        self._full_buffer = None

    # ------------------------------------------------------------------ gradients
    def prepare_grad_buffer(self) -> None:
        """Give every parameter a bf16 ``main_grad`` view of a zeroed transient buffer
        (dp > 1) for the upcoming backward of this unit."""
        if self.direct or self._grad_buffer is not None:
            return
        if self.symm_grad is not None:
            # persistent symmetric buffer: every peer finished reading it in the previous
            # step (the optimizer step is followed by a device-side barrier)
            heap = self.symm[0]
            gb = heap.view(self.symm_grad[0], self.padded_size, self.grad_dtype)
            gb.zero_()
        else:
            gb = torch.zeros(self.padded_size, dtype=self.grad_dtype, device=self.device)
        self._grad_buffer = gb
        for pg, l in zip(self.param_groups, self.layouts):
            pg.compute.main_grad = gb[l.global_offset:l.global_end].view(l.original_shape)

    def reduce_scatter_grads(self) -> None:
        if self.direct:
            self._grad_fresh = False
            return
        gb = self._grad_buffer
        if gb is None:
            return
        self._grad_buffer = None
        for pg in self.param_groups:
            pg.compute.main_grad = None
        fresh = self._grad_fresh
        self._grad_fresh = False
        if self.symm_grad is not None:
            self._p2p_reduce_scatter(accumulate=not fresh)
            return
        use_stream = self.comm_stream is not None and self.device.type == "cuda"
        if use_stream:
            cur = torch.cuda.current_stream(self.device)
            self.comm_stream.wait_stream(cur)
            gb.record_stream(self.comm_stream)
            ctx = torch.cuda.stream(self.comm_stream)
        else:
            import contextlib
            ctx = contextlib.nullcontext()
        with ctx:
            tmp = torch.empty(self.shard_size, dtype=gb.dtype, device=self.device)
            dist.reduce_scatter_tensor(tmp, gb, op=dist.ReduceOp.AVG, group=self.dp_group)
            if fresh:
                self.flat_grad_shard.copy_(tmp)
            else:
                self.flat_grad_shard.add_(tmp.to(torch.float32))

    def _p2p_reduce_scatter(self, accumulate: bool) -> None:
        from femtotron_b200.ops.ext import error_flag, native
        C = native()
        heap = self.symm[0]
        goff, foff = self.symm_grad
        self._rs_epoch += 1
        ep = self._rs_epoch
        R, rank = self.dp_size, self.dp_rank
        flags = [heap.peer_ptr(r, foff) for r in range(R)]
        cur = torch.cuda.current_stream(self.device)
        C.p2p_publish(flags, rank, ep)          # after this unit's backward kernels
        st = self.rs_stream or self.comm_stream
        st.wait_stream(cur)
        f32 = self.grad_dtype == torch.float32
        with torch.cuda.stream(st):
            if self.rs_mode == "p2p":
                C.p2p_reduce_scatter([heap.peer_ptr(r, goff) for r in range(R)], flags[rank], flags,
                                     self.flat_grad_shard, self.shard_size, rank, ep, 1.0 / R,
                                     accumulate, error_flag(self.device), f32, P2P_TIMEOUT_MS)
                return
            nb = self.shard_size * (4 if f32 else 2)
            for r in range(R):                  # peers' flags, waited in the stream (no SMs)
                if r != rank:
                    C.stream_wait_geq(flags[rank] + 4 * r, ep)
            stage = torch.empty(R - 1, self.shard_size, dtype=self.grad_dtype, device=self.device)
            peers = [r for r in range(R) if r != rank]
            C.copy_from_ptrs([stage[i].data_ptr() for i in range(R - 1)],
                             [heap.peer_ptr(r, goff) + rank * nb for r in peers], [nb] * (R - 1))
            own = heap.peer_ptr(rank, goff) + rank * nb
            C.reduce_slices_f32([own] + [stage[i].data_ptr() for i in range(R - 1)],
                                self.flat_grad_shard, self.shard_size, 1.0 / R, accumulate, f32)

    def populate_master_grad(self) -> None:
        """Point the optimizer's views at the reduced fp32 gradient (no copy)."""
        if self._grad_fresh:
            self.flat_grad_shard.zero_()
            self._grad_fresh = False
        self.master.grad = self.flat_grad_shard
        for pg, l in zip(self.param_groups, self.layouts):
            if l.has_local_view:
                self.param_views[pg.name].grad = self.flat_grad_shard.narrow(0, l.local_offset, l.local_numel)

    def sync_master_to_compute(self) -> None:
        with torch.no_grad():
            self.flat_param_shard.copy_(self.master)

    def zero_grad(self) -> None:
        self.master.grad = None
        for v in self.param_views.values():
            v.grad = None
        if self.direct:
            self.flat_grad_shard.zero_()
            self._grad_fresh = False
        else:
            self._grad_fresh = True

    # ------------------------------------------------------------------ diagnostics
    def memory_footprint(self) -> dict:
        es = torch.tensor([], dtype=self.compute_dtype).element_size()
        return {
            "name": self.name,
            "flat_param_shard_bytes": self.shard_size * es,
            "master_bytes": self.master.numel() * self.master.element_size(),
            "flat_grad_shard_bytes": self.flat_grad_shard.numel() * 4,
            "full_buffer_bytes": (self.padded_size * es) if self._full_buffer is not None else 0,
        }

    def state_dict(self) -> dict:
        return {"master": self.master.detach().cpu(), "shard_size": self.shard_size,
                "dp_rank": self.dp_rank, "dp_size": self.dp_size,
                "names": [pg.name for pg in self.param_groups]}

    def load_state_dict(self, sd: dict) -> None:
        if sd["shard_size"] != self.shard_size or sd["dp_size"] != self.dp_size:
            raise RuntimeError(f"cluster {self.name}: shard layout mismatch")
        with torch.no_grad():
            self.master.copy_(sd["master"].to(self.master.device))
            self.flat_param_shard.copy_(self.master)
