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
    go to a transient bf16 buffer that ``reduce_scatter_grads`` reduce-scatters (AVG) on the
    communication stream and adds into flat_grad_shard.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from .cluster_sharding_spec import compute_cluster_layout


class ParamGroupCluster:
    def __init__(self, name: str, module: nn.Module, param_groups: list, dp_group,
                 master_dtype: torch.dtype, comm_stream: torch.cuda.Stream | None = None,
                 symm=None):
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
            [pg.compute.dtype for pg in param_groups], self.dp_rank, self.dp_size)
        self.total_numel = sum(l.numel for l in self.layouts)
        self.padded_size = self.shard_size * self.dp_size
        self.direct = self.dp_size == 1
        # (SymmetricHeap, byte offset): flat_param_shard lives in symmetric memory and the
        # all-gather is a set of copy-engine pulls of every peer's shard (no SMs used)
        self.symm = symm

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

    @staticmethod
    def shard_numel(param_groups, dp_size: int) -> int:
        total = sum(pg.compute.numel() for pg in param_groups)
        return (total + dp_size - 1) // dp_size

    def _gather_into(self, buf: torch.Tensor) -> None:
        """All-gather the packed parameters into `buf` on the current stream."""
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
        if self._prefetch is not None:
            buf, ev = self._prefetch
            self._prefetch = None
            cur = torch.cuda.current_stream(self.device)
            cur.wait_event(ev)
            buf.record_stream(cur)
        else:
            buf = torch.empty(self.padded_size, dtype=self.compute_dtype, device=self.device)
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
        gb = torch.zeros(self.padded_size, dtype=self.compute_dtype, device=self.device)
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
