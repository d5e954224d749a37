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
    communication stream), ``reshard`` drops them; during a unit's backward the gradients go
    to an unsharded buffer that ``reduce_scatter_grads`` reduces (AVG) into flat_grad_shard.

With a symmetric heap (CUDA, dp > 1) the packed parameter shard and the unsharded gradient
buffer live in IPC-shared memory:
  * all-gather: copy-engine pulls of every peer's shard (no SM, no flag: a shard only changes
    in the optimizer step, and every step ends with a device-side barrier);
  * reduce-scatter: after the unit's last backward of the step, the compute stream writes the
    unit's epoch into every peer's flag slot for this rank (a stream memory write, no SM);
    on the reduce stream a one-warp kernel waits, with a time limit, until every peer's flag
    for the unit reached the epoch, then one kernel (``rs_adamw``) reads this rank's slice of
    every peer's buffer over NVLink, averages in fp32 and writes the fp32 gradient shard --
    and, when the optimizer allows it, applies AdamW to the shard and writes the bf16
    parameter shard in the same pass.  A peer that falls behind makes the wait give up with
    an error code (KernelTimeoutError on the host) instead of hanging.  NCCL is not called
    from the backward at all: its only use per step is the barrier at the end of the step,
    from the training loop's thread, which also tells every rank that its peers finished
    reading its gradient buffers.
The reference does both with NCCL collectives (femtotron/sharding/param_group_cluster.py:
248-252, :321-324) and the update as separate passes (mixed_precision_manager.py:318-331).
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist
from torch import nn

from .cluster_sharding_spec import compute_cluster_layout

# bound of the wait for the peers' gradient flags (a peer that late has failed)
RS_TIMEOUT_MS = int(os.environ.get("FT_COMM_TIMEOUT_MS", "30000"))
RS_WAIT_CODE = 120   # + index of the first peer whose flag is missing


class ParamGroupCluster:
    # shard size granularity (elements) when the unit lives in symmetric memory: every slice
    # of the fused reduce kernel starts on a 16-byte boundary
    SYMM_ALIGN = 64

    def __init__(self, name: str, module: nn.Module | None, param_groups: list, dp_group,
                 master_dtype: torch.dtype, comm_stream: torch.cuda.Stream | None = None,
                 symm=None, grad_offset: int | None = None, flag_offset: int | None = None):
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
        # byte offsets of the unit's unsharded gradient buffer and of its flag array (one
        # int32 per rank: the last epoch for which that rank's buffer is complete) in the heap
        self.grad_offset = grad_offset if symm is not None else None
        self.flag_offset = flag_offset if symm is not None else None
        self._rs_epoch = 0
        # stream of the reduce-scatter (and of the fused update); set by the strategy
        self.rs_stream = None
        # dtype of the unsharded gradient buffer the backward accumulates into (dp > 1);
        # fp32 lets the weight-gradient GEMMs accumulate through the TMA reduce-add epilogue
        # and keeps micro-batch accumulation exact; the strategy may choose bf16 to save memory
        self.grad_dtype = self.compute_dtype
        # kept gathered from its first use in a step until the step ends (set by the strategy)
        self.keep = False
        # optional callable(cluster) -> dict of fused-AdamW arguments for this step's update of
        # the shard, or None; installed by the mixed-precision manager
        self.early_update = None

        self.flat_param_shard = self._initialize_flat_param_shard()
        self.master = self.flat_param_shard.to(master_dtype)
        self.param_views: dict[str, torch.Tensor] = {}
        self.compute_views: dict[str, torch.Tensor] = {}
        for pg, l in zip(param_groups, self.layouts):
            if l.has_local_view:
                self.param_views[pg.name] = self.master.narrow(0, l.local_offset, l.local_numel).detach().requires_grad_(True)
                self.compute_views[pg.name] = self.flat_param_shard.narrow(0, l.local_offset, l.local_numel)
        # dp > 1: allocated on first use -- the fused reduce-scatter + AdamW never needs it
        self._flat_grad_shard: torch.Tensor | None = None
        if self.direct:
            self._flat_grad_shard = torch.zeros(self.shard_size, dtype=torch.float32, device=self.device)
        # dp > 1: the first reduce-scatter of a step overwrites instead of adding
        self._grad_fresh = not self.direct
        self._full_buffer: torch.Tensor | None = None
        self._prefetch: tuple[torch.Tensor, torch.cuda.Event] | None = None
        self._grad_buffer: torch.Tensor | None = None
        self.in_backward = False
        # the shard was updated early (fused with this step's reduce-scatter)
        self.updated_early = False
        self.opt_config = dict(param_groups[0].opt_config)
        self._take_over_param_groups()

    @property
    def flat_grad_shard(self) -> torch.Tensor:
        """fp32 gradient of this rank's shard (allocated on first use)."""
        if self._flat_grad_shard is None:
            self._flat_grad_shard = torch.zeros(self.shard_size, dtype=torch.float32, device=self.device)
        return self._flat_grad_shard

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
    def shard_numel(param_groups, dp_size: int, align: int = 1) -> int:
        total = sum(pg.compute.numel() for pg in param_groups)
        unit = dp_size * max(1, align)
        return (total + unit - 1) // unit * max(1, align)

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

    def drop_prefetch(self) -> None:
        """Forget a prefetched gather (its content is stale after the shards were rewritten)."""
        self._prefetch = None

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

    @property
    def is_gathered(self) -> bool:
        return self._full_buffer is not None

    # ------------------------------------------------------------------ gradients
    def prepare_grad_buffer(self) -> None:
        """Give every parameter a ``main_grad`` view of the unit's unsharded gradient buffer
        (dp > 1) for the upcoming backward(s) of this step."""
        if self.direct or self._grad_buffer is not None:
            return
        if self.grad_offset is not None:
            # persistent symmetric buffer: every peer finished reading it in the previous
            # step (the optimizer step ends with a device-side barrier).  No memset: the
            # first gradient write of the step stores instead of accumulating, and the
            # alignment padding is never written (zeroed at allocation).
            heap = self.symm[0]
            gb = heap.view(self.grad_offset, self.padded_size, self.grad_dtype)
            for pg in self.param_groups:
                pg.compute.grad_overwrite = True
        else:
            gb = torch.zeros(self.padded_size, dtype=self.grad_dtype, device=self.device)
        self._grad_buffer = gb
        for pg, l in zip(self.param_groups, self.layouts):
            pg.compute.main_grad = gb[l.global_offset:l.global_end].view(l.original_shape)

    def reduce_scatter_grads(self) -> None:
        if self.direct:
            self._grad_fresh = False
            if self.early_update is not None and self.device.type == "cuda":
                self._reduce_symm(None, accumulate=False)
            return
        gb = self._grad_buffer
        if gb is None:
            return
        self._grad_buffer = None
        unwritten = []
        for pg, l in zip(self.param_groups, self.layouts):
            if getattr(pg.compute, "grad_overwrite", False):
                unwritten.append(l)          # no gradient this step: its slice must read as 0
                pg.compute.grad_overwrite = False
            pg.compute.main_grad = None
        fresh = self._grad_fresh
        self._grad_fresh = False
        if self.grad_offset is not None:
            for l in unwritten:
                gb[l.global_offset:l.global_end].zero_()
            self._reduce_symm(gb, accumulate=not fresh)
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

    def _reduce_symm(self, gb, accumulate: bool) -> None:
        """Reduce-scatter over the symmetric gradient buffers (dp > 1) -- or, in direct mode,
        just the fused update of the local gradient -- on the reduce stream."""
        from femtotron_b200.ops.ext import native
        C = native()
        cur = torch.cuda.current_stream(self.device)
        st = self.rs_stream or self.comm_stream or cur
        upd = self.early_update(self) if self.early_update is not None else None
        if self.direct and upd is None:
            return      # the gradient is already complete in flat_grad_shard
        if not self.direct:
            # publish: this rank's buffer of the unit is complete for epoch ep (written into
            # every peer's flag array once the compute stream's backward kernels are done)
            self._rs_epoch += 1
            ep = self._rs_epoch
            heap = self.symm[0]
            for r in range(self.dp_size):
                C.stream_write(heap.peer_ptr(r, self.flag_offset) + 4 * self.dp_rank, ep)
        st.wait_stream(cur)
        with torch.cuda.stream(st):
            if self.direct:
                srcs, base, f32, scale = [self.flat_grad_shard.data_ptr()], 0, True, 1.0
            else:
                from femtotron_b200.ops.ext import error_flag
                local = heap.peer_ptr(self.dp_rank, self.flag_offset)
                C.wait_flags_geq([local + 4 * r for r in range(self.dp_size)], ep,
                                 error_flag(self.device), RS_TIMEOUT_MS, RS_WAIT_CODE)
                srcs = [heap.peer_ptr(r, self.grad_offset) for r in range(self.dp_size)]
                base, f32 = self.dp_rank * self.shard_size, self.grad_dtype == torch.float32
                scale = 1.0 / self.dp_size
            if upd is None:
                C.rs_adamw(srcs, base, self.shard_size, f32, scale, accumulate, self.flat_grad_shard,
                           True, None, None, None, None, None, 0.9, 0.999, 1e-8, 1)
            else:
                # the fp32 gradient shard is only written when it exists already (direct mode,
                # or an earlier reduction of this step): the update itself does not need it
                keep = self._flat_grad_shard is not None
                gs = self._flat_grad_shard if keep else self.master[:0]
                C.rs_adamw(srcs, base, self.shard_size, f32, scale, accumulate and keep, gs,
                           keep, self.master, upd["exp_avg"], upd["exp_avg_sq"], self.flat_param_shard,
                           upd["segments"], upd["beta1"], upd["beta2"], upd["eps"], upd["step"])
                self.updated_early = True

    def populate_master_grad(self) -> None:
        """Point the optimizer's views at the reduced fp32 gradient (no copy).  Nothing to do
        when the fused reduce-scatter already applied this step's update."""
        if self.updated_early:
            return
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
        self.updated_early = False
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
            "flat_grad_shard_bytes": self._flat_grad_shard.numel() * 4 if self._flat_grad_shard is not None else 0,
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
