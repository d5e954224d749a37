"""ZeRO-3: parameters, gradients and optimizer state sharded over data parallelism.

Units are chosen by a wrap policy (default: one per decoder block).  Each unit becomes a
ParamGroupCluster and gets four module hooks (as in the reference,
femtotron/sharding/zero3.py:191-226), with these B200-specific behaviours:
  * forward-pre: unshard (consume the prefetched all-gather) and prefetch the NEXT unit on
    the communication stream, so the gather overlaps the current unit's compute;
  * forward-post: reshard — except during an activation-checkpoint recompute inside the
    backward, where the parameters must stay until the unit's backward is done;
  * backward-pre: unshard, allocate the transient gradient buffer, prefetch the PREVIOUS
    unit;
  * backward-post: reduce-scatter the unit's gradients on the communication stream
    (skipped under ``no_sync``), then reshard.
Parameters outside every unit (embedding, final norm, lm_head) keep unsharded fp32 masters
and are all-reduced (AVG) at step time, like the reference.
With dp_size == 1 the clusters run in direct mode (no hooks, no copies).
"""
from __future__ import annotations

import os
from contextlib import contextmanager

import torch
import torch.distributed as dist
from torch import nn

from .param_group_cluster import ParamGroupCluster


class ZeRO3Strategy:
    def __init__(self, dp_group, wrap_policy, prefetch: bool = True, symmetric: bool | None = None):
        self.dp_group = dp_group
        self.dp_rank = dist.get_rank(dp_group) if dp_group is not None else 0
        self.dp_size = dist.get_world_size(dp_group) if dp_group is not None else 1
        self.wrap_policy = wrap_policy
        self.prefetch_enabled = prefetch
        self.clusters: list[ParamGroupCluster] = []
        self._hook_handles: list = []
        self._sync_enabled = True
        self.comm_stream = None
        # all-gather through copy engines from symmetric (IPC-shared) shards and a reduce-scatter
        # over symmetric gradient buffers; default on for CUDA with dp > 1 (FT_ZERO3_SYMM=0
        # selects NCCL for both; FT_ZERO3_RS=ce|p2p|nccl picks the reduce-scatter flavour)
        env = os.environ.get("FT_ZERO3_SYMM")
        self.symmetric = symmetric if symmetric is not None else (env != "0")
        self.heap = None
        self._barrier_t = None
        # bounded host run-ahead: before issuing a gather, the host waits for the gather
        # issued `runahead` units earlier to finish, which caps the number of in-flight
        # full-parameter and gradient buffers (their memory is pinned by cross-stream use)
        self.runahead = int(os.environ.get("FT_ZERO3_RUNAHEAD", "3"))
        self._inflight: list = []
        self.ar_stream = None
        self.rs_stream = None
        # keep every unit gathered from its first use in a step until the step ends (trades
        # one full bf16 copy of the unit parameters for 2*grad_accum-1 fewer gathers per
        # unit and step); off by default: ZeRO-3 reshards after every use
        self.keep_in_step = os.environ.get("FT_ZERO3_KEEP_IN_STEP") == "1"
        self._early_reduced: set[int] = set()

    def make_master(self, compute: nn.Parameter, master_dtype: torch.dtype):
        master = compute.detach().clone().to(master_dtype)
        master.requires_grad_(True)
        return master, None

    def make_clusters(self, model: nn.Module, groups: list, master_dtype):
        if master_dtype is None:
            raise ValueError("ZeRO-3 requires a master_dtype (the optimizer state to shard)")
        units = [m for m in model.modules() if self.wrap_policy(m)]
        if not units:
            raise RuntimeError("ZeRO-3 wrap_policy matched no module")
        ids = {id(u) for u in units}
        for u in units:
            for sub in u.modules():
                if sub is not u and id(sub) in ids:
                    raise RuntimeError(f"nested ZeRO-3 units: {type(sub).__name__} inside {type(u).__name__}")
        by_id = {id(pg.compute): pg for pg in groups}
        dev = groups[0].compute.device if groups else torch.device("cpu")
        if dev.type == "cuda" and self.dp_size > 1:
            self.comm_stream = torch.cuda.Stream(device=dev)
        names = {m: n for n, m in model.named_modules()}
        unit_pgs = []
        for u in units:
            pgs, seen = [], set()
            for p in u.parameters():
                if id(p) in seen:
                    continue
                seen.add(id(p))
                pg = by_id.get(id(p))
                if pg is None:
                    continue
                if pg.cluster is not None:
                    raise RuntimeError(f"parameter {pg.name} claimed by two units")
                pgs.append(pg)
            if pgs:
                unit_pgs.append((u, pgs))
        use_symm = self.symmetric and dev.type == "cuda" and self.dp_size > 1
        rs_mode = os.environ.get("FT_ZERO3_RS", "ce")   # ce | p2p | nccl
        use_p2p_rs = use_symm and rs_mode in ("ce", "p2p")
        grad_dtype = self._pick_grad_dtype(unit_pgs, dev)
        offsets, grad_offsets = [], []
        if use_symm:
            from femtotron_b200.parallel.symm import SymmetricAllocator, SymmetricHeap
            alloc = SymmetricAllocator()
            es = groups[0].compute.element_size()
            al = ParamGroupCluster.SYMM_ALIGN
            for i, (u, pgs) in enumerate(unit_pgs):
                shard = ParamGroupCluster.shard_numel(pgs, self.dp_size, al)
                offsets.append(alloc.reserve(f"unit{i}", shard * es))
                if use_p2p_rs:
                    # bf16 gradient buffer of the whole unit + one flag per rank
                    ges = torch.tensor([], dtype=grad_dtype).element_size()
                    grad_offsets.append((alloc.reserve(f"grad{i}", shard * self.dp_size * ges),
                                         alloc.reserve(f"flags{i}", 4 * self.dp_size)))
            self.heap = SymmetricHeap(self.dp_group, None, alloc.size, dev)
            self._barrier_t = torch.zeros(1, device=dev)
        for i, (u, pgs) in enumerate(unit_pgs):
            c = ParamGroupCluster(names.get(u, type(u).__name__) or "<root>", u, pgs, self.dp_group,
                                  master_dtype, comm_stream=self.comm_stream,
                                  symm=(self.heap, offsets[i]) if use_symm else None,
                                  symm_grad=grad_offsets[i] if use_p2p_rs else None)
            self.clusters.append(c)
        for c in self.clusters:
            c.grad_dtype = grad_dtype
        if use_p2p_rs:
            self.rs_stream = torch.cuda.Stream(device=dev)
            for c in self.clusters:
                c.rs_mode = rs_mode
                c.rs_stream = self.rs_stream
        for i, c in enumerate(self.clusters):
            c.index = i
            if not c.direct:
                self._install_hooks(c)
        # free (non-unit) parameters accumulate an fp32 gradient in place; with dp > 1 on CUDA
        # their all-reduce starts on a side stream as soon as the last micro-batch's backward
        # has produced the gradient (lm_head and the final norm come first in the backward)
        for pg in groups:
            if pg.cluster is None and pg.compute.requires_grad:
                pg.compute.main_grad = torch.zeros(pg.compute.shape, dtype=torch.float32,
                                                   device=pg.compute.device)
                if self.comm_stream is not None:
                    pg.compute._ft_grad_ready = (lambda p=pg.compute: self._free_grad_ready(p))
        if self.comm_stream is not None:
            self.ar_stream = torch.cuda.Stream(device=dev)
        self.shards_written()
        return self.clusters

    def shards_written(self) -> None:
        """Call after this rank wrote its parameter shards into symmetric memory (construction,
        checkpoint load): peers' copy engines read those shards directly, so every rank's
        writes must be complete before any rank gathers."""
        if self.heap is not None:
            torch.cuda.synchronize(self.heap.device)
            dist.barrier(group=self.dp_group)

    def _pick_grad_dtype(self, unit_pgs, dev) -> torch.dtype:
        """fp32 unsharded gradient buffers when they fit comfortably (they are persistent when
        they live in symmetric memory), else the compute dtype.  FT_ZERO3_GRAD_DTYPE=fp32|bf16
        forces the choice."""
        first = unit_pgs[0][1][0].compute.dtype
        env = os.environ.get("FT_ZERO3_GRAD_DTYPE", "auto")
        if env == "fp32":
            return torch.float32
        if env == "bf16" or dev.type != "cuda" or self.dp_size == 1:
            return first
        total = sum(pg.compute.numel() for _, pgs in unit_pgs for pg in pgs)
        cap = torch.cuda.get_device_properties(dev).total_memory
        return torch.float32 if total * 4 <= 0.25 * cap else first

    def _free_grad_ready(self, p) -> None:
        if not self._sync_enabled:
            return
        mg = p.main_grad
        cur = torch.cuda.current_stream(mg.device)
        self.ar_stream.wait_stream(cur)
        with torch.cuda.stream(self.ar_stream):
            dist.all_reduce(mg, op=dist.ReduceOp.AVG, group=self.dp_group)
        self._early_reduced.add(id(mg))

    # ------------------------------------------------------------------ hooks
    def _install_hooks(self, c: ParamGroupCluster) -> None:
        m = c.module
        self._hook_handles += [
            m.register_forward_pre_hook(lambda mod, args, c=c: self._pre_forward(c)),
            m.register_forward_hook(lambda mod, args, out, c=c: self._post_forward(c)),
            m.register_full_backward_pre_hook(lambda mod, go, c=c: self._pre_backward(c)),
            m.register_full_backward_hook(lambda mod, gi, go, c=c: self._post_backward(c)),
        ]

    def _neighbor(self, c, step):
        j = c.index + step
        return self.clusters[j] if 0 <= j < len(self.clusters) else None

    def _throttle(self) -> None:
        if self.comm_stream is None or self.runahead <= 0:
            return
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.comm_stream.device))
        self._inflight.append(ev)
        while len(self._inflight) > self.runahead:
            self._inflight.pop(0).synchronize()

    def _pre_forward(self, c):
        self._throttle()
        c.unshard()
        if self.prefetch_enabled and not c.in_backward:
            n = self._neighbor(c, +1)
            if n is not None:
                n.prefetch()

    def _post_forward(self, c):
        if c.in_backward or (self.keep_in_step and torch.is_grad_enabled()):
            return
        # the last unit's backward comes right after the forward: keep it gathered
        if c.index == len(self.clusters) - 1 and torch.is_grad_enabled():
            return
        c.reshard()

    def _pre_backward(self, c):
        self._throttle()
        c.in_backward = True
        c.unshard()
        c.prepare_grad_buffer()
        if self.prefetch_enabled:
            n = self._neighbor(c, -1)
            if n is not None:
                n.prefetch()

    def _post_backward(self, c):
        c.in_backward = False
        if self._sync_enabled:
            c.reduce_scatter_grads()
        elif c.index == 0 or self.keep_in_step:
            # under no_sync another micro-batch follows and starts with this unit; its
            # parameters cannot change before then (no optimizer step), so keep them
            return
        c.reshard()

    # ------------------------------------------------------------------ strategy protocol
    def prepare_for_backward(self, groups: list) -> None:
        pass

    def reduce_grads(self, compute_grads: list, targets: list, target_specs: list) -> list:
        """Free parameters: all-reduce (AVG) over DP and return fp32 gradients."""
        from femtotron_b200.utils.comm_timing import TIMER
        if self.comm_stream is not None:
            cur = torch.cuda.current_stream(self.comm_stream.device)
            with TIMER.wait("grad_reduce"):
                cur.wait_stream(self.comm_stream)
                cur.wait_stream(self.ar_stream)
                if self.rs_stream is not None:
                    cur.wait_stream(self.rs_stream)
        early, self._early_reduced = self._early_reduced, set()
        out = []
        for g, t in zip(compute_grads, targets):
            if g is None:
                out.append(torch.zeros_like(t))
                continue
            if self.dp_size > 1 and id(g) not in early:
                with TIMER.wait("free_grad_allreduce"):
                    dist.all_reduce(g, op=dist.ReduceOp.AVG, group=self.dp_group)
            out.append(g if g.dtype == t.dtype else g.to(t.dtype))
        return out

    def wait_comm(self) -> None:
        if self.comm_stream is not None:
            cur = torch.cuda.current_stream(self.comm_stream.device)
            for st in (self.comm_stream, self.ar_stream, self.rs_stream):
                if st is not None:
                    cur.wait_stream(st)

    def gather_weights(self, groups: list) -> None:
        for g in groups:
            if g.master is not None:
                with torch.no_grad():
                    g.compute.copy_(g.master)

    def post_step(self) -> None:
        # Copy-engine gathers read peers' shards directly: every rank's optimizer update must
        # be complete before any rank gathers again.  A one-element all-reduce on the compute
        # stream is that device-side barrier.  (Peers finish reading a shard before its owner
        # updates it because every gather of a step precedes that step's last reduce-scatter
        # on the same communication stream, and the update waits for that reduce-scatter.)
        if self.heap is not None:
            from femtotron_b200.utils.comm_timing import TIMER
            with TIMER.wait("step_barrier"):
                dist.all_reduce(self._barrier_t, group=self.dp_group)
        # a unit still gathered now (kept across a forward whose backward never ran) holds
        # pre-update parameters
        for c in self.clusters:
            if not c.in_backward:
                c.reshard()

    def grads_are_dp_sharded(self) -> bool:
        return True

    @contextmanager
    def no_sync(self):
        prev = self._sync_enabled
        self._sync_enabled = False
        try:
            yield
        finally:
            self._sync_enabled = prev

    def sync_gradients(self) -> None:
        pass

    def state_dict(self) -> dict:
        return {}

    def load_state_dict(self, sd: dict) -> None:
        pass

    def force_reshard_all(self) -> None:
        """Exception recovery: drop every gathered buffer and pending prefetch."""
        self._early_reduced = set()
        for c in self.clusters:
            try:
                c._prefetch = None
                c._grad_buffer = None
                c.in_backward = False
                c.reshard()
            except Exception:
                pass

    def summary(self) -> dict:
        return {"num_clusters": len(self.clusters),
                "total_sharded_params": sum(c.total_numel for c in self.clusters),
                "memory_per_cluster": [c.memory_footprint() for c in self.clusters]}

    def cleanup(self) -> None:
        for h in self._hook_handles:
            h.remove()
        self._hook_handles.clear()
        self.clusters.clear()
        if self.heap is not None:
            torch.cuda.synchronize()
            self.heap.close()
            self.heap = None
