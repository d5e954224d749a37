"""ZeRO-3: parameters, gradients and optimizer state sharded over data parallelism.

Units are chosen by a wrap policy (default: one per decoder block).  Each unit becomes a
ParamGroupCluster and gets four module hooks (the roles of the reference's hooks,
femtotron/sharding/zero3.py:191-226), with these B200-specific behaviours:
  * forward-pre: unshard (consume the prefetched all-gather) and prefetch the NEXT unit on
    the communication stream, so the gather overlaps the current unit's compute;
  * forward-post: reshard -- except during an activation-checkpoint recompute inside the
    backward, and except when the unit is kept for the step (below);
  * backward-pre: unshard, attach the gradient buffer, prefetch the PREVIOUS unit;
  * backward-post: reduce-scatter the unit's gradients on the reduce stream (skipped under
    ``no_sync``), fused with the AdamW update of the shard when the optimizer allows it.

Memory-budgeted gather cache: when every unit's gathered bf16 parameters fit in a fraction
of the GPU's memory (FT_ZERO3_KEEP_IN_STEP=auto, the default; 1/0 force it), a unit stays
gathered from its first use in a step until its last backward of that step.  Parameters,
gradients and optimizer state stay sharded between steps, but a step gathers each unit once
instead of twice per micro-batch (forward, and again for the checkpoint recompute).

Free parameters (outside every unit: embedding, final norm, LM head) are sharded too
(FT_ZERO3_SHARD_FREE=1, the default): one cluster per owning module, gathered when the model's
forward starts and kept until the step ends, reduce-scattered as soon as the last
micro-batch's backward has produced its gradient.  The reference keeps them replicated with
unsharded fp32 masters and all-reduces their gradient (femtotron/sharding/zero3.py:67-79,
:231-261), which costs a full copy of their AdamW state on every rank.

Host waits are bounded: the run-ahead throttle polls its event with a deadline
(FT_HOST_WAIT_S, default 300 s) and raises instead of blocking forever.
With dp_size == 1 the clusters run in direct mode (no gathers, no copies).
"""
from __future__ import annotations

import os
import time
import warnings
from contextlib import contextmanager

import torch
import torch.distributed as dist
from torch import nn

from .param_group_cluster import ParamGroupCluster


class HostWaitTimeout(RuntimeError):
    """The host waited longer than its deadline for this rank's own GPU work."""


def wait_event_bounded(ev: torch.cuda.Event, deadline_s: float, what: str) -> None:
    """Block until `ev` completes, polling; raise HostWaitTimeout after `deadline_s`."""
    if ev.query():
        return
    t0 = time.monotonic()
    while not ev.query():
        if time.monotonic() - t0 > deadline_s:
            raise HostWaitTimeout(f"{what}: GPU work did not complete within {deadline_s:.0f} s "
                                  "(a peer stopped making progress?)")
        time.sleep(50e-6)


class ZeRO3Strategy:
    def __init__(self, dp_group, wrap_policy, prefetch: bool = True, symmetric: bool | None = None):
        self.dp_group = dp_group
        self.dp_rank = dist.get_rank(dp_group) if dp_group is not None else 0
        self.dp_size = dist.get_world_size(dp_group) if dp_group is not None else 1
        self.wrap_policy = wrap_policy
        self.prefetch_enabled = prefetch
        self.clusters: list[ParamGroupCluster] = []     # units, in model order
        self.free_clusters: list[ParamGroupCluster] = []
        self._hook_handles: list = []
        self._sync_enabled = True
        self.comm_stream = None
        self.rs_stream = None
        # all-gather through copy engines from symmetric (IPC-shared) shards and the fused
        # reduce-scatter over symmetric gradient buffers; default on for CUDA with dp > 1
        # (FT_ZERO3_SYMM=0 selects NCCL collectives for both)
        env = os.environ.get("FT_ZERO3_SYMM")
        self.symmetric = symmetric if symmetric is not None else (env != "0")
        self.heap = None
        self._barrier_t = None
        # bounded host run-ahead: before issuing a gather, the host waits for the point of the
        # compute stream reached `runahead` hooks earlier, which caps the in-flight buffers
        self.runahead = int(os.environ.get("FT_ZERO3_RUNAHEAD", "3"))
        self.host_wait_s = float(os.environ.get("FT_HOST_WAIT_S", "300"))
        self._inflight: list = []
        self.keep_mode = os.environ.get("FT_ZERO3_KEEP_IN_STEP", "auto")
        self.keep_in_step = False
        self.shard_free = os.environ.get("FT_ZERO3_SHARD_FREE", "1") != "0"
        self._free_ready: dict[int, set] = {}
        # set by the mixed-precision manager around the last backward before the step
        self.in_final_backward = False

    def make_master(self, compute: nn.Parameter, master_dtype: torch.dtype):
        # clusters build their own sharded fp32 masters; parameters that stay unsharded get
        # theirs in make_clusters (a full fp32 copy of every parameter first would cost
        # 4 bytes per parameter of transient memory, 70 GB per GPU on a 70B model at TP=4)
        self._master_dtype = master_dtype
        return None, None

    # ------------------------------------------------------------------ construction
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
        cuda = dev.type == "cuda"
        if cuda and self.dp_size > 1:
            self.comm_stream = torch.cuda.Stream(device=dev)
        if cuda:
            self.rs_stream = torch.cuda.Stream(device=dev)
        names = {m: n for n, m in model.named_modules()}
        unit_pgs, claimed = [], set()
        for u in units:
            pgs = []
            for p in u.parameters():
                if id(p) in claimed:
                    continue
                claimed.add(id(p))
                pg = by_id.get(id(p))
                if pg is None:
                    continue
                if pg.cluster is not None:
                    raise RuntimeError(f"parameter {pg.name} claimed by two units")
                pgs.append(pg)
            if pgs:
                unit_pgs.append((u, pgs))
        # free parameters, grouped by the module that owns them (dp > 1 only: with one rank
        # there is nothing to shard)
        free_pgs = []
        if self.dp_size > 1 and self.shard_free:
            owner = {}
            for m in model.modules():
                for p in m._parameters.values():
                    if p is not None:
                        owner.setdefault(id(p), m)
            by_owner: dict[int, tuple] = {}
            for pg in groups:
                if id(pg.compute) in claimed or not pg.compute.requires_grad:
                    continue
                m = owner.get(id(pg.compute))
                if m is None:
                    continue
                by_owner.setdefault(id(m), (m, []))[1].append(pg)
                claimed.add(id(pg.compute))
            free_pgs = list(by_owner.values())
        use_symm = self.symmetric and cuda and self.dp_size > 1
        grad_dtype = self._pick_grad_dtype(unit_pgs + free_pgs, dev)
        offsets, grad_offsets = [], []
        if use_symm:
            from femtotron_b200.parallel.symm import SymmetricAllocator, SymmetricHeap
            alloc = SymmetricAllocator()
            es = groups[0].compute.element_size()
            ges = torch.tensor([], dtype=grad_dtype).element_size()
            al = ParamGroupCluster.SYMM_ALIGN
            for i, (u, pgs) in enumerate(unit_pgs + free_pgs):
                shard = ParamGroupCluster.shard_numel(pgs, self.dp_size, al)
                offsets.append(alloc.reserve(f"unit{i}", shard * es))
                grad_offsets.append((alloc.reserve(f"grad{i}", shard * self.dp_size * ges),
                                     alloc.reserve(f"flags{i}", 4 * self.dp_size)))
            self.heap = SymmetricHeap(self.dp_group, None, alloc.size, dev)
            self._barrier_t = torch.zeros(1, device=dev)
        for i, (u, pgs) in enumerate(unit_pgs + free_pgs):
            c = ParamGroupCluster(names.get(u, type(u).__name__) or "<root>", u, pgs, self.dp_group,
                                  master_dtype, comm_stream=self.comm_stream,
                                  symm=(self.heap, offsets[i]) if use_symm else None,
                                  grad_offset=grad_offsets[i][0] if use_symm else None,
                                  flag_offset=grad_offsets[i][1] if use_symm else None)
            c.grad_dtype = grad_dtype
            c.rs_stream = self.rs_stream
            (self.clusters if i < len(unit_pgs) else self.free_clusters).append(c)
        self.keep_in_step = self._decide_keep(dev)
        for i, c in enumerate(self.clusters):
            c.index = i
            c.keep = self.keep_in_step
            if c.direct:
                self._install_direct_hook(c)
            else:
                self._install_hooks(c)
        for c in self.free_clusters:
            c.index = -1
            c.keep = True
            self._install_free_ready(c)
        if self.free_clusters:
            # the LM head and the final norm may be used through their weights only (fused
            # LM-head + loss), so the gathers hang off the root module's forward
            self._hook_handles.append(
                model.register_forward_pre_hook(lambda mod, args: self._pre_forward_root()))
        # unsharded free parameters (one rank, or sharding disabled) get a full fp32 master and
        # accumulate an fp32 gradient in place, all-reduced at step time
        for pg in groups:
            if pg.cluster is None and pg.compute.requires_grad:
                pg.master = pg.compute.detach().clone().to(master_dtype).requires_grad_(True)
                pg.compute.main_grad = torch.zeros(pg.compute.shape, dtype=torch.float32,
                                                   device=pg.compute.device)
        self.shards_written()
        return self.clusters + self.free_clusters

    def _decide_keep(self, dev) -> bool:
        if self.keep_mode in ("0", "1"):
            return self.keep_mode == "1"
        if dev.type != "cuda" or self.dp_size == 1:
            return False
        full = sum(c.padded_size * c.flat_param_shard.element_size() for c in self.clusters)
        cap = torch.cuda.get_device_properties(dev).total_memory
        return full <= 0.15 * cap

    def shards_written(self) -> None:
        """Call after this rank wrote its parameter shards into symmetric memory (construction,
        checkpoint load): peers' copy engines read those shards directly, so every rank's
        writes must be complete before any rank gathers.  Prefetched gathers are dropped."""
        for c in self.clusters + self.free_clusters:
            c.drop_prefetch()
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

    # ------------------------------------------------------------------ hooks
    def _install_hooks(self, c: ParamGroupCluster) -> None:
        m = c.module
        self._hook_handles += [
            m.register_forward_pre_hook(lambda mod, args, c=c: self._pre_forward(c)),
            m.register_forward_hook(lambda mod, args, out, c=c: self._post_forward(c)),
            m.register_full_backward_pre_hook(lambda mod, go, c=c: self._pre_backward(c)),
            m.register_full_backward_hook(lambda mod, gi, go, c=c: self._post_backward(c)),
        ]

    def _install_direct_hook(self, c: ParamGroupCluster) -> None:
        # one rank: only the end of the unit's backward matters (fused optimizer update)
        self._hook_handles.append(
            c.module.register_full_backward_hook(lambda mod, gi, go, c=c: self._post_backward_direct(c)))

    def _install_free_ready(self, c: ParamGroupCluster) -> None:
        params = [pg.compute for pg in c.param_groups if pg.compute.requires_grad]
        self._free_ready[id(c)] = set()
        for p in params:
            p._ft_grad_ready = (lambda p=p, c=c, n=len(params): self._free_grad_ready(c, p, n))

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
            wait_event_bounded(self._inflight.pop(0), self.host_wait_s, "ZeRO-3 run-ahead throttle")

    def _pre_forward(self, c):
        if not c.is_gathered:
            self._throttle()
        c.unshard()
        if self.prefetch_enabled and not c.in_backward:
            n = self._neighbor(c, +1)
            if n is not None:
                n.prefetch()

    def _post_forward(self, c):
        if c.in_backward or (c.keep and torch.is_grad_enabled()):
            return
        # the last unit's backward comes right after the forward: keep it gathered
        if c.index == len(self.clusters) - 1 and torch.is_grad_enabled():
            return
        c.reshard()

    def _pre_backward(self, c):
        if not c.is_gathered:
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
        elif c.index == 0 or c.keep:
            # under no_sync another micro-batch follows and starts with this unit; its
            # parameters cannot change before then (no optimizer step), so keep them
            return
        c.reshard()

    def _post_backward_direct(self, c):
        if self._sync_enabled:
            c.reduce_scatter_grads()

    def _pre_forward_root(self):
        """Gather every free cluster (kept until the step ends) and attach its gradient
        buffer; start the first unit's gather."""
        if self.prefetch_enabled:
            for c in self.free_clusters + self.clusters[:1]:
                c.prefetch()
        for c in self.free_clusters:
            c.unshard()
            if torch.is_grad_enabled():
                c.prepare_grad_buffer()

    def _free_grad_ready(self, c, p, n_params) -> None:
        # reduce as soon as the gradient is complete only inside the trainer's final backward
        # (exactly one backward follows); otherwise more backwards of the step may still add to
        # the buffer (pipeline micro-batches), and the reduction happens at step time
        if not (self._sync_enabled and self.in_final_backward):
            return
        ready = self._free_ready[id(c)]
        ready.add(id(p))
        if len(ready) >= n_params:
            ready.clear()
            c.reduce_scatter_grads()

    # ------------------------------------------------------------------ strategy protocol
    def prepare_for_backward(self, groups: list) -> None:
        pass

    def reduce_grads(self, compute_grads: list, targets: list, target_specs: list) -> list:
        """Unsharded free parameters: all-reduce (AVG) over DP and return fp32 gradients."""
        from femtotron_b200.utils.comm_timing import TIMER
        out = []
        for g, t in zip(compute_grads, targets):
            if g is None:
                out.append(torch.zeros_like(t))
                continue
            if self.dp_size > 1:
                with TIMER.wait("free_grad_allreduce"):
                    dist.all_reduce(g, op=dist.ReduceOp.AVG, group=self.dp_group)
            out.append(g if g.dtype == t.dtype else g.to(t.dtype))
        return out

    def wait_comm(self) -> None:
        # a unit whose backward hook did not reduce its gradients (e.g. a free parameter
        # whose gradient skipped the ready callback) is reduced now
        if self._sync_enabled:
            for c in self.clusters + self.free_clusters:
                if c._grad_buffer is not None:
                    c.reduce_scatter_grads()
        for ready in self._free_ready.values():
            ready.clear()
        if self.comm_stream is not None or self.rs_stream is not None:
            from femtotron_b200.utils.comm_timing import TIMER
            dev = (self.rs_stream or self.comm_stream).device
            cur = torch.cuda.current_stream(dev)
            with TIMER.wait("grad_reduce"):
                for st in (self.comm_stream, self.rs_stream):
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
        # stream (which waited for the reduce stream) is that device-side barrier.  It also
        # tells every rank that its peers finished reading its gradient buffers, which the
        # next step's backward overwrites.
        if self.heap is not None:
            from femtotron_b200.utils.comm_timing import TIMER
            with TIMER.wait("step_barrier"):
                dist.all_reduce(self._barrier_t, group=self.dp_group)
        # a unit still gathered now holds pre-update parameters
        for c in self.clusters + self.free_clusters:
            if not c.in_backward:
                c.reshard()
        # start the next step's first gathers right away (the embedding and the first unit)
        if self.prefetch_enabled and self.comm_stream is not None:
            for c in self.free_clusters[:1] + self.clusters[:1]:
                c.prefetch()

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
        """Exception recovery: drop every gathered buffer, pending prefetch and gradient
        buffer attachment."""
        for ready in self._free_ready.values():
            ready.clear()
        self._inflight.clear()
        for c in self.clusters + self.free_clusters:
            try:
                c._prefetch = None
                if c._grad_buffer is not None:
                    for pg in c.param_groups:
                        pg.compute.main_grad = None
                        pg.compute.grad_overwrite = False
                c._grad_buffer = None
                c.in_backward = False
                c.reshard()
            except Exception as e:      # recovery must not mask the error being handled
                warnings.warn(f"ZeRO-3 recovery could not reset cluster {c.name}: {e!r}")

    def summary(self) -> dict:
        cs = self.clusters + self.free_clusters
        return {"num_clusters": len(cs),
                "total_sharded_params": sum(c.total_numel for c in cs),
                "keep_in_step": self.keep_in_step,
                "memory_per_cluster": [c.memory_footprint() for c in cs]}

    def cleanup(self) -> None:
        for h in self._hook_handles:
            h.remove()
        self._hook_handles.clear()
        self.clusters.clear()
        self.free_clusters.clear()
        if self.heap is not None:
            torch.cuda.synchronize()
            self.heap.close()
            self.heap = None
