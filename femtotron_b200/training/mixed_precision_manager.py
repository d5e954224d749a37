"""bf16 compute parameters + fp32 master weights + optimizer, under a sharding strategy.

Public API of the reference (femtotron/training/mixed_precision_manager.py:22-476):
``MixedPrecisionManager(model, parallel_ctx, parallel_plan, config, inner_optimizer_cls,
inner_optimizer_kwargs, compute_param_groups, grad_transforms=None, sharding_strategy=None)``
with ``step()`` = copy_grads_to_master -> transforms -> inner.step -> sync_weights ->
zero_grad, and ``state_dict`` / ``load_state_dict``.

B200 specifics:
  * gradients are read from ``main_grad`` (fp32, written in place by the fused wgrad GEMMs)
    when present, so no bf16 -> fp32 gradient copy is made for those parameters;
  * with :class:`FusedAdamW` as the inner optimizer, the update writes the new bf16 compute
    values in the same kernel pass wherever the master and the compute tensor have the same
    layout (replicated masters, ZeRO-3 shards), replacing the separate cast/copy;
  * ZeRO-3 cluster masters are part of ``state_dict`` (the reference omits them).
"""
from __future__ import annotations

import os
from collections import defaultdict
from contextlib import contextmanager

import torch
from torch import nn

from femtotron_b200.sharding.no_shard import NoShardStrategy
from .grad_accumulator import GradAccumulator
from .optimizer import FusedAdamW
from .param_group import ParamGroup


class MixedPrecisionManager:
    def __init__(self, model: nn.Module, parallel_ctx, parallel_plan, config, inner_optimizer_cls,
                 inner_optimizer_kwargs: dict, compute_param_groups: list[dict],
                 grad_transforms: list | None = None, sharding_strategy=None):
        self.parallel_ctx = parallel_ctx
        self.strategy = sharding_strategy if sharding_strategy is not None else NoShardStrategy(parallel_ctx.dp_group)
        meta = {}
        for cg in compute_param_groups:
            m = {k: v for k, v in cg.items() if k != "params"}
            for p in cg["params"]:
                meta[id(p)] = m
        self.groups: list[ParamGroup] = []
        for name, p in model.named_parameters():
            if config.master_dtype is not None:
                master, spec = self.strategy.make_master(p, config.master_dtype)
            else:
                master, spec = None, None
            self.groups.append(ParamGroup(name, p, master, meta.get(id(p), {}), parallel_ctx,
                                          parallel_plan, master_spec=spec))
        self.grad_accs = [GradAccumulator(g, config, parallel_ctx) for g in self.groups]
        self.clusters = self.strategy.make_clusters(model=model, groups=self.groups,
                                                    master_dtype=config.master_dtype)
        targets = []
        for g in self.groups:
            if g.master is not None:
                targets.append((g, g.master))
            elif g.cluster is not None:
                v = g.cluster.param_views.get(g.name)
                if v is not None:
                    targets.append((g, v))
            elif config.master_dtype is None:
                targets.append((g, g.compute))
        self.opt_targets = targets
        by_cfg = defaultdict(list)
        for g, t in targets:
            by_cfg[frozenset(g.opt_config.items())].append(t)
        opt_groups = [{"params": ts, **dict(k)} for k, ts in by_cfg.items()]
        self.inner = inner_optimizer_cls(opt_groups, **inner_optimizer_kwargs)
        self.config = config
        self.grad_transforms = grad_transforms or []
        self._fused_groups: set[int] = set()
        self._fused_clusters: set[int] = set()
        # inside final_backward(): ZeRO units may apply their optimizer update fused with the
        # gradient reduce-scatter of this (last) backward of the step
        self._early_ok = False
        if isinstance(self.inner, FusedAdamW):
            self._register_fused_writeback()
            if os.environ.get("FT_FUSED_RS_ADAMW", "1") != "0":
                self._install_early_updates()

    # ------------------------------------------------------------------ setup helpers
    def _register_fused_writeback(self) -> None:
        opt = self.inner
        cluster_views_done = defaultdict(int)
        for g, t in self.opt_targets:
            if g.master is not None and g.master_spec is None and g.compute.is_contiguous() \
                    and g.master.numel() == g.compute.numel() and g.compute.numel() > 0:
                opt.bf16_targets[id(t)] = g.compute.data.view(-1) if g.master.dim() == 1 else g.compute.data
                self._fused_groups.add(id(g))
            elif g.cluster is not None and g.name in g.cluster.compute_views:
                opt.bf16_targets[id(t)] = g.cluster.compute_views[g.name]
                cluster_views_done[id(g.cluster)] += 1
        for c in self.clusters:
            if cluster_views_done[id(c)] == len(c.param_views):
                self._fused_clusters.add(id(c))

    def _install_early_updates(self) -> None:
        """Give every CUDA cluster whose update the fused kernel can do a flat fp32 buffer
        for each AdamW moment (the optimizer's per-view state becomes slices of it) and the
        callback that supplies the fused update's arguments."""
        opt = self.inner
        group_of = {id(p): grp for grp in opt.param_groups for p in grp["params"]}
        for c in self.clusters:
            if c.device.type != "cuda" or id(c) not in self._fused_clusters or not c.param_views:
                continue
            m = torch.zeros(c.shard_size, dtype=torch.float32, device=c.device)
            v = torch.zeros_like(m)
            segs = []
            for pg, l in zip(c.param_groups, c.layouts):
                if not l.has_local_view:
                    continue
                t = c.param_views[pg.name]
                opt.bind_state(t, m.narrow(0, l.local_offset, l.local_numel),
                               v.narrow(0, l.local_offset, l.local_numel))
                segs.append((l.local_offset, l.local_end, group_of[id(t)], t))
            c._flat_m, c._flat_v, c._segs = m, v, segs
            c.early_update = self._early_args

    def _early_args(self, c):
        """Arguments of the fused reduce-scatter + AdamW update of cluster c for this step, or
        None when the update must wait for step() (outside final_backward(), gradient
        clipping or another transform, or a second reduction of the same step)."""
        if not self._early_ok or c.updated_early or self.grad_transforms or \
                self.inner.grad_scale is not None:
            return None
        hyper = {(tuple(g["betas"]), g["eps"]) for _, _, g, _ in c._segs}
        if len(hyper) != 1:
            return None
        (betas, eps), = hyper
        step = self.inner.mark_updated([t for _, _, _, t in c._segs])
        segs = torch.tensor([[s, e, g["lr"], g["weight_decay"]] for s, e, g, _ in c._segs],
                            dtype=torch.float64)
        return dict(exp_avg=c._flat_m, exp_avg_sq=c._flat_v, segments=segs, beta1=betas[0],
                    beta2=betas[1], eps=eps, step=step)

    @contextmanager
    def final_backward(self):
        """Wrap the last backward before ``step()``: ZeRO units whose gradients are complete
        after it may be updated by the fused reduce-scatter + AdamW kernel right away, on
        the reduce stream, while the rest of the backward runs."""
        prev = self._early_ok
        prev_s = getattr(self.strategy, "in_final_backward", None)
        self._early_ok = True
        if prev_s is not None:
            self.strategy.in_final_backward = True
        try:
            yield
        finally:
            self._early_ok = prev
            if prev_s is not None:
                self.strategy.in_final_backward = prev_s

    @property
    def compute_dtype(self) -> torch.dtype:
        return self.config.param_dtype

    def cleanup(self):
        if hasattr(self.strategy, "cleanup"):
            self.strategy.cleanup()
        self.inner.state.clear()
        self.inner.param_groups.clear()
        self.opt_targets.clear()
        self.clusters.clear()
        self.groups.clear()

    # ------------------------------------------------------------------ step pieces
    def accumulate_grads(self) -> None:
        for ga in self.grad_accs:
            ga.accumulate()

    def copy_grads_to_master(self):
        wait = getattr(self.strategy, "wait_comm", None)
        if wait is not None:
            wait()
        sg, sm, ss, sl = [], [], [], []
        for i, g in enumerate(self.groups):
            if g.master is None:
                continue
            sg.append(g)
            sm.append(g.master)
            ss.append(g.master_spec)
            sl.append(self.grad_accs[i].finalize())
        if sg:
            filled = [x if x is not None else torch.zeros(g.compute.shape, dtype=torch.float32,
                                                          device=g.master.device)
                      for x, g in zip(sl, sg)]
            synced = self.strategy.reduce_grads(compute_grads=filled, targets=sm, target_specs=ss)
            for g, s in zip(sg, synced):
                g.assign_grad(s.reshape(g.master.shape))
        for c in self.clusters:
            c.populate_master_grad()
        if self.config.master_dtype is None:
            for i, g in enumerate(self.groups):
                if g.master is None and g.cluster is None:
                    fin = self.grad_accs[i].finalize()
                    if fin is not None and fin is not g.compute.grad:
                        g.compute.grad = fin.to(g.compute.dtype)
        return self.grad_transform()

    def grad_transform(self) -> list:
        gs, grads = [], []
        for g, t in self.opt_targets:
            if t.grad is not None:
                gs.append(g)
                grads.append(t.grad)
        return [tr(gs, grads) for tr in self.grad_transforms]

    def sync_weights(self) -> None:
        if self._fused_groups:
            self.strategy.gather_weights([g for g in self.groups if id(g) not in self._fused_groups])
        else:
            self.strategy.gather_weights(self.groups)
        for c in self.clusters:
            if id(c) not in self._fused_clusters:
                c.sync_master_to_compute()

    def zero_grad(self) -> None:
        for ga in self.grad_accs:
            ga.reset()
        for g in self.groups:
            g.zero_grad()
            mg = getattr(g.compute, "main_grad", None)
            if mg is not None and g.cluster is None:
                mg.zero_()
        for c in self.clusters:
            c.zero_grad()
        self.strategy.post_step()

    def step(self) -> bool:
        self.copy_grads_to_master()
        self.inner.step()
        self.sync_weights()
        self.zero_grad()
        return True

    # ------------------------------------------------------------------ checkpoint
    def state_dict(self) -> dict:
        return {
            "version": 1,
            "master_weights": {g.name: g.master.detach().cpu() for g in self.groups if g.master is not None},
            "master_specs": {g.name: g.master_spec for g in self.groups if g.master_spec is not None},
            "cluster_masters": {c.name: c.state_dict() for c in self.clusters},
            "inner_optimizer": self.inner.state_dict(),
            "grad_accumulators": {g.name: ga.state_dict() for g, ga in zip(self.groups, self.grad_accs)},
            "config": {
                "master_dtype": str(self.config.master_dtype) if self.config.master_dtype else None,
                "param_dtype": str(self.config.param_dtype),
                "num_groups": len(self.groups),
                "param_names": [g.name for g in self.groups],
                "dp_size": self.parallel_ctx.dp_size,
                "tp_size": self.parallel_ctx.tp_size,
                "sharding_strategy_kind": type(self.strategy).__name__,
            },
        }

    def load_state_dict(self, sd: dict) -> None:
        version = sd.get("version", 1)
        if version > 2:
            raise ValueError(f"unsupported checkpoint version {version}")
        cfg = sd["config"]
        if cfg["num_groups"] != len(self.groups):
            raise RuntimeError(f"param group count mismatch: ckpt {cfg['num_groups']} vs {len(self.groups)}")
        exp = str(self.config.master_dtype) if self.config.master_dtype else None
        if cfg["master_dtype"] != exp:
            raise RuntimeError(f"master_dtype mismatch: ckpt={cfg['master_dtype']}, current={exp}")
        if cfg.get("sharding_strategy_kind") not in (None, type(self.strategy).__name__):
            raise RuntimeError(f"sharding strategy mismatch: ckpt={cfg['sharding_strategy_kind']}, "
                               f"current={type(self.strategy).__name__}")
        if type(self.strategy).__name__ != "NoShardStrategy" and cfg.get("dp_size") not in (None, self.parallel_ctx.dp_size):
            raise RuntimeError(f"dp_size mismatch under {type(self.strategy).__name__}")
        names = [g.name for g in self.groups]
        if cfg["param_names"] != names:
            a, b = set(cfg["param_names"]) - set(names), set(names) - set(cfg["param_names"])
            raise RuntimeError(f"param names mismatch; only in ckpt: {sorted(a)[:5]}, only current: {sorted(b)[:5]}")
        mw = sd["master_weights"]
        for g in self.groups:
            if g.master is None:
                continue
            if g.name not in mw:
                raise RuntimeError(f"missing master weight for {g.name}")
            w = mw[g.name]
            if w.shape != g.master.shape:
                raise RuntimeError(f"shape mismatch for {g.name}: ckpt {tuple(w.shape)} vs {tuple(g.master.shape)}")
            with torch.no_grad():
                g.master.copy_(w.to(g.master.device))
        cm = sd.get("cluster_masters", {})
        for c in self.clusters:
            if c.name in cm:
                c.load_state_dict(cm[c.name])
        written = getattr(self.strategy, "shards_written", None)
        if written is not None:
            written()   # peers read the rewritten shards directly: order them before any gather
        self.inner.load_state_dict(sd["inner_optimizer"])
        gas = sd.get("grad_accumulators", {})
        for g, ga in zip(self.groups, self.grad_accs):
            if g.name in gas:
                ga.load_state_dict(gas[g.name])
