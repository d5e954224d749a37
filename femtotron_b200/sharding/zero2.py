"""ZeRO-2: ZeRO-1 plus gradient sharding during the backward (reference
femtotron/sharding/zero2.py:17-158).

Gradients are reduce-scattered as soon as a unit (decoder block) has finished its backward
(module backward hook), instead of per parameter as in the reference — the fused kernels
write gradients in place, so no per-parameter autograd hook fires.  The shard is accumulated
in fp32 and the full gradient is released.  Parameters outside any unit are reduced at
step time.  ``no_sync`` defers the reduction (the full gradient keeps accumulating), which
also makes this object the gradient synchroniser.
"""
from __future__ import annotations

from contextlib import contextmanager

import torch
import torch.distributed as dist
from torch import nn

from .sharding_spec import ShardingSpec
from .zero1 import _flat_padded
from femtotron_b200.training.param_group import local_grad


class ZeRO2Strategy:
    def __init__(self, dp_group, unit_policy=None):
        self.dp_group = dp_group
        self.dp_rank = dist.get_rank(dp_group)
        self.dp_size = dist.get_world_size(dp_group)
        self.unit_policy = unit_policy
        self._sync_enabled = True
        self._grad_shards: dict[str, torch.Tensor] = {}
        self.groups_ref: list = []
        self._hook_handles: list = []
        self._registered = False
        self._model = None

    def make_master(self, compute: nn.Parameter, master_dtype: torch.dtype):
        spec = ShardingSpec.from_full(compute, self.dp_rank, self.dp_size)
        full = _flat_padded(compute.detach(), spec, master_dtype)
        shard = full[spec.shard_start:spec.shard_end].clone()
        shard.requires_grad_(True)
        return shard, spec

    def make_clusters(self, model, groups, master_dtype):
        self._model = model
        return []

    def prepare_for_backward(self, groups) -> None:
        if self._registered:
            return
        self.groups_ref = list(groups)
        by_id = {id(g.compute): g for g in groups}
        policy = self.unit_policy
        if policy is None:
            from .wrap_policy import llama_wrap_policy
            policy = llama_wrap_policy
        if self._model is not None:
            for m in self._model.modules():
                if policy(m):
                    unit_groups = [by_id[id(p)] for p in m.parameters() if id(p) in by_id]
                    self._hook_handles.append(m.register_full_backward_hook(
                        lambda mod, gi, go, ug=unit_groups: self._reduce_groups(ug)))
        self._registered = True

    def _reduce_groups(self, groups) -> None:
        if not self._sync_enabled:
            return
        for g in groups:
            grad = local_grad(g.compute)
            if grad is None or g.master_spec is None:
                continue
            spec = g.master_spec
            flat = _flat_padded(grad, spec, torch.bfloat16 if grad.dtype == torch.bfloat16 else None)
            shard = torch.empty(spec.shard_size, dtype=flat.dtype, device=flat.device)
            dist.reduce_scatter_tensor(shard, flat, op=dist.ReduceOp.AVG, group=self.dp_group)
            prev = self._grad_shards.get(g.name)
            if prev is None:
                self._grad_shards[g.name] = shard.to(torch.float32)
            else:
                prev.add_(shard.to(torch.float32))
            if getattr(g.compute, "main_grad", None) is not None:
                g.compute.main_grad.zero_()
            else:
                g.compute.grad = None

    def reduce_grads(self, compute_grads, targets, target_specs):
        # flush parameters whose gradients were not reduced by a unit hook
        pending = [g for g in self.groups_ref if g.name not in self._grad_shards]
        self._reduce_groups(pending)
        out = []
        for g, t in zip(self.groups_ref, targets):
            s = self._grad_shards.get(g.name)
            out.append(torch.zeros_like(t) if s is None else (s if s.dtype == t.dtype else s.to(t.dtype)))
        return out

    def gather_weights(self, groups):
        with torch.no_grad():
            for g in groups:
                if g.master is None or g.master_spec is None:
                    continue
                spec = g.master_spec
                src = g.master.detach().to(g.compute.dtype)
                full = torch.empty(spec.flat_size, dtype=src.dtype, device=src.device)
                dist.all_gather_into_tensor(full, src, group=self.dp_group)
                g.compute.copy_(full[: spec.flat_size - spec.pad_size].view(spec.full_shape))

    def post_step(self) -> None:
        self._grad_shards.clear()

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

    def load_state_dict(self, sd) -> None:
        pass

    def cleanup(self):
        for h in self._hook_handles:
            h.remove()
        self._hook_handles.clear()
        self._grad_shards.clear()
        self.groups_ref = []
