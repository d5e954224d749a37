"""Gradient transforms applied to master gradients before the optimizer step.

ClipGradNorm: global L2 norm over all master gradients, split into TP-sharded and replicated
parts (reference femtotron/training/grad_transform.py:13-83): the sharded sum of squares is
reduced over TP, the total over DP when gradients are DP-sharded, and — unlike the
reference — over PP as well (each stage holds different layers).  The sums of squares come
from one multi-tensor kernel launch, and the clip coefficient stays on the device (no host
synchronisation); it is exported as ``last_norm`` / ``coef``.
"""
from __future__ import annotations

from typing import Protocol

import torch
import torch.distributed as dist

from femtotron_b200.ops.kernels import sumsq_multi


class GradTransform(Protocol):
    def __call__(self, param_groups: list, grads: list[torch.Tensor]) -> torch.Tensor: ...


class ClipGradNorm:
    def __init__(self, max_norm: float, parallel_ctx, *, dp_sharded: bool = False,
                 reduce_pp: bool = True):
        self.max_norm = float(max_norm)
        self.parallel_ctx = parallel_ctx
        self.dp_sharded = dp_sharded
        self.reduce_pp = reduce_pp
        self.last_norm: torch.Tensor | None = None
        self.coef: torch.Tensor | None = None

    def __call__(self, param_groups: list, grads: list[torch.Tensor]) -> torch.Tensor:
        dev = grads[0].device if grads else torch.device("cpu")
        sq = torch.zeros(2, dtype=torch.float32, device=dev)  # [tp-sharded, replicated]
        slots = [0 if g_.is_tp_sharded else 1 for g_ in param_groups]
        sumsq_multi(list(grads), slots, sq)
        ctx = self.parallel_ctx
        if ctx.tp_size > 1 and ctx.tp_group is not None:
            shard = sq[0:1].clone()
            dist.all_reduce(shard, group=ctx.tp_group)
            total = shard[0] + sq[1]
        else:
            total = sq[0] + sq[1]
        total = total.reshape(1)
        if self.dp_sharded and ctx.dp_size > 1 and ctx.dp_group is not None:
            dist.all_reduce(total, group=ctx.dp_group)
        if self.reduce_pp and ctx.pp_size > 1 and ctx.pp_group is not None:
            dist.all_reduce(total, group=ctx.pp_group)
        norm = total.sqrt()[0]
        coef = (self.max_norm / (norm + 1e-6)).clamp(max=1.0)
        if grads:
            torch._foreach_mul_(list(grads), coef)
        self.last_norm, self.coef = norm, coef
        return norm
