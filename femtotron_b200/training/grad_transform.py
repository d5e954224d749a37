"""Gradient transforms applied to master gradients before the optimizer step.

ClipGradNorm: global L2 norm over all master gradients (reference
femtotron/training/grad_transform.py:13-83).  Each gradient's sum of squares is reduced over
exactly the groups that shard it: over TP for TP-sharded parameters, over DP for DP-sharded
gradients (ZeRO-1/2 master shards, ZeRO-3 cluster shards), over PP always (each stage holds
different layers; the reference omits PP).  Gradients replicated across a group are counted
once: the reference all-reduces the whole total over DP whenever the strategy shards, which
counts ZeRO-3's unsharded free parameters (embedding, LM head, final norm) dp times.  The sums of squares come
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

    @staticmethod
    def _dp_sharded(g) -> bool:
        """True when this rank's gradient of group `g` is its DP shard (ZeRO-1/2 master shard,
        ZeRO-3 cluster view), False when every DP rank holds the whole gradient (ZeRO-0, and
        ZeRO-3's unsharded free parameters such as the embedding and the LM head)."""
        return getattr(g, "cluster", None) is not None or getattr(g, "master_spec", None) is not None

    def __call__(self, param_groups: list, grads: list[torch.Tensor]) -> torch.Tensor:
        dev = grads[0].device if grads else torch.device("cpu")
        # slots: 0 tp-sharded & dp-sharded, 1 tp-replicated & dp-sharded,
        #        2 tp-sharded & dp-replicated, 3 tp-replicated & dp-replicated
        sq = torch.zeros(4, dtype=torch.float32, device=dev)
        slots = [(0 if g_.is_tp_sharded else 1) + (0 if self.dp_sharded and self._dp_sharded(g_) else 2)
                 for g_ in param_groups]
        sumsq_multi(list(grads), slots, sq)
        ctx = self.parallel_ctx
        if ctx.tp_size > 1 and ctx.tp_group is not None:   # TP shards: sum over the TP group
            t = sq[0::2].clone()
            dist.all_reduce(t, group=ctx.tp_group)
            sq[0::2] = t
        if self.dp_sharded and ctx.dp_size > 1 and ctx.dp_group is not None:   # DP shards
            t = sq[0:2].clone()
            dist.all_reduce(t, group=ctx.dp_group)
            sq[0:2] = t
        # replicated gradients are counted once: they are not reduced over the group that
        # replicates them
        total = sq.sum().reshape(1)
        if self.reduce_pp and ctx.pp_size > 1 and ctx.pp_group is not None:
            dist.all_reduce(total, group=ctx.pp_group)
        norm = total.sqrt()[0]
        coef = (self.max_norm / (norm + 1e-6)).clamp(max=1.0)
        if grads:
            torch._foreach_mul_(list(grads), coef)
        self.last_norm, self.coef = norm, coef
        return norm
