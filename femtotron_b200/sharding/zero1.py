"""ZeRO-1: the fp32 master and optimizer state are DP shards of each flattened, padded
parameter (reference femtotron/sharding/zero1.py:16-112).  At step time each gradient is
reduce-scattered (AVG) into this rank's shard; after the update the updated masters are
all-gathered back into the compute parameters.  Collectives of all parameters are issued
back to back inside one NCCL coalescing group."""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from .sharding_spec import ShardingSpec


def _flat_padded(t: torch.Tensor, spec: ShardingSpec, dtype=None) -> torch.Tensor:
    flat = t.reshape(-1)
    if dtype is not None and flat.dtype != dtype:
        flat = flat.to(dtype)
    if spec.pad_size > 0:
        flat = torch.cat([flat, torch.zeros(spec.pad_size, dtype=flat.dtype, device=flat.device)])
    return flat


class ZeRO1Strategy:
    def __init__(self, dp_group):
        self.dp_group = dp_group
        self.dp_rank = dist.get_rank(dp_group)
        self.dp_size = dist.get_world_size(dp_group)

    def make_master(self, compute: nn.Parameter, master_dtype: torch.dtype):
        spec = ShardingSpec.from_full(compute, self.dp_rank, self.dp_size)
        full = _flat_padded(compute.detach(), spec, master_dtype)
        shard = full[spec.shard_start:spec.shard_end].clone()
        shard.requires_grad_(True)
        return shard, spec

    def prepare_for_backward(self, groups) -> None:
        pass

    def reduce_grads(self, compute_grads, targets, target_specs):
        out = []
        for g, t, spec in zip(compute_grads, targets, target_specs):
            if spec is None or spec.world_size == 1:
                if self.dp_size > 1:
                    dist.all_reduce(g, op=dist.ReduceOp.AVG, group=self.dp_group)
                out.append(g if g.dtype == t.dtype else g.to(t.dtype))
                continue
            flat = _flat_padded(g, spec)
            shard = torch.empty(spec.shard_size, dtype=flat.dtype, device=flat.device)
            dist.reduce_scatter_tensor(shard, flat, op=dist.ReduceOp.AVG, group=self.dp_group)
            out.append(shard if shard.dtype == t.dtype else shard.to(t.dtype))
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

    def grads_are_dp_sharded(self) -> bool:
        return True

    def post_step(self) -> None:
        pass

    def make_clusters(self, model, groups, master_dtype):
        return []

    def cleanup(self):
        pass
