"""ZeRO-0: replicated fp32 master (reference femtotron/sharding/no_shard.py:16-67).
Gradient communication is left to the DDP synchroniser; this strategy only casts."""
from __future__ import annotations

import torch
from torch import nn


class NoShardStrategy:
    def __init__(self, dp_group):
        self.dp_group = dp_group

    def make_master(self, compute: nn.Parameter, master_dtype: torch.dtype):
        master = compute.detach().clone().to(master_dtype)
        master.requires_grad_(True)
        return master, None

    def prepare_for_backward(self, groups: list) -> None:
        pass

    def reduce_grads(self, compute_grads, targets, target_specs):
        return [g if g.dtype == t.dtype else g.to(t.dtype) for g, t in zip(compute_grads, targets)]

    def gather_weights(self, groups):
        for g in groups:
            g.sync_master_to_compute()

    def grads_are_dp_sharded(self) -> bool:
        return False

    def post_step(self) -> None:
        pass

    def make_clusters(self, model, groups, master_dtype):
        return []

    def cleanup(self):
        pass
