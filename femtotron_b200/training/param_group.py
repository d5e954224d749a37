"""One logical parameter and its storages (reference femtotron/training/param_group.py:29-161):
the compute parameter (bf16), an optional master (fp32, possibly a DP shard) with its
ShardingSpec, the optimizer options, the owning ZeRO-3 cluster, and TP metadata derived
from the parallel plan."""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn


def local_grad(p: torch.Tensor) -> torch.Tensor | None:
    """The gradient accumulated for compute parameter p: the fp32 ``main_grad`` buffer if
    the fused kernels write one, else ``p.grad``."""
    mg = getattr(p, "main_grad", None)
    return mg if mg is not None else p.grad


class ParamGroup:
    def __init__(self, name: str, compute: nn.Parameter, master: torch.Tensor | None,
                 opt_config: dict, parallel_ctx, parallel_plan, master_spec=None):
        self.name = name
        self.compute = compute
        self.master = master
        self.master_spec = master_spec
        self.opt_config = dict(opt_config)
        self.cluster = None
        module_name = name.rsplit(".", 1)[0] if "." in name else name
        rule = parallel_plan.get_rule(module_name) if parallel_plan is not None else None
        tp = parallel_ctx.tp_size if parallel_ctx is not None else 1
        kind = rule.parallel_type if rule is not None else None
        if kind is None or kind == "replicate" or tp <= 1:
            self.is_tp_sharded, self.tp_shard_dim = False, None
        elif kind in ("column", "vocab_embed"):
            self.is_tp_sharded, self.tp_shard_dim = True, 0
        elif kind == "row":
            self.is_tp_sharded, self.tp_shard_dim = True, 1
        else:
            self.is_tp_sharded, self.tp_shard_dim = False, None
        if name.endswith(".bias") and kind == "row":
            self.is_tp_sharded, self.tp_shard_dim = False, None
        self.is_replicated_across_dp = True

    def sync_master_to_compute(self) -> None:
        if self.master is None:
            return
        with torch.no_grad():
            self.compute.copy_(self.master.view(self.compute.shape) if self.master.numel() == self.compute.numel()
                               else self.master)

    def init_master_from_compute(self) -> None:
        if self.master is None:
            return
        with torch.no_grad():
            self.master.copy_(self.compute.reshape(self.master.shape))

    @property
    def optimized_param(self) -> torch.Tensor:
        return self.master if self.master is not None else self.compute

    @property
    def is_master_sharded(self) -> bool:
        return self.master_spec is not None and self.master_spec.world_size > 1

    @property
    def has_own_master(self) -> bool:
        return self.master is not None

    @property
    def is_clustered(self) -> bool:
        return self.cluster is not None

    def assign_grad(self, grad: torch.Tensor | None) -> None:
        target = self.optimized_param
        if grad is None:
            target.grad = None
            return
        if grad.shape != target.shape:
            raise ValueError(f"{self.name}: grad shape {tuple(grad.shape)} != {tuple(target.shape)}")
        target.grad = grad

    def gather_master_to_compute(self, dp_group) -> None:
        m = self.master
        if m is None:
            return
        if not self.is_master_sharded:
            self.sync_master_to_compute()
            return
        spec = self.master_spec
        gathered = torch.empty(spec.flat_size, dtype=m.dtype, device=m.device)
        dist.all_gather_into_tensor(gathered, m, group=dp_group)
        full = gathered[: spec.flat_size - spec.pad_size].view(spec.full_shape)
        with torch.no_grad():
            self.compute.copy_(full)

    def zero_grad(self) -> None:
        self.optimized_param.grad = None
