"""Optimizer parameter groups and the fused multi-tensor AdamW.

``get_param_groups`` follows the reference rule (femtotron/training/optimizer.py:5-40):
weight decay for >=2-D parameters whose name contains neither "bias" nor "embed".

``FusedAdamW`` is a torch.optim.Optimizer with torch.optim.AdamW semantics and state format
(``step``, ``exp_avg``, ``exp_avg_sq`` per parameter), whose update of all parameters of a
group is one multi-tensor sm_100a kernel launch.  ``bf16_targets`` maps a parameter to a
compute-dtype tensor that receives the updated value in the same pass (fusing the
master -> compute cast).  A device-side ``grad_scale`` (e.g. a clip coefficient) can be
applied without a host synchronisation.

Early (fused) updates: a ZeRO unit whose gradient shard is final before ``step()`` (the
reduce-scatter of the last micro-batch) can be updated by the fused reduce-scatter + AdamW
kernel while the backward still runs.  Its parameters' ``exp_avg``/``exp_avg_sq`` are then
slices of one flat buffer per unit (``bind_state``), and ``mark_updated`` tells ``step()`` to
skip them for this step.  The state dict format is unchanged.
"""
from __future__ import annotations

import torch
from torch import nn

from femtotron_b200.ops.kernels import adamw_multi


def get_param_groups(model: nn.Module, weight_decay: float = 0.01) -> list[dict]:
    decay, no_decay = [], []
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        if p.ndim <= 1 or "bias" in name or "embed" in name:
            no_decay.append(p)
        else:
            decay.append(p)
    return [{"params": decay, "weight_decay": weight_decay},
            {"params": no_decay, "weight_decay": 0.0}]


class FusedAdamW(torch.optim.Optimizer):
    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2, **kwargs):
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
        super().__init__(params, defaults)
        self.bf16_targets: dict[int, torch.Tensor] = {}
        self.grad_scale: torch.Tensor | None = None
        # parameters already updated this step by a fused reduce-scatter + AdamW pass
        self._early_done: set[int] = set()
        # parameter id -> (param, exp_avg view, exp_avg_sq view) of flat per-unit state
        self._bound: dict[int, tuple] = {}

    def bind_state(self, p: torch.Tensor, exp_avg: torch.Tensor, exp_avg_sq: torch.Tensor) -> None:
        """Make p's AdamW moments the given tensors (views of a flat buffer), keeping any
        values already in the state."""
        st = self.state[p]
        if len(st) == 0:
            st["step"] = torch.tensor(0.0)
        else:
            exp_avg.copy_(st["exp_avg"].view_as(exp_avg))
            exp_avg_sq.copy_(st["exp_avg_sq"].view_as(exp_avg_sq))
        st["exp_avg"] = exp_avg
        st["exp_avg_sq"] = exp_avg_sq
        self._bound[id(p)] = (p, exp_avg, exp_avg_sq)

    def mark_updated(self, params) -> int:
        """Advance the step count of `params` (updated outside ``step()``) and return it."""
        step_val = None
        for p in params:
            st = self.state[p]
            st["step"] += 1
            step_val = int(st["step"].item()) if step_val is None else step_val
            self._early_done.add(id(p))
        return step_val

    def load_state_dict(self, state_dict):
        super().load_state_dict(state_dict)
        for p, m, v in list(self._bound.values()):
            st = self.state[p]
            if "exp_avg" in st and st["exp_avg"] is not m:
                m.copy_(st["exp_avg"].view_as(m).to(m.device))
                v.copy_(st["exp_avg_sq"].view_as(v).to(v.device))
                st["exp_avg"], st["exp_avg_sq"] = m, v

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        for group in self.param_groups:
            ps, ms, vs, gs, outs, wds = [], [], [], [], [], []
            step_val = None
            for p in group["params"]:
                if p.grad is None or id(p) in self._early_done:
                    continue
                st = self.state[p]
                if len(st) == 0:
                    st["step"] = torch.tensor(0.0)
                    st["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                    st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                st["step"] += 1
                step_val = int(st["step"].item()) if step_val is None else step_val
                ps.append(p)
                ms.append(st["exp_avg"])
                vs.append(st["exp_avg_sq"])
                g = p.grad
                gs.append(g if g.is_contiguous() else g.contiguous())
                outs.append(self.bf16_targets.get(id(p)))
                wds.append(group["weight_decay"])
            if not ps:
                continue
            b1, b2 = group["betas"]
            adamw_multi(ps, ms, vs, gs, outs if any(o is not None for o in outs) else None, wds,
                        lr=group["lr"], beta1=b1, beta2=b2, eps=group["eps"], step=step_val,
                        grad_scale=self.grad_scale)
        self._early_done.clear()
        return loss
