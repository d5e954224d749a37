"""Optional separate gradient-accumulation buffer per parameter (reference
femtotron/training/grad_accumulator.py:24-72).

With ``grad_acc_dtype=None`` gradients accumulate in place (in ``main_grad`` or ``.grad``;
the fused wgrad GEMMs already accumulate in their epilogue).  With a dtype, every
``accumulate()`` adds the current gradient into a buffer of that dtype and clears it.
(The reference's ``load_state_dict`` passes ``...`` to ``.to``; this one restores onto the
parameter's device.)"""
from __future__ import annotations

import torch

from .param_group import local_grad


class GradAccumulator:
    def __init__(self, group, train_config, parallel_ctx):
        self.group = group
        self.train_config = train_config
        self.parallel_ctx = parallel_ctx
        self.acc_buffer: torch.Tensor | None = None

    def accumulate(self) -> None:
        g = local_grad(self.group.compute)
        if g is None or self.train_config.grad_acc_dtype is None:
            return
        if self.acc_buffer is None:
            self.acc_buffer = torch.zeros_like(g, dtype=self.train_config.grad_acc_dtype)
        self.acc_buffer.add_(g.to(self.train_config.grad_acc_dtype))
        g.zero_()

    def finalize(self) -> torch.Tensor | None:
        if self.acc_buffer is not None:
            return self.acc_buffer
        return local_grad(self.group.compute)

    def reset(self) -> None:
        if self.acc_buffer is not None:
            self.acc_buffer.zero_()
        p = self.group.compute
        if getattr(p, "main_grad", None) is not None:
            p.grad_overwrite = True  # next wgrad stores instead of accumulating (no memset)
        elif p.grad is not None:
            p.grad = None

    def state_dict(self) -> dict:
        return {"acc_buffer": self.acc_buffer.detach().cpu() if self.acc_buffer is not None else None}

    def load_state_dict(self, sd: dict) -> None:
        buf = sd.get("acc_buffer")
        if buf is None:
            self.acc_buffer = None
        elif self.acc_buffer is None:
            self.acc_buffer = buf.to(self.group.compute.device)
        else:
            self.acc_buffer.copy_(buf.to(self.acc_buffer.device))
