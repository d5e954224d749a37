"""Linear warmup then cosine decay to min_lr_ratio (reference
femtotron/training/lr_schedule.py:5-41, including its one-step shift: the lambda sees
current_step + 1)."""
from __future__ import annotations

import math

import torch


def create_lr_schedule(optimizer, warmup_steps: int, total_steps: int, min_lr_ratio: float = 0.1):
    if not 0 <= warmup_steps <= total_steps:
        raise ValueError(f"warmup_steps ({warmup_steps}) must be in [0, total_steps={total_steps}]")
    if not 0.0 <= min_lr_ratio <= 1.0:
        raise ValueError(f"min_lr_ratio ({min_lr_ratio}) must be in [0, 1]")
    decay = max(1, total_steps - warmup_steps)

    def lr_lambda(step: int) -> float:
        step = step + 1
        if step < warmup_steps:
            return float(step) / max(1, warmup_steps)
        progress = min((step - warmup_steps) / decay, 1.0)
        return min_lr_ratio + (1.0 - min_lr_ratio) * 0.5 * (1.0 + math.cos(math.pi * progress))

    return torch.optim.lr_scheduler.LambdaLR(optimizer, lr_lambda)
