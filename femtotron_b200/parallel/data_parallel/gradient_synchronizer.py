"""Gradient synchronisation across data-parallel replicas (reference
femtotron/parallel/data_parallel/gradient_synchronizer.py:22-87).  Strategies that reduce
gradients themselves (ZeRO-1/2/3) need no synchroniser; ZeRO-2 and ZeRO-3 double as one
because their reduce-scatter is gated by ``no_sync``.

ZeRO-3 differs from the reference here: the reference returns a no-op synchroniser for it, so
its trainer's ``no_sync`` never reaches the strategy and every micro-batch reduce-scatters
every unit.  Here the trainer's ``no_sync`` keeps the unsharded gradients accumulating over
the micro-batches of a step and each unit is reduce-scattered once, after the last one."""
from __future__ import annotations

from contextlib import AbstractContextManager, nullcontext
from typing import Protocol

from .ddp import DataParallelGradSync


class GradientSynchronizer(Protocol):
    def sync_gradients(self) -> None: ...
    def no_sync(self) -> AbstractContextManager[None]: ...
    def state_dict(self) -> dict: ...
    def load_state_dict(self, sd: dict) -> None: ...


class NoOpGradSync:
    def sync_gradients(self):
        pass

    def no_sync(self):
        return nullcontext()

    def state_dict(self):
        return {}

    def load_state_dict(self, sd):
        pass


def create_grad_synchronizer(groups, parallel_ctx, strategy):
    from femtotron_b200.sharding.zero2 import ZeRO2Strategy
    from femtotron_b200.sharding.zero3 import ZeRO3Strategy
    if isinstance(strategy, (ZeRO2Strategy, ZeRO3Strategy)):
        return strategy
    if strategy.grads_are_dp_sharded() or parallel_ctx.dp_size == 1:
        return NoOpGradSync()
    return DataParallelGradSync(groups, parallel_ctx)
