"""Gradient synchronisation across data-parallel replicas (reference
femtotron/parallel/data_parallel/gradient_synchronizer.py:22-87).  Strategies that reduce
gradients themselves (ZeRO-1/2/3) need no synchroniser; ZeRO-2 doubles as one because its
reduce-scatter is gated by ``no_sync``."""
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
    if isinstance(strategy, ZeRO2Strategy):
        return strategy
    if strategy.grads_are_dp_sharded() or parallel_ctx.dp_size == 1:
        return NoOpGradSync()
    return DataParallelGradSync(groups, parallel_ctx)
