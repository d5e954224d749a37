"""Stage number -> sharding strategy (reference femtotron/sharding/factory.py:22-42)."""
from __future__ import annotations

from .no_shard import NoShardStrategy
from .zero1 import ZeRO1Strategy
from .zero2 import ZeRO2Strategy
from .zero3 import ZeRO3Strategy
from .zero_config import ZeROConfig


def create_sharding_strategy(parallel_ctx, config: ZeROConfig):
    if config.stage == 0:
        return NoShardStrategy(parallel_ctx.dp_group)
    if config.stage == 1:
        return ZeRO1Strategy(parallel_ctx.dp_group)
    if config.stage == 2:
        return ZeRO2Strategy(parallel_ctx.dp_group)
    if config.stage == 3:
        if config.wrap_policy is None:
            raise ValueError("ZeRO-3 requires wrap_policy (a callable selecting the units, "
                             "typically each transformer block)")
        return ZeRO3Strategy(parallel_ctx.dp_group, config.wrap_policy, prefetch=config.prefetch)
    raise ValueError(f"unknown ZeRO stage {config.stage}")
