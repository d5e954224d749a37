"""ZeRO configuration: the reference's fields (femtotron/sharding/zero_config.py:8) plus
``prefetch`` for the ZeRO-3 parameter gathers."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

from torch import nn


@dataclass
class ZeROConfig:
    stage: int = 0                                    # 0 none, 1 optimizer, 2 +grads, 3 +params
    wrap_policy: Callable[[nn.Module], bool] | None = None  # ZeRO-3 unit selector
    prefetch: bool = True                             # ZeRO-3: all-gather the next unit early
