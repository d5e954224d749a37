"""Layout of the parameters of one ZeRO-3 unit inside its flat, DP-sharded buffer.

The parameters are concatenated in order into one flat vector padded to a multiple of
dp_size; rank r owns [r*shard, (r+1)*shard).  Each parameter has a global offset and, when
it intersects this rank's shard, a local offset/length (parameters may straddle ranks).
Same layout rule as the reference (femtotron/sharding/cluster_sharding_spec.py:18-159), which
the unit tests of that rule pin down.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class ClusterShardingSpec:
    global_offset: int
    numel: int
    original_shape: torch.Size
    original_dtype: torch.dtype
    has_local_view: bool
    local_offset: int = 0
    local_numel: int = 0

    @property
    def global_end(self) -> int:
        return self.global_offset + self.numel

    @property
    def local_end(self) -> int:
        return self.local_offset + self.local_numel

    @property
    def is_fully_local(self) -> bool:
        return self.has_local_view and self.local_numel == self.numel

    @property
    def is_partially_local(self) -> bool:
        return self.has_local_view and self.local_numel < self.numel


def compute_cluster_layout(param_numels, param_shapes, param_dtypes, dp_rank: int, dp_size: int,
                           align: int = 1):
    """Returns (layouts, shard_size, pad_size).  ``align`` rounds the shard size up to a
    multiple of that many elements (vectorised peer reductions need 16-byte slices)."""
    if not (len(param_numels) == len(param_shapes) == len(param_dtypes)):
        raise ValueError("param_numels, param_shapes and param_dtypes differ in length")
    total = sum(param_numels)
    unit = dp_size * max(1, int(align))
    padded = ((total + unit - 1) // unit) * unit
    shard = padded // dp_size
    lo, hi = dp_rank * shard, dp_rank * shard + shard
    layouts = []
    off = 0
    for n, shp, dt in zip(param_numels, param_shapes, param_dtypes):
        a, b = max(off, lo), min(off + n, hi)
        if a < b:
            layouts.append(ClusterShardingSpec(off, n, shp, dt, True, a - lo, b - a))
        else:
            layouts.append(ClusterShardingSpec(off, n, shp, dt, False, 0, 0))
        off += n
    return layouts, shard, padded - total
