"""Per-tensor data-parallel shard description (same fields as the reference's
femtotron/sharding/sharding_spec.py:7-48, kept identical because it is stored in
checkpoints): the tensor is flattened, padded to a multiple of world_size and split evenly."""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class ShardingSpec:
    full_shape: torch.Size
    flat_size: int          # padded flat size
    shard_size: int
    rank: int
    world_size: int
    pad_size: int = 0

    @property
    def shard_start(self) -> int:
        return self.rank * self.shard_size

    @property
    def shard_end(self) -> int:
        return self.shard_start + self.shard_size

    @classmethod
    def from_full(cls, full_tensor: torch.Tensor, rank: int, world_size: int) -> "ShardingSpec":
        n = full_tensor.numel()
        shard = (n + world_size - 1) // world_size
        return cls(full_shape=full_tensor.shape, flat_size=shard * world_size, shard_size=shard,
                   rank=rank, world_size=world_size, pad_size=shard * world_size - n)

    @classmethod
    def no_shard(cls, full_tensor: torch.Tensor) -> "ShardingSpec":
        n = full_tensor.numel()
        return cls(full_shape=full_tensor.shape, flat_size=n, shard_size=n, rank=0, world_size=1)
