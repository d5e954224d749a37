"""Data-parallel sampler.

The sample order is an interface shared with the reference (femtotron/data/distributed_sampler.py:
8-110), so that runs and checkpoints carry over between the two frameworks: per epoch one global
permutation from a generator seeded with ``seed + epoch``, cut to a multiple of the DP size
(``drop_last``) or wrapped around to one, and split into contiguous DP-rank blocks, so
tensor- and pipeline-parallel peers (same dp_rank) read the same samples.  A resume offset
skips the samples a checkpointed run already consumed.

The order is computed by :func:`dp_shard_order`, a pure function of those settings; the
sampler only keeps the epoch and the offset.
"""
from __future__ import annotations

import torch
from torch.utils.data import Sampler


def dp_shard_order(dataset_size: int, dp_rank: int, dp_size: int, seed: int, epoch: int,
                   shuffle: bool = True, drop_last: bool = True) -> torch.Tensor:
    """Indices read by `dp_rank` in `epoch`, in order (int64 tensor)."""
    if shuffle:
        order = torch.randperm(dataset_size, generator=torch.Generator().manual_seed(seed + epoch))
    else:
        order = torch.arange(dataset_size)
    if drop_last:
        order = order[: dataset_size - dataset_size % dp_size]
    else:
        # wrap around to the next multiple of dp_size (with fewer samples than ranks the wrap
        # cannot fill it, and the blocks are as long as what there is allows)
        short = -dataset_size % dp_size
        order = torch.cat([order, order[:short]])
    block = order.numel() // dp_size
    return order[dp_rank * block:(dp_rank + 1) * block]


class DistributedSampler(Sampler[int]):
    def __init__(self, dataset_size: int, parallel_ctx, *, seed: int = 42, shuffle: bool = True,
                 drop_last: bool = True):
        if dataset_size <= 0:
            raise ValueError("empty dataset")
        if not 0 <= parallel_ctx.dp_rank < parallel_ctx.dp_size:
            raise ValueError("dp_rank out of range")
        self.dataset_size = dataset_size
        self.dp_rank, self.dp_size = parallel_ctx.dp_rank, parallel_ctx.dp_size
        self.seed, self.shuffle, self.drop_last = seed, shuffle, drop_last
        self.epoch = 0
        self._consumed = 0          # samples of this epoch already read (resume offset)

    def set_epoch(self, epoch: int) -> None:
        """Start `epoch` from its first sample."""
        self.epoch, self._consumed = epoch, 0

    def advance(self, n: int) -> None:
        """Mark n more samples of the epoch as consumed."""
        self._consumed += n

    def __iter__(self):
        order = dp_shard_order(self.dataset_size, self.dp_rank, self.dp_size, self.seed,
                               self.epoch, self.shuffle, self.drop_last)
        return iter(order[self._consumed:].tolist())

    def __len__(self) -> int:
        per_rank = -(-self.dataset_size // self.dp_size) if not self.drop_last else \
            self.dataset_size // self.dp_size
        return max(0, per_rank - self._consumed)

    # checkpoint format (dataloader_dp<d>.pt): the reference's keys
    def state_dict(self) -> dict:
        return {"epoch": self.epoch, "start_offset": self._consumed, "seed": self.seed,
                "dp_size": self.dp_size, "dataset_size": self.dataset_size}

    def load_state_dict(self, sd: dict) -> None:
        for key, mine, what in (("seed", self.seed, "sampler seed"),
                                ("dp_size", self.dp_size, "dp_size"),
                                ("dataset_size", self.dataset_size, "dataset size")):
            if sd[key] != mine:
                raise ValueError(f"{what} changed: checkpoint {sd[key]} vs current {mine}")
        self.epoch, self._consumed = sd["epoch"], sd["start_offset"]
