"""Data-parallel sampler (reference femtotron/data/distributed_sampler.py:8-110): one seeded
global permutation per epoch, sharded by dp_rank (so TP/PP peers read the same samples),
with a resumable consumption offset."""
from __future__ import annotations

import torch
from torch.utils.data import Sampler


class DistributedSampler(Sampler[int]):
    def __init__(self, dataset_size: int, parallel_ctx, *, seed: int = 42, shuffle: bool = True,
                 drop_last: bool = True):
        dp_rank, dp_size = parallel_ctx.dp_rank, parallel_ctx.dp_size
        if not 0 <= dp_rank < dp_size:
            raise ValueError("dp_rank out of range")
        if dataset_size <= 0:
            raise ValueError("empty dataset")
        self.dataset_size = dataset_size
        self.dp_rank, self.dp_size = dp_rank, dp_size
        self.seed, self.shuffle, self.drop_last = seed, shuffle, drop_last
        self.epoch = 0
        self._start_offset = 0

    def set_epoch(self, epoch: int) -> None:
        self.epoch = epoch
        self._start_offset = 0

    def _compute_indices(self) -> list[int]:
        if self.shuffle:
            g = torch.Generator()
            g.manual_seed(self.seed + self.epoch)
            idx = torch.randperm(self.dataset_size, generator=g).tolist()
        else:
            idx = list(range(self.dataset_size))
        if self.drop_last:
            idx = idx[: (self.dataset_size // self.dp_size) * self.dp_size]
        else:
            tot = ((self.dataset_size + self.dp_size - 1) // self.dp_size) * self.dp_size
            idx = idx + idx[: tot - self.dataset_size]
        per = len(idx) // self.dp_size
        return idx[self.dp_rank * per:(self.dp_rank + 1) * per]

    def __iter__(self):
        yield from self._compute_indices()[self._start_offset:]

    def __len__(self) -> int:
        full = self.dataset_size // self.dp_size if self.drop_last else \
            (self.dataset_size + self.dp_size - 1) // self.dp_size
        return max(0, full - self._start_offset)

    def state_dict(self) -> dict:
        return {"epoch": self.epoch, "start_offset": self._start_offset, "seed": self.seed,
                "dp_size": self.dp_size, "dataset_size": self.dataset_size}

    def load_state_dict(self, sd: dict) -> None:
        if sd["seed"] != self.seed:
            raise ValueError("sampler seed mismatch")
        if sd["dp_size"] != self.dp_size:
            raise ValueError(f"dp_size changed {sd['dp_size']} -> {self.dp_size}")
        if sd["dataset_size"] != self.dataset_size:
            raise ValueError("dataset changed")
        self.epoch = sd["epoch"]
        self._start_offset = sd["start_offset"]

    def advance(self, n: int) -> None:
        self._start_offset += n
