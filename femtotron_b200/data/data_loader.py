"""Distributed data loader (reference femtotron/data/data_loader.py:17-142): sampler ->
dataset -> collator through a torch DataLoader (pinned memory, worker prefetch), with a
resumable state dict."""
from __future__ import annotations

from typing import Callable

import torch

from .distributed_sampler import DistributedSampler


class DistributedDataLoader:
    def __init__(self, dataset, parallel_ctx, micro_batch_size: int, collator: Callable | None = None,
                 sampler: DistributedSampler | None = None, *, seed: int = 42, num_workers: int = 2,
                 prefetch_factor: int = 2, pin_memory: bool = True, drop_last: bool = True):
        if collator is None:
            raise ValueError("a collator is required")
        self.parallel_ctx = parallel_ctx
        self.micro_batch_size = micro_batch_size
        self.dataset = dataset
        self.collator = collator
        self.num_workers = num_workers
        self.seed = seed
        self.sampler = sampler if sampler is not None else DistributedSampler(
            len(dataset), parallel_ctx, seed=seed, shuffle=True, drop_last=drop_last)
        self._inner = torch.utils.data.DataLoader(
            dataset, batch_size=micro_batch_size, sampler=self.sampler, collate_fn=collator,
            num_workers=num_workers, prefetch_factor=prefetch_factor if num_workers > 0 else None,
            pin_memory=pin_memory and torch.cuda.is_available(), drop_last=drop_last,
            persistent_workers=num_workers > 0)

    def __iter__(self):
        for batch in self._inner:
            self.sampler.advance(self.micro_batch_size)
            yield batch

    def __len__(self):
        return len(self._inner)

    def set_epoch(self, epoch: int):
        self.sampler.set_epoch(epoch)

    def state_dict(self) -> dict:
        return {"sampler": self.sampler.state_dict(), "seed": self.seed,
                "micro_batch_size": self.micro_batch_size}

    def load_state_dict(self, sd: dict) -> None:
        if sd["seed"] != self.seed:
            raise ValueError(f"seed mismatch on resume: ckpt={sd['seed']}, current={self.seed}")
        if sd["micro_batch_size"] != self.micro_batch_size:
            raise ValueError("micro_batch_size mismatch on resume")
        self.sampler.load_state_dict(sd["sampler"])

    @property
    def tokens_per_step(self) -> int:
        seq = self.dataset.shape[1] if hasattr(self.dataset, "shape") else 0
        return self.micro_batch_size * seq * self.parallel_ctx.dp_size
