"""Split a batch along dim 0 into equal micro-batches (views); reference:
femtotron/parallel/pipeline_parallel/microbatch.py:16."""
from __future__ import annotations

import torch


def split_microbatches(batch: torch.Tensor, num_microbatches: int) -> list[torch.Tensor]:
    if num_microbatches <= 0:
        raise ValueError(f"num_microbatches must be >= 1, got {num_microbatches}")
    if batch.shape[0] % num_microbatches != 0:
        raise ValueError(f"batch_size {batch.shape[0]} not divisible by num_microbatches {num_microbatches}")
    return list(batch.split(batch.shape[0] // num_microbatches, dim=0))
