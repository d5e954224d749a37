"""Synthetic pretraining data: uniform random token ids of a fixed shape from a seed (the
data of the benchmark configurations), as a dataset usable with DistributedDataLoader."""
from __future__ import annotations

import torch
from torch.utils.data import Dataset


class SyntheticTokens(Dataset):
    def __init__(self, num_samples: int, seq_len: int, vocab_size: int, seed: int = 0):
        g = torch.Generator()
        g.manual_seed(seed)
        self.data = torch.randint(0, vocab_size, (num_samples, seq_len), generator=g, dtype=torch.long)
        self.shape = self.data.shape

    @property
    def seq_len(self) -> int:
        return self.data.shape[1]

    def __len__(self) -> int:
        return self.data.shape[0]

    def __getitem__(self, idx: int) -> torch.Tensor:
        return self.data[idx]
