"""Packed token dataset: a [num_samples, seq_len] int tensor saved with torch.save, opened
memory-mapped (reference femtotron/data/data_source.py:7-27)."""
from __future__ import annotations

import torch
from torch.utils.data import Dataset


class PackedDataset(Dataset):
    def __init__(self, path_or_tensor, mmap: bool = True):
        if isinstance(path_or_tensor, torch.Tensor):
            self.data = path_or_tensor
        else:
            self.data = torch.load(path_or_tensor, mmap=mmap, weights_only=True)
        if self.data.dim() != 2:
            raise ValueError(f"packed dataset must be 2-D [N, seq_len], got {tuple(self.data.shape)}")
        self.shape = self.data.shape

    @property
    def seq_len(self) -> int:
        return self.data.shape[1]

    def __len__(self) -> int:
        return self.data.shape[0]

    def __getitem__(self, idx: int) -> torch.Tensor:
        return self.data[idx]
