"""Batch collators (reference femtotron/data/collator.py:16-75).  Pretraining: fixed-length
packed samples stacked; labels are a copy of the ids (the model shifts internally).  SFT:
pad to the batch max (or a fixed length) and mask prompt/padding labels with -100."""
from __future__ import annotations

from typing import Protocol

import torch


class Collator(Protocol):
    def __call__(self, samples: list) -> dict[str, torch.Tensor]: ...


def simple_pretrain_collator(samples: list) -> dict[str, torch.Tensor]:
    if isinstance(samples[0], torch.Tensor):
        ids = torch.stack(samples).long()
    else:
        ids = torch.tensor(samples, dtype=torch.long)
    return {"input_ids": ids, "labels": ids.clone()}


class PadSftCollator:
    def __init__(self, pad_token_id: int, seq_len: int | None = None, ignore_index: int = -100):
        self.pad_token_id = pad_token_id
        self.seq_len = seq_len
        self.ignore_index = ignore_index

    def __call__(self, samples: list[dict]) -> dict[str, torch.Tensor]:
        L = self.seq_len or max(len(s["input_ids"]) for s in samples)
        ids, lab, mask = [], [], []
        for s in samples:
            x, y = list(s["input_ids"]), list(s["labels"])
            pad = L - len(x)
            if pad < 0:
                raise ValueError(f"sample length {len(x)} > target length {L}")
            ids.append(x + [self.pad_token_id] * pad)
            lab.append(y + [self.ignore_index] * pad)
            mask.append([1] * len(x) + [0] * pad)
        return {"input_ids": torch.tensor(ids, dtype=torch.long),
                "labels": torch.tensor(lab, dtype=torch.long),
                "attention_mask": torch.tensor(mask, dtype=torch.long)}
