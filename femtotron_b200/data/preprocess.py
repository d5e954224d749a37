"""Tokenise a text dataset, append EOS, concatenate and pack into [N, seq_len] (reference
femtotron/data/preprocess.py:9-71).  Needs `datasets`/tokenizer access (network or a local
cache); the training paths of this package also run on SyntheticTokens without it."""
from __future__ import annotations

import torch


def preprocess(dataset_name: str, tokenizer_name: str, output_path: str, seq_len: int,
               split: str = "train", num_samples: int | None = None, text_field: str = "text"):
    from datasets import load_dataset  # optional dependency
    from transformers import AutoTokenizer
    tok = AutoTokenizer.from_pretrained(tokenizer_name)
    ds = load_dataset(dataset_name, split=split)
    if num_samples is not None:
        ds = ds.select(range(min(num_samples, len(ds))))
    eos = tok.eos_token_id
    buf: list[int] = []
    rows: list[list[int]] = []
    for ex in ds:
        buf.extend(tok(ex[text_field], add_special_tokens=False)["input_ids"] + [eos])
        while len(buf) >= seq_len:
            rows.append(buf[:seq_len])
            buf = buf[seq_len:]
    data = torch.tensor(rows, dtype=torch.int32 if tok.vocab_size < 2 ** 31 else torch.long)
    torch.save(data, output_path)
    return data
