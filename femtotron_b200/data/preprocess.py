"""Tokenise a text dataset, append EOS after every document, concatenate and pack into
[N, seq_len] rows saved with torch.save (reference femtotron/data/preprocess.py:9-71).

Sources: a Hugging Face dataset name (``datasets.load_dataset``, needs the hub or a local
cache), or a local file — ``.txt`` (one document per line), ``.jsonl`` (one JSON object per
line, text in ``text_field``) — or a directory of such files.  Tokenizers: a Hugging Face
name or local path (``AutoTokenizer``), or ``"bytes"``: UTF-8 bytes as ids 0..255 with EOS =
256 (vocabulary 257), which needs nothing from the network.  The training paths of this
package also run on SyntheticTokens without any of this.
"""
from __future__ import annotations

import json
import os
from typing import Iterable, Iterator

import torch

BYTES_EOS = 256
BYTES_VOCAB = 257


def _local_docs(path: str, text_field: str) -> Iterator[str]:
    files = [path] if os.path.isfile(path) else sorted(
        os.path.join(path, f) for f in os.listdir(path) if f.endswith((".txt", ".jsonl")))
    for fn in files:
        with open(fn, encoding="utf-8") as f:
            for line in f:
                line = line.rstrip("\n")
                if not line:
                    continue
                yield json.loads(line)[text_field] if fn.endswith(".jsonl") else line


def iter_documents(dataset_name: str, split: str = "train", num_samples: int | None = None,
                   text_field: str = "text") -> Iterator[str]:
    """Documents of a local file / directory or of a Hugging Face dataset, at most
    `num_samples` of them."""
    if os.path.exists(dataset_name):
        src: Iterable[str] = _local_docs(dataset_name, text_field)
    else:
        from datasets import load_dataset  # optional dependency
        ds = load_dataset(dataset_name, split=split)
        if num_samples is not None:
            ds = ds.select(range(min(num_samples, len(ds))))
        src = (ex[text_field] for ex in ds)
    for i, doc in enumerate(src):
        if num_samples is not None and i >= num_samples:
            return
        yield doc


def make_tokenizer(tokenizer_name: str):
    """(encode: str -> list[int], eos_id, vocab_size)."""
    if tokenizer_name == "bytes":
        return (lambda s: list(s.encode("utf-8"))), BYTES_EOS, BYTES_VOCAB
    from transformers import AutoTokenizer
    tok = AutoTokenizer.from_pretrained(tokenizer_name)
    return (lambda s: tok(s, add_special_tokens=False)["input_ids"]), tok.eos_token_id, len(tok)


def pack_tokens(docs: Iterable[list[int]], eos: int, seq_len: int) -> torch.Tensor:
    """Concatenate documents, each followed by `eos`, into full rows of `seq_len` tokens (the
    incomplete tail is dropped)."""
    buf: list[int] = []
    rows: list[list[int]] = []
    for ids in docs:
        buf.extend(ids)
        buf.append(eos)
        while len(buf) >= seq_len:
            rows.append(buf[:seq_len])
            buf = buf[seq_len:]
    return torch.tensor(rows, dtype=torch.int64).reshape(-1, seq_len)


def preprocess(dataset_name: str, tokenizer_name: str, output_path: str, seq_len: int,
               split: str = "train", num_samples: int | None = None, text_field: str = "text"):
    encode, eos, vocab = make_tokenizer(tokenizer_name)
    data = pack_tokens((encode(d) for d in iter_documents(dataset_name, split, num_samples, text_field)),
                       eos, seq_len)
    data = data.to(torch.int32 if vocab < 2 ** 31 else torch.int64)
    d = os.path.dirname(os.path.abspath(output_path))
    os.makedirs(d, exist_ok=True)
    torch.save(data, output_path)
    return data
