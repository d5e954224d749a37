"""Vocab-parallel embedding (reference femtotron/parallel/tensor_parallel/embedding.py:12-126).

Each TP rank holds rows [rank*V/tp, (rank+1)*V/tp) of the table; out-of-shard ids give zero
rows, and the TP reduction completes the lookup: an all-reduce in plain TP, a reduce-scatter
over tokens with sequence parallelism.  The lookup and its scatter-add backward are sm_100a
kernels (the backward accumulates straight into the fp32 gradient buffer).

Note: the reference computes vocab_start from the LOCAL vocab size
(rank * vocab_size, with vocab_size already divided), which is what this class does too.
"""
from __future__ import annotations

import torch
from torch import nn

from femtotron_b200.ops.functional import EmbeddingFn
from femtotron_b200.parallel.tensor_parallel import comm_ops as C


class VocabParallelEmbedding(nn.Module):
    def __init__(self, vocab_size: int, hidden_size: int, parallel_ctx, parallel_dim_name="tp",
                 device=None, dtype=None, sequence_parallel: bool = False):
        super().__init__()
        self.group = parallel_ctx.get_group(parallel_dim_name)
        self.world_size = parallel_ctx.get_size(parallel_dim_name)
        self.rank = parallel_ctx.get_rank(parallel_dim_name)
        self.num_embeddings = vocab_size
        self.embedding_dim = hidden_size
        self.weight = nn.Parameter(torch.empty(vocab_size, hidden_size, device=device, dtype=dtype))
        self.vocab_start_idx = self.rank * vocab_size
        self.vocab_end_idx = (self.rank + 1) * vocab_size
        self.sequence_parallel = sequence_parallel
        if device is None or torch.device(device).type != "meta":
            nn.init.normal_(self.weight, std=0.02)

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        out = EmbeddingFn.apply(input_ids, self.weight, self.vocab_start_idx)
        if self.sequence_parallel:
            return C.reduce_scatter_to_sp(out.reshape(-1, out.shape[-1]), self.group)
        return C.reduce_from_tp(out, self.group)

    @classmethod
    def from_embedding(cls, embedding: nn.Embedding, parallel_ctx, rule):
        ws = parallel_ctx.get_size("tp")
        if embedding.num_embeddings % ws != 0:
            raise ValueError(f"vocab {embedding.num_embeddings} not divisible by tp={ws}")
        return cls(embedding.num_embeddings // ws, embedding.embedding_dim, parallel_ctx,
                   device=embedding.weight.device, dtype=embedding.weight.dtype,
                   sequence_parallel=rule.kwargs.get("sequence_parallel", False))

    @classmethod
    def from_embedding_temp(cls, embedding: nn.Embedding, parallel_ctx):
        ws, r = parallel_ctx.get_size("tp"), parallel_ctx.get_rank("tp")
        chunk = embedding.num_embeddings // ws
        m = cls(chunk, embedding.embedding_dim, parallel_ctx, device=embedding.weight.device,
                dtype=embedding.weight.dtype)
        with torch.no_grad():
            m.weight.copy_(embedding.weight[r * chunk:(r + 1) * chunk])
        return m
