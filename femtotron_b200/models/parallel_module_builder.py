"""Registry of builders that turn a plain module into its parallel counterpart, keyed by
(rule kind, source module type) with an MRO fallback (reference
femtotron/model/parallel_module_builder.py:20-43)."""
from __future__ import annotations

from typing import Callable

from torch import nn

from femtotron_b200.parallel.tensor_parallel.embedding import VocabParallelEmbedding
from femtotron_b200.parallel.tensor_parallel.linear import ColumnParallelLinear, RowParallelLinear

ParallelBuilder = Callable[[nn.Module, object, object], nn.Module]
_BUILDER_REGISTRY: dict[tuple[str, type], ParallelBuilder] = {}


def register_builder(kind: str, source_type: type):
    def deco(fn):
        _BUILDER_REGISTRY[(kind, source_type)] = fn
        return fn
    return deco


@register_builder("column", nn.Linear)
def _build_column(old, ctx, rule):
    return ColumnParallelLinear.from_linear(old, ctx, rule)


@register_builder("row", nn.Linear)
def _build_row(old, ctx, rule):
    return RowParallelLinear.from_linear(old, ctx, rule)


@register_builder("vocab_embed", nn.Embedding)
def _build_vocab(old, ctx, rule):
    return VocabParallelEmbedding.from_embedding(old, ctx, rule)


@register_builder("replicate", nn.Module)
def _build_replicate(old, ctx, rule):
    return old
