"""How each kind of parallel rule slices a checkpoint tensor for one TP rank (reference
femtotron/model/shard_loader.py:43-64): column and vocab-embedding weights split dim 0,
row-parallel weights split dim 1 (their bias is replicated), everything else is replicated.
Loaders work on safetensors slice handles (``get_shape()`` + slicing) and on tensors."""
from __future__ import annotations

from typing import Callable, Protocol


class ShardLoader(Protocol):
    def load(self, handle, rank: int, world_size: int): ...


class ReplicateLoader:
    def load(self, handle, rank, world_size):
        return handle[:]


class DimShardLoader:
    def __init__(self, dim: int):
        self.dim = dim

    def load(self, handle, rank, world_size):
        shape = handle.get_shape() if hasattr(handle, "get_shape") else list(handle.shape)
        size = shape[self.dim]
        if size % world_size != 0:
            raise ValueError(f"dim {self.dim} of size {size} not divisible by {world_size}")
        chunk = size // world_size
        sl = [slice(None)] * len(shape)
        sl[self.dim] = slice(rank * chunk, (rank + 1) * chunk)
        return handle[tuple(sl)]


_LOADER_REGISTRY: dict[str, Callable] = {}


def register_loader(kind: str):
    def deco(fn):
        _LOADER_REGISTRY[kind] = fn
        return fn
    return deco


@register_loader("column")
def _column(rule, suffix):
    return DimShardLoader(0)


@register_loader("row")
def _row(rule, suffix):
    return ReplicateLoader() if suffix == ".bias" else DimShardLoader(1)


@register_loader("vocab_embed")
def _vocab(rule, suffix):
    return DimShardLoader(0)


@register_loader("replicate")
def _replicate(rule, suffix):
    return ReplicateLoader()


def resolve_loader(rule, name: str):
    if rule is None:
        return ReplicateLoader()
    suffix = "." + name.rsplit(".", 1)[-1] if "." in name else ""
    fn = _LOADER_REGISTRY.get(rule.parallel_type)
    if fn is None:
        raise ValueError(f"no shard loader for parallel type {rule.parallel_type!r}")
    return fn(rule, suffix)
