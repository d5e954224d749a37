"""Assign decoder layers to pipeline stages: uniform (earlier stages take the remainder) or
manual per-stage counts (reference femtotron/parallel/pipeline_parallel/partition.py:19-115)."""
from __future__ import annotations


def partition_layers(num_layers: int, pp_size: int, strategy: str = "uniform", **kwargs) -> list[range]:
    if pp_size < 1:
        raise ValueError(f"pp_size must be >= 1, got {pp_size}")
    if num_layers < pp_size:
        raise ValueError(f"num_layers={num_layers} < pp_size={pp_size}; need >= 1 layer per stage")
    if strategy == "uniform":
        base, rem = divmod(num_layers, pp_size)
        counts = [base + (1 if i < rem else 0) for i in range(pp_size)]
    elif strategy == "manual":
        counts = kwargs.get("layer_counts")
        if counts is None:
            raise ValueError("strategy='manual' requires layer_counts")
        if len(counts) != pp_size:
            raise ValueError(f"layer_counts has {len(counts)} entries, expected pp_size={pp_size}")
        if any(c < 1 for c in counts):
            raise ValueError(f"each stage needs >= 1 layer, got {list(counts)}")
        if sum(counts) != num_layers:
            raise ValueError(f"sum(layer_counts)={sum(counts)} != num_layers={num_layers}")
    else:
        raise NotImplementedError(f"unknown partition strategy {strategy!r} (uniform, manual)")
    out, s = [], 0
    for c in counts:
        out.append(range(s, s + c))
        s += c
    return out
