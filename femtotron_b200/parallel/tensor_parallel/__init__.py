from .comm_ops import (CopyToTPRegion, GatherFromSequenceParallelRegion, GatherFromTPRegion,
                       ReduceFromTPRegion, ReduceScatterToSequenceParallelRegion, ScatterToTPRegion)
from .embedding import VocabParallelEmbedding
from .linear import ColumnParallelLinear, RowParallelLinear

__all__ = [
    "ColumnParallelLinear", "RowParallelLinear", "VocabParallelEmbedding", "CopyToTPRegion",
    "ReduceFromTPRegion", "GatherFromTPRegion", "ScatterToTPRegion",
    "GatherFromSequenceParallelRegion", "ReduceScatterToSequenceParallelRegion",
]
