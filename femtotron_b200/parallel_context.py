"""N-dimensional process topology: a rank grid over (pp, dp, ep, cp, tp) with one process
group per dimension.

Behaviour matches the reference topology object (femtotron/parallel_context.py:12-206):
dimensions are normalised to the fixed order pp, dp, ep, cp, tp (missing ones get size 1),
ranks are laid out row-major so tp is the innermost (adjacent GPUs), and every rank takes
part in creating every group of every dimension.

Additions for B200: the context also owns per-group communication resources that the
fused compute+collective kernels need (symmetric peer buffers over NVLink), created lazily
through :meth:`symmetric_heap`.
"""
from __future__ import annotations

import math
from collections import OrderedDict

import torch
import torch.distributed as dist

SUPPORTED_PARALLEL_DIMS = ["pp", "dp", "ep", "cp", "tp"]


class ParallelContext:
    def __init__(self, parallel_dims: "OrderedDict[str, int] | dict[str, int]", *,
                 world_size: int | None = None, world_rank: int | None = None):
        self.parallel_dims = self._normalize_parallel_dims(parallel_dims)
        self.world_size = world_size if world_size is not None else dist.get_world_size()
        self.world_rank = world_rank if world_rank is not None else dist.get_rank()
        self.dim_names = list(self.parallel_dims.keys())
        self.dim_sizes = list(self.parallel_dims.values())
        if math.prod(self.dim_sizes) != self.world_size:
            raise ValueError(f"product of parallel dims {math.prod(self.dim_sizes)} != "
                             f"world_size {self.world_size}")
        # rank r sits at the row-major position of r, so the last dimension (tp) is the
        # fastest-varying one and tensor-parallel peers are adjacent GPUs
        self.rank_grid = torch.arange(self.world_size).reshape(self.dim_sizes)
        self.local_coord = [int(c) for c in torch.nonzero(self.rank_grid == self.world_rank)[0]]
        self.groups: dict[str, dist.ProcessGroup | None] = {}
        self.ranks_in: dict[str, list[int]] = {}
        self._heaps: dict = {}
        create = dist.is_available() and dist.is_initialized()
        for d, name in enumerate(self.dim_names):
            self.groups[name], self.ranks_in[name] = self._groups_of_dim(d, create)

    @staticmethod
    def _normalize_parallel_dims(parallel_dims) -> "OrderedDict[str, int]":
        for name in parallel_dims:
            if name not in SUPPORTED_PARALLEL_DIMS:
                raise ValueError(f"unsupported parallel dim {name!r}; supported: {SUPPORTED_PARALLEL_DIMS}")
        out: OrderedDict[str, int] = OrderedDict()
        for name in SUPPORTED_PARALLEL_DIMS:
            size = int(parallel_dims.get(name, 1))
            if size < 1:
                raise ValueError(f"parallel dim {name} must be >= 1, got {size}")
            out[name] = size
        return out

    def slices_of_dim(self, d: int) -> list[list[int]]:
        """Every group of dimension d: moving d to the last axis makes each row of the grid
        one set of ranks that differ only in their coordinate along d."""
        rows = self.rank_grid.movedim(d, -1).reshape(-1, self.dim_sizes[d])
        return [[int(r) for r in row] for row in rows]

    def _groups_of_dim(self, d: int, create: bool):
        """(this rank's group, its ranks) along dimension d.  ``new_group`` is collective over
        the world, so every rank creates every slice, in the same order."""
        mine = (None, None)
        for ranks in self.slices_of_dim(d):
            group = dist.new_group(ranks) if create else None
            if self.world_rank in ranks:
                mine = (group, ranks)
        return mine

    def _neighbor_along(self, dim_name: str, step: int) -> int | None:
        ranks = self.ranks_in[dim_name]
        j = ranks.index(self.world_rank) + step
        return ranks[j] if 0 <= j < len(ranks) else None

    # ---------------------------------------------------------------- generic accessors
    def get_rank(self, dim_name: str) -> int:
        return self.local_coord[self.dim_names.index(dim_name)]

    def get_size(self, dim_name: str) -> int:
        return self.parallel_dims[dim_name]

    def get_group(self, dim_name: str):
        return self.groups[dim_name]

    def get_ranks_in_group(self, dim_name: str) -> list[int]:
        return self.ranks_in[dim_name]

    # ---------------------------------------------------------------- shortcuts
    @property
    def dp_rank(self): return self.get_rank("dp")
    @property
    def tp_rank(self): return self.get_rank("tp")
    @property
    def pp_rank(self): return self.get_rank("pp")
    @property
    def dp_size(self): return self.get_size("dp")
    @property
    def tp_size(self): return self.get_size("tp")
    @property
    def pp_size(self): return self.get_size("pp")
    @property
    def dp_group(self): return self.get_group("dp")
    @property
    def tp_group(self): return self.get_group("tp")
    @property
    def pp_group(self): return self.get_group("pp")

    def get_prev_rank_in(self, dim_name: str) -> int | None:
        return self._neighbor_along(dim_name, -1)

    def get_next_rank_in(self, dim_name: str) -> int | None:
        return self._neighbor_along(dim_name, +1)

    @property
    def pp_prev_rank(self): return self.get_prev_rank_in("pp")
    @property
    def pp_next_rank(self): return self.get_next_rank_in("pp")

    # ---------------------------------------------------------------- device
    @property
    def device(self) -> torch.device:
        if torch.cuda.is_available():
            return torch.device("cuda", torch.cuda.current_device())
        return torch.device("cpu")

    def symmetric_heap(self, dim_name: str, nbytes: int):
        """Per-group symmetric buffer (one allocation per rank, every peer mapped) used by
        the fused NVLink kernels.  Created on first use and cached per (dim, size)."""
        from femtotron_b200.parallel.symm import SymmetricHeap
        key = (dim_name, nbytes)
        heap = self._heaps.get(key)
        if heap is None:
            heap = SymmetricHeap(self.get_group(dim_name), self.get_ranks_in_group(dim_name),
                                 nbytes, self.device)
            self._heaps[key] = heap
        return heap

    def close(self) -> None:
        for h in self._heaps.values():
            h.close()
        self._heaps.clear()

    def __repr__(self) -> str:
        dims = ", ".join(f"{k}={v}" for k, v in self.parallel_dims.items())
        return f"ParallelContext({dims}, rank={self.world_rank}, coord={self.local_coord})"
