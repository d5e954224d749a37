"""Autograd-aware tensor-parallel communication regions (Megatron-style).

Plain TP (reference femtotron/parallel/tensor_parallel/comm_ops.py:6-183):
  CopyToTPRegion       fwd identity        bwd all-reduce SUM
  ReduceFromTPRegion   fwd all-reduce SUM  bwd identity
  GatherFromTPRegion   fwd all-gather(dim) bwd take own slice
  ScatterToTPRegion    fwd take own slice  bwd all-gather(dim)
    (the reference's scatter is broken: its chunk is not divided by tp and its backward
     returns one value for three inputs; this one is correct)

Sequence parallelism over the TP group (token dim 0 of a [T, H] activation):
  GatherFromSequenceParallelRegion      fwd all-gather(0)     bwd reduce-scatter(0)
  ReduceScatterToSequenceParallelRegion fwd reduce-scatter(0) bwd all-gather(0)
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch.autograd import Function


def _ws(group) -> int:
    return 1 if group is None else dist.get_world_size(group)


def _all_gather(x: torch.Tensor, group, dim: int) -> torch.Tensor:
    ws = _ws(group)
    if ws == 1:
        return x
    x = x.contiguous()
    if dim == 0:
        out = torch.empty((ws * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x, group=group)
        return out
    xt = x.movedim(dim, 0).contiguous()
    out = torch.empty((ws * xt.shape[0],) + tuple(xt.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, xt, group=group)
    return out.movedim(0, dim).contiguous()


def _reduce_scatter(x: torch.Tensor, group, dim: int = 0) -> torch.Tensor:
    ws = _ws(group)
    if ws == 1:
        return x
    xt = x.movedim(dim, 0).contiguous() if dim != 0 else x.contiguous()
    if xt.shape[0] % ws != 0:
        raise ValueError(f"reduce-scatter dim {xt.shape[0]} not divisible by {ws}")
    out = torch.empty((xt.shape[0] // ws,) + tuple(xt.shape[1:]), dtype=x.dtype, device=x.device)
    dist.reduce_scatter_tensor(out, xt, op=dist.ReduceOp.SUM, group=group)
    return out.movedim(0, dim).contiguous() if dim != 0 else out


def _own_slice(x: torch.Tensor, group, dim: int) -> torch.Tensor:
    ws = _ws(group)
    if ws == 1:
        return x
    if x.shape[dim] % ws != 0:
        raise ValueError(f"dim {dim} size {x.shape[dim]} not divisible by tp={ws}")
    chunk = x.shape[dim] // ws
    return x.narrow(dim, dist.get_rank(group) * chunk, chunk).contiguous()


def _all_reduce(x: torch.Tensor, group) -> torch.Tensor:
    if _ws(group) == 1:
        return x
    x = x.contiguous().clone()
    dist.all_reduce(x, group=group)
    return x


class CopyToTPRegion(Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):
        return _all_reduce(g, ctx.group), None


class ReduceFromTPRegion(Function):
    @staticmethod
    def forward(ctx, x, group):
        return _all_reduce(x, group)

    @staticmethod
    def backward(ctx, g):
        return g, None


class GatherFromTPRegion(Function):
    @staticmethod
    def forward(ctx, x, group, dim=-1):
        d = dim % x.dim()
        ctx.group, ctx.dim = group, d
        return _all_gather(x, group, d)

    @staticmethod
    def backward(ctx, g):
        return _own_slice(g, ctx.group, ctx.dim), None, None


class ScatterToTPRegion(Function):
    @staticmethod
    def forward(ctx, x, group, dim=-1):
        d = dim % x.dim()
        ctx.group, ctx.dim = group, d
        return _own_slice(x, group, d)

    @staticmethod
    def backward(ctx, g):
        return _all_gather(g, ctx.group, ctx.dim), None, None


class GatherFromSequenceParallelRegion(Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _all_gather(x, group, 0)

    @staticmethod
    def backward(ctx, g):
        return _reduce_scatter(g, ctx.group, 0), None


class ReduceScatterToSequenceParallelRegion(Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return _reduce_scatter(x, group, 0)

    @staticmethod
    def backward(ctx, g):
        return _all_gather(g, ctx.group, 0), None


def copy_to_tp(x, group):
    return x if _ws(group) == 1 else CopyToTPRegion.apply(x, group)


def reduce_from_tp(x, group):
    return x if _ws(group) == 1 else ReduceFromTPRegion.apply(x, group)


def gather_from_tp(x, group, dim=-1):
    return x if _ws(group) == 1 else GatherFromTPRegion.apply(x, group, dim)


def scatter_to_tp(x, group, dim=-1):
    return x if _ws(group) == 1 else ScatterToTPRegion.apply(x, group, dim)


def gather_from_sp(x, group):
    return x if _ws(group) == 1 else GatherFromSequenceParallelRegion.apply(x, group)


def reduce_scatter_to_sp(x, group):
    return x if _ws(group) == 1 else ReduceScatterToSequenceParallelRegion.apply(x, group)
