"""Column- and row-parallel linear layers, optionally sequence parallel.

Same constructor contract as the reference (femtotron/parallel/tensor_parallel/linear.py:14-272):
`out_features` of a ColumnParallelLinear and `in_features` of a RowParallelLinear are the
LOCAL (already divided) sizes; the weight is [out, in] like nn.Linear.

Compute runs through the fused sm_100a GEMM (`femtotron_b200.ops.functional.linear`), whose
weight gradient is accumulated in place.  With ``sequence_parallel=True`` the column layer
all-gathers its token-sharded input (AG -> GEMM) and the row layer reduce-scatters its
output (GEMM -> RS) instead of the all-reduces of plain TP.
"""
from __future__ import annotations

import torch
from torch import nn

from femtotron_b200.ops.functional import linear as _linear
from femtotron_b200.parallel.tensor_parallel import comm_ops as C


class ColumnParallelLinear(nn.Module):
    def __init__(self, in_features: int, out_features: int, parallel_ctx, parallel_dim_name="tp",
                 bias=False, gather_output=False, device=None, dtype=None,
                 sequence_parallel: bool = False):
        super().__init__()
        self.group = parallel_ctx.get_group(parallel_dim_name)
        self.world_size = parallel_ctx.get_size(parallel_dim_name)
        self.rank = parallel_ctx.get_rank(parallel_dim_name)
        self.in_features = in_features
        self.out_features = out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features, device=device, dtype=dtype))
        self.bias = nn.Parameter(torch.zeros(out_features, device=device, dtype=dtype)) if bias else None
        self.parallel_ctx = parallel_ctx
        self.gather_output = gather_output
        self.sequence_parallel = sequence_parallel
        if device is None or torch.device(device).type != "meta":
            nn.init.normal_(self.weight, std=0.02)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.sequence_parallel:
            x = C.gather_from_sp(x.reshape(-1, x.shape[-1]), self.group)
        else:
            x = C.copy_to_tp(x, self.group)
        y = _linear(x, self.weight)
        if self.bias is not None:
            y = y + self.bias
        if self.gather_output:
            y = C.gather_from_tp(y, self.group, -1)
        return y

    @classmethod
    def from_linear(cls, linear: nn.Linear, parallel_ctx, rule) -> "ColumnParallelLinear":
        ws = parallel_ctx.tp_size
        if linear.out_features % ws != 0:
            raise ValueError(f"out_features {linear.out_features} not divisible by tp={ws}")
        return cls(linear.in_features, linear.out_features // ws, parallel_ctx,
                   bias=linear.bias is not None,
                   gather_output=rule.kwargs.get("gather_output", False),
                   sequence_parallel=rule.kwargs.get("sequence_parallel", False),
                   device=linear.weight.device, dtype=linear.weight.dtype)

    @classmethod
    def from_linear_temp(cls, linear: nn.Linear, parallel_ctx, gather_output=False,
                         sequence_parallel=False):
        """Copy this rank's row slice of a full nn.Linear (tests and conversions)."""
        ws, r = parallel_ctx.get_size("tp"), parallel_ctx.get_rank("tp")
        out = linear.out_features // ws
        m = cls(linear.in_features, out, parallel_ctx, bias=linear.bias is not None,
                gather_output=gather_output, sequence_parallel=sequence_parallel,
                device=linear.weight.device, dtype=linear.weight.dtype)
        with torch.no_grad():
            m.weight.copy_(linear.weight[r * out:(r + 1) * out])
            if m.bias is not None:
                m.bias.copy_(linear.bias[r * out:(r + 1) * out])
        return m


class RowParallelLinear(nn.Module):
    def __init__(self, in_features: int, out_features: int, parallel_ctx, parallel_dim_name="tp",
                 bias=False, scatter_input=False, device=None, dtype=None,
                 sequence_parallel: bool = False):
        super().__init__()
        self.group = parallel_ctx.get_group(parallel_dim_name)
        self.world_size = parallel_ctx.get_size(parallel_dim_name)
        self.rank = parallel_ctx.get_rank(parallel_dim_name)
        self.in_features = in_features
        self.out_features = out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features, device=device, dtype=dtype))
        self.bias = nn.Parameter(torch.zeros(out_features, device=device, dtype=dtype)) if bias else None
        self.parallel_ctx = parallel_ctx
        self.scatter_input = scatter_input
        self.sequence_parallel = sequence_parallel
        if device is None or torch.device(device).type != "meta":
            nn.init.normal_(self.weight, std=0.02)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.scatter_input:
            x = C.scatter_to_tp(x, self.group, -1)
        y = _linear(x, self.weight)
        if self.sequence_parallel:
            y = C.reduce_scatter_to_sp(y.reshape(-1, y.shape[-1]), self.group)
        else:
            y = C.reduce_from_tp(y, self.group)
        if self.bias is not None:
            y = y + self.bias
        return y

    @classmethod
    def from_linear(cls, linear: nn.Linear, parallel_ctx, rule) -> "RowParallelLinear":
        ws = parallel_ctx.tp_size
        # (the reference checks out_features here, femtotron/parallel/tensor_parallel/linear.py:224;
        #  the sharded dimension of a row-parallel layer is in_features)
        if linear.in_features % ws != 0:
            raise ValueError(f"in_features {linear.in_features} not divisible by tp={ws}")
        return cls(linear.in_features // ws, linear.out_features, parallel_ctx,
                   bias=linear.bias is not None,
                   scatter_input=rule.kwargs.get("scatter_input", False),
                   sequence_parallel=rule.kwargs.get("sequence_parallel", False),
                   device=linear.weight.device, dtype=linear.weight.dtype)

    @classmethod
    def from_linear_temp(cls, linear: nn.Linear, parallel_ctx, scatter_input=False,
                         sequence_parallel=False):
        ws, r = parallel_ctx.get_size("tp"), parallel_ctx.get_rank("tp")
        inf = linear.in_features // ws
        m = cls(inf, linear.out_features, parallel_ctx, bias=linear.bias is not None,
                scatter_input=scatter_input, sequence_parallel=sequence_parallel,
                device=linear.weight.device, dtype=linear.weight.dtype)
        with torch.no_grad():
            m.weight.copy_(linear.weight[:, r * inf:(r + 1) * inf])
            if m.bias is not None:
                m.bias.copy_(linear.bias)
        return m
