"""LLaMA building blocks with HF-compatible parameter names and a fused B200 fast path.

Parameter names match transformers' LlamaDecoderLayer (self_attn.{q,k,v,o}_proj,
mlp.{gate,up,down}_proj, input_layernorm, post_attention_layernorm), so checkpoints,
parallel plans and loaders written for HF names apply unchanged.  The reference wraps the HF
layer itself (femtotron/model/llama_partial_model.py:35-39, 143-146); this file is a new
implementation whose forward runs:

    RMSNorm kernel -> one QKV GEMM + in-place RoPE -> causal GQA attention
      -> o_proj GEMM with the residual add in its epilogue
    RMSNorm kernel -> one gate|up GEMM with the SwiGLU epilogue
      -> down_proj GEMM with the residual add in its epilogue

When the projections are tensor-parallel modules, the matching TP/SP collectives wrap the
GEMMs.  If the projections are replaced by anything the fast path does not understand (a
bias, custom modules), the layer falls back to calling the submodules one by one.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from femtotron_b200.ops import functional as FN
from femtotron_b200.ops.kernels import rope_tables
from femtotron_b200.parallel.tensor_parallel import comm_ops as C
from femtotron_b200.parallel.tensor_parallel.linear import ColumnParallelLinear, RowParallelLinear
from femtotron_b200.utils.tracing import nvtx_range


def _cfg(config, name, default=None):
    v = getattr(config, name, None)
    return default if v is None else v


def head_dim_of(config) -> int:
    hd = getattr(config, "head_dim", None)
    return hd if hd else config.hidden_size // config.num_attention_heads


class LlamaRMSNorm(nn.Module):
    def __init__(self, hidden_size: int, eps: float = 1e-6, device=None, dtype=None):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size, device=device, dtype=dtype))
        self.variance_epsilon = eps
        # set under sequence parallelism: the TP group over which tokens are sharded
        self.sp_group = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.weight.dtype == x.dtype and x.dtype == torch.bfloat16 or not x.is_cuda:
            return FN.rms_norm(x, self.weight, self.variance_epsilon, self.sp_group)
        # non-bf16 CUDA input: PyTorch math (kept for generality; the model runs in bf16)
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.variance_epsilon)
        return self.weight * y.to(x.dtype)

    def extra_repr(self) -> str:
        return f"{self.weight.shape[0]}, eps={self.variance_epsilon}"


class LlamaRotaryEmbedding(nn.Module):
    """Holds the rotary configuration and serves cached (cos, sin) tables [max_pos, d/2].

    Tables are computed from the config on demand (not from a buffer), so models built on
    the meta device need no re-initialisation after materialisation."""

    def __init__(self, config, device=None):
        super().__init__()
        self.head_dim = head_dim_of(config)
        self.theta = float(_cfg(config, "rope_theta", None) or
                           (getattr(config, "rope_parameters", None) or {}).get("rope_theta", 10000.0))
        self.max_position_embeddings = int(_cfg(config, "max_position_embeddings", 2048))
        self._cache: dict = {}

    def tables(self, device, dtype, length: int):
        n = max(length, self.max_position_embeddings)
        key = (str(device), dtype, n)
        t = self._cache.get(key)
        if t is None:
            t = rope_tables(self.head_dim, n, self.theta, device, dtype)
            self._cache = {key: t}
        return t

    def forward(self, x: torch.Tensor, position_ids: torch.Tensor | None = None, seq_len: int | None = None):
        n = seq_len if seq_len is not None else (x.shape[1] if x.dim() == 3 else x.shape[0])
        if position_ids is not None:
            n = max(n, int(position_ids.max().item()) + 1) if position_ids.numel() else n
        cos, sin = self.tables(x.device, torch.bfloat16 if x.dtype != torch.float32 else x.dtype, n)
        return cos, sin


def causal_attention(qkv: torch.Tensor, B: int, S: int, nq: int, nkv: int, d: int) -> torch.Tensor:
    """Causal GQA attention over a packed [B*S, (nq+2nkv)*d] projection; returns [B*S, nq*d]."""
    from femtotron_b200.ops import attention as A
    if qkv.is_cuda:
        if A.USE_NATIVE and A.flash_available(d, S):
            return A.flash_attention(qkv, B, S, nq, nkv, d)
        A.note_fallback(d, S)
    q = qkv[:, : nq * d].view(B, S, nq, d).transpose(1, 2)
    k = qkv[:, nq * d:(nq + nkv) * d].view(B, S, nkv, d).transpose(1, 2)
    v = qkv[:, (nq + nkv) * d:(nq + 2 * nkv) * d].view(B, S, nkv, d).transpose(1, 2)
    o = F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=1.0 / math.sqrt(d),
                                       enable_gqa=(nq != nkv))
    return o.transpose(1, 2).reshape(B * S, nq * d)


def _tp_info(col: nn.Module):
    if isinstance(col, ColumnParallelLinear):
        return col.group if col.world_size > 1 else None, col.sequence_parallel and col.world_size > 1
    return None, False


def _plain_col(m: nn.Module) -> bool:
    return (type(m) is nn.Linear and m.bias is None) or (
        isinstance(m, ColumnParallelLinear) and m.bias is None and not m.gather_output)


def _plain_row(m: nn.Module) -> bool:
    return (type(m) is nn.Linear and m.bias is None) or (
        isinstance(m, RowParallelLinear) and m.bias is None and not m.scatter_input)


def _sp_comm(x: torch.Tensor, group, sp: bool, world: int):
    """The fused NVLink communication object for sequence parallelism on CUDA (else None)."""
    if not (sp and group is not None and x.is_cuda and x.dtype == torch.bfloat16):
        return None
    import os
    if os.environ.get("FT_TP_FUSED", "1") == "0":
        return None
    from femtotron_b200.parallel.tensor_parallel.fused import tp_fused_comm
    rows = x.reshape(-1, x.shape[-1]).shape[0]
    return tp_fused_comm(group, rows, x.shape[-1], x.device)


def _enter(x: torch.Tensor, group, sp: bool) -> torch.Tensor:
    if group is None:
        return x
    return C.gather_from_sp(x, group) if sp else C.copy_to_tp(x, group)


def _exit(y_partial_or_full, group, sp: bool, residual):
    """Finish a row-parallel projection: reduce across TP and add the residual."""
    if sp:
        return C.reduce_scatter_to_sp(y_partial_or_full, group) + residual
    return C.reduce_from_tp(y_partial_or_full, group) + residual


class LlamaAttention(nn.Module):
    def __init__(self, config, layer_idx: int, device=None, dtype=None):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.head_dim = head_dim_of(config)
        self.num_heads = config.num_attention_heads
        self.num_key_value_heads = _cfg(config, "num_key_value_heads", config.num_attention_heads)
        bias = bool(_cfg(config, "attention_bias", False))
        H = config.hidden_size
        d = self.head_dim
        self.q_proj = nn.Linear(H, self.num_heads * d, bias=bias, device=device, dtype=dtype)
        self.k_proj = nn.Linear(H, self.num_key_value_heads * d, bias=bias, device=device, dtype=dtype)
        self.v_proj = nn.Linear(H, self.num_key_value_heads * d, bias=bias, device=device, dtype=dtype)
        self.o_proj = nn.Linear(self.num_heads * d, H, bias=bias, device=device, dtype=dtype)

    def _fusable(self) -> bool:
        return all(_plain_col(m) for m in (self.q_proj, self.k_proj, self.v_proj)) and _plain_row(self.o_proj)

    def forward(self, x: torch.Tensor, position_embeddings, batch_shape, residual=None):
        """x: [T_local, H] tokens (T_local = B*S, or B*S/tp under sequence parallelism)."""
        B, S = batch_shape
        cos, sin, pos = position_embeddings
        d = self.head_dim
        nq = self.q_proj.weight.shape[0] // d
        nkv = self.k_proj.weight.shape[0] // d
        group, sp = _tp_info(self.q_proj)
        comm = _sp_comm(x, group, sp, 0) if self._fusable() else None
        if comm is not None and self.o_proj.weight.shape[0] == x.shape[-1]:
            from femtotron_b200.parallel.tensor_parallel.fused import SPColumnFn, SPRowFn
            qkv = SPColumnFn.apply(x, comm, "qkv_rope", (cos, sin, pos, nq + nkv, d, S),
                                   self.q_proj.weight, self.k_proj.weight, self.v_proj.weight)
            o = causal_attention(qkv, B, S, nq, nkv, d)
            return SPRowFn.apply(o, residual, comm, self.o_proj.weight)
        if self._fusable():
            xin = _enter(x, group, sp)
            qkv = FN.QKVRopeFn.apply(xin, cos, sin, pos, nq + nkv, d, S,
                                     self.q_proj.weight, self.k_proj.weight, self.v_proj.weight)
            o = causal_attention(qkv, B, S, nq, nkv, d)
            if group is None:
                return FN.linear(o, self.o_proj.weight, residual=residual) if residual is not None \
                    else FN.linear(o, self.o_proj.weight)
            y = FN.linear(o, self.o_proj.weight)
            return _exit(y, group, sp, residual if residual is not None else 0)
        # generic path: call the (possibly replaced) submodules
        q2 = self.q_proj(x).reshape(-1, nq * d)
        k2 = self.k_proj(x).reshape(-1, nkv * d)
        v2 = self.v_proj(x).reshape(-1, nkv * d)
        qk = _RopeFn.apply(torch.cat([q2, k2], -1), cos, sin, pos, nq + nkv, d, S)
        qkv = torch.cat([qk, v2], -1).contiguous()
        o = causal_attention(qkv, B, S, nq, nkv, d)
        y = self.o_proj(o)
        return y + residual if residual is not None else y


class _RopeFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qk, cos, sin, pos, n, d, S):
        from femtotron_b200.ops.kernels import rope_
        out = rope_(qk.contiguous().clone(), cos, sin, n, d, S, pos=pos)
        ctx.save_for_backward(cos, sin, pos if pos is not None else torch.empty(0))
        ctx.meta = (n, d, S, pos is not None)
        return out

    @staticmethod
    def backward(ctx, g):
        from femtotron_b200.ops.kernels import rope_
        cos, sin, pos = ctx.saved_tensors
        n, d, S, has = ctx.meta
        return rope_(g.contiguous().clone(), cos, sin, n, d, S, inverse=True,
                     pos=pos if has else None), None, None, None, None, None, None


class LlamaMLP(nn.Module):
    def __init__(self, config, device=None, dtype=None):
        super().__init__()
        H, I = config.hidden_size, config.intermediate_size
        bias = bool(_cfg(config, "mlp_bias", False))
        self.gate_proj = nn.Linear(H, I, bias=bias, device=device, dtype=dtype)
        self.up_proj = nn.Linear(H, I, bias=bias, device=device, dtype=dtype)
        self.down_proj = nn.Linear(I, H, bias=bias, device=device, dtype=dtype)

    def _fusable(self) -> bool:
        return _plain_col(self.gate_proj) and _plain_col(self.up_proj) and _plain_row(self.down_proj)

    def forward(self, x: torch.Tensor, residual=None):
        group, sp = _tp_info(self.gate_proj)
        comm = _sp_comm(x, group, sp, 0) if self._fusable() else None
        if comm is not None:
            from femtotron_b200.parallel.tensor_parallel.fused import SPColumnFn, SPRowFn
            h = SPColumnFn.apply(x, comm, "swiglu", None, self.gate_proj.weight, self.up_proj.weight)
            return SPRowFn.apply(h, residual, comm, self.down_proj.weight)
        if self._fusable():
            xin = _enter(x, group, sp)
            h = FN.GateUpSwiGLUFn.apply(xin, self.gate_proj.weight, self.up_proj.weight)
            if group is None:
                return FN.linear(h, self.down_proj.weight, residual=residual) if residual is not None \
                    else FN.linear(h, self.down_proj.weight)
            y = FN.linear(h, self.down_proj.weight)
            return _exit(y, group, sp, residual if residual is not None else 0)
        y = self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))
        return y + residual if residual is not None else y


class LlamaDecoderLayer(nn.Module):
    """Pre-norm LLaMA block.  Registration order (self_attn, mlp, input_layernorm,
    post_attention_layernorm) matches HF, which keeps q|k|v and gate|up consecutive when a
    unit's parameters are packed into one flat buffer."""

    def __init__(self, config, layer_idx: int, device=None, dtype=None):
        super().__init__()
        self.hidden_size = config.hidden_size
        self.layer_idx = layer_idx
        self.self_attn = LlamaAttention(config, layer_idx, device=device, dtype=dtype)
        self.mlp = LlamaMLP(config, device=device, dtype=dtype)
        eps = float(_cfg(config, "rms_norm_eps", 1e-6))
        self.input_layernorm = LlamaRMSNorm(config.hidden_size, eps, device=device, dtype=dtype)
        self.post_attention_layernorm = LlamaRMSNorm(config.hidden_size, eps, device=device, dtype=dtype)

    def forward(self, hidden_states: torch.Tensor, attention_mask=None, position_ids=None,
                past_key_values=None, use_cache=False, position_embeddings=None,
                batch_shape=None, **kwargs) -> torch.Tensor:
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1])
        if batch_shape is None:
            batch_shape = (shape[0], shape[1]) if len(shape) == 3 else (1, shape[0])
        if position_embeddings is None:
            raise ValueError("LlamaDecoderLayer needs position_embeddings (cos, sin, pos)")
        if len(position_embeddings) == 2:
            position_embeddings = (position_embeddings[0], position_embeddings[1], None)
        with nvtx_range(f"layer{self.layer_idx}"):
            n = self.input_layernorm(x)
            h = self.self_attn(n, position_embeddings, batch_shape, residual=x)
            n2 = self.post_attention_layernorm(h)
            out = self.mlp(n2, residual=h)
        return out.view(shape)
