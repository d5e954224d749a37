"""Autograd functions of the LLaMA hot path, built on the sm_100a kernels.

They replace what the reference runs through Hugging Face modules and ATen: the decoder
layers' RMSNorm, RoPE, attention and SwiGLU (femtotron/model/llama_partial_model.py:143-157),
the column/row-parallel ``F.linear`` calls (femtotron/parallel/tensor_parallel/linear.py:72,
:206), and the LM-head loss, which the reference computes with ``F.cross_entropy`` on full-vocab
logits gathered over TP (femtotron/model/llama.py:91-111,
femtotron/parallel/tensor_parallel/comm_ops.py:72-82); here the loss is vocab-parallel.

Gradient sinks
--------------
Weight gradients are written by the wgrad GEMM epilogue directly into their destination:
  * ``param.main_grad`` (fp32, usually a view into a flat per-unit buffer) when present;
    ``param.grad_overwrite = True`` asks the next write to store instead of accumulate;
  * otherwise ``param.grad`` (compute dtype), created on first use and accumulated after.
The functions therefore return ``None`` for weights: autograd never materialises a separate
weight-gradient tensor, and gradient accumulation over micro-batches is fused into the GEMM.

Several weights that are consecutive in memory (q|k|v, gate|up) are used as one operand
without copying, so each of these projections is a single GEMM.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch.autograd import Function

from . import kernels as K
from .matmul import gemm, linear_dgrad, linear_fwd, linear_wgrad


# ------------------------------------------------------------------------------ helpers
def consecutive_rows(ts) -> torch.Tensor | None:
    """The given 2-D tensors as one [sum rows, cols] view when they are contiguous, share a
    dtype and column count, and follow each other in one storage; otherwise None."""
    ts = list(ts)
    first = ts[0]
    if len(ts) == 1:
        return first
    if not all(t.dim() == 2 and t.is_contiguous() and t.dtype == first.dtype and
               t.shape[1] == first.shape[1] for t in ts):
        return None
    base = first.untyped_storage().data_ptr()
    ptr = first.data_ptr()
    for t in ts:
        if t.untyped_storage().data_ptr() != base or t.data_ptr() != ptr:
            return None
        ptr += t.numel() * t.element_size()
    rows = sum(t.shape[0] for t in ts)
    v = torch.empty(0, dtype=first.dtype, device=first.device)
    v.set_(first.untyped_storage(), first.storage_offset(), (rows, first.shape[1]),
           (first.shape[1], 1))
    return v


def cat_rows_view(ts) -> torch.Tensor:
    """Rows of the given 2-D tensors as one operand: a view when consecutive in memory,
    otherwise a concatenated copy."""
    ts = list(ts)
    v = consecutive_rows(ts)
    return v if v is not None else torch.cat([t.reshape(t.shape[0], -1) for t in ts], 0)


def _grad_target(p: torch.Tensor):
    """(tensor, accumulate) destination for the gradient of parameter p, creating .grad if
    needed (then the first write stores)."""
    mg = getattr(p, "main_grad", None)
    if mg is not None:
        acc = not getattr(p, "grad_overwrite", False)
        p.grad_overwrite = False
        return mg, acc
    if p.grad is None:
        p.grad = torch.empty_like(p)
        return p.grad, False
    return p.grad, True


def grad_ready(p: torch.Tensor) -> None:
    """Tell the owner of parameter p (a sharding strategy) that this backward's contribution
    to its gradient has been enqueued, so a reduction can start early."""
    cb = getattr(p, "_ft_grad_ready", None)
    if cb is not None:
        cb()


def write_weight_grad(params, compute):
    """Route `compute(dst2d, accumulate)` (dst2d = [sum rows, cols]) to the gradient sinks of
    the 2-D weights `params`, used together as one stacked operand."""
    params = list(params)
    _write_weight_grad(params, compute)
    for p in params:
        grad_ready(p)


def _write_weight_grad(params, compute):
    targets = [_grad_target(p) for p in params]
    dsts = [t.view(p.shape) for (t, _), p in zip(targets, params)]
    accs = [a for _, a in targets]
    if len(set(accs)) == 1 and len({d.dtype for d in dsts}) == 1:
        v = consecutive_rows(dsts)
        if v is not None:
            compute(v, accs[0])
            return
    rows = sum(p.shape[0] for p in params)
    tmp = torch.empty(rows, params[0].shape[1], dtype=torch.float32, device=params[0].device)
    compute(tmp, False)
    r = 0
    for p, d, a in zip(params, dsts, accs):
        part = tmp[r:r + p.shape[0]]
        if a:
            d.add_(part.to(d.dtype))
        else:
            d.copy_(part)
        r += p.shape[0]


def write_vector_grad(p: torch.Tensor, g32: torch.Tensor):
    """Add an fp32 gradient vector/matrix into the sink of parameter p."""
    dst, acc = _grad_target(p)
    g = g32.view(dst.shape)
    if acc:
        dst.add_(g.to(dst.dtype))
    else:
        dst.copy_(g)
    grad_ready(p)


def _as2d(x: torch.Tensor) -> torch.Tensor:
    x2 = x.reshape(-1, x.shape[-1])
    return x2 if x2.is_contiguous() else x2.contiguous()


# ------------------------------------------------------------------------------ linear
class LinearFn(Function):
    """y = x @ cat(weights)^T (+ residual)."""

    @staticmethod
    def forward(ctx, x, residual, *weights):
        x2 = _as2d(x)
        W = cat_rows_view(weights)
        res2 = _as2d(residual) if residual is not None else None
        y = linear_fwd(x2, W, res2)
        ctx.save_for_backward(x2, *[w.detach() for w in weights])
        ctx.params = weights
        ctx.has_res = residual is not None
        ctx.xshape = x.shape
        return y.view(*x.shape[:-1], W.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, *weights = ctx.saved_tensors
        W = cat_rows_view(weights)
        dy2 = _as2d(dy)
        dx = linear_dgrad(dy2, W).view(ctx.xshape) if ctx.needs_input_grad[0] else None
        if any(ctx.needs_input_grad[2:]):
            write_weight_grad(ctx.params, lambda dst, acc: linear_wgrad(dy2, x2, dst, acc))
        ctx.params = None
        dres = dy if ctx.has_res else None
        return (dx, dres) + (None,) * len(weights)


def linear(x, *weights, residual=None):
    return LinearFn.apply(x, residual, *weights)


# ------------------------------------------------------------------------------ QKV + RoPE
class QKVRopeFn(Function):
    """qkv = x @ [Wq;Wk;Wv]^T, then RoPE on the q and k heads (the first nq+nkv heads of each
    row), in one GEMM plus one in-place rotation."""

    @staticmethod
    def forward(ctx, x, cos, sin, pos, n_rot_heads, head_dim, seq_len, *weights):
        x2 = _as2d(x)
        W = cat_rows_view(weights)
        qkv = linear_fwd(x2, W)
        K.rope_(qkv, cos, sin, n_rot_heads, head_dim, seq_len, pos=pos)
        ctx.save_for_backward(x2, cos, sin, pos if pos is not None else torch.empty(0),
                              *[w.detach() for w in weights])
        ctx.params = weights
        ctx.meta = (n_rot_heads, head_dim, seq_len, pos is not None)
        ctx.xshape = x.shape
        return qkv

    @staticmethod
    def backward(ctx, dqkv):
        x2, cos, sin, pos, *weights = ctx.saved_tensors
        n_rot, hd, seq, has_pos = ctx.meta
        d = dqkv.contiguous().clone()
        K.rope_(d, cos, sin, n_rot, hd, seq, inverse=True, pos=pos if has_pos else None)
        W = cat_rows_view(weights)
        dx = linear_dgrad(d, W).view(ctx.xshape) if ctx.needs_input_grad[0] else None
        if any(ctx.needs_input_grad[7:]):
            write_weight_grad(ctx.params, lambda dst, acc: linear_wgrad(d, x2, dst, acc))
        ctx.params = None
        return (dx, None, None, None, None, None, None) + (None,) * len(weights)


# ------------------------------------------------------------------------------ gate/up + SwiGLU
class GateUpSwiGLUFn(Function):
    """h = silu(x Wg^T) * (x Wu^T) as one GEMM whose tiles pair gate and up rows; the bf16
    pre-activations [g|u] are kept for the backward."""

    @staticmethod
    def forward(ctx, x, w_gate, w_up):
        x2 = _as2d(x)
        F_ = w_gate.shape[0]
        W = cat_rows_view([w_gate, w_up])
        T = x2.shape[0]
        h = torch.empty(T, F_, dtype=x2.dtype, device=x2.device)
        gu = torch.empty(T, 2 * F_, dtype=x2.dtype, device=x2.device)
        gemm(x2, W, h, mode="swiglu", gu=gu, gate_up_off=F_)
        ctx.save_for_backward(x2, gu, w_gate.detach(), w_up.detach())
        ctx.params = (w_gate, w_up)
        ctx.xshape = x.shape
        return h.view(*x.shape[:-1], F_)

    @staticmethod
    def backward(ctx, dh):
        x2, gu, w_gate, w_up = ctx.saved_tensors
        F_ = w_gate.shape[0]
        dgu = K.swiglu_bwd(_as2d(dh), gu, F_, out=gu)  # overwrite the saved pre-activations
        W = cat_rows_view([w_gate, w_up])
        dx = linear_dgrad(dgu, W).view(ctx.xshape) if ctx.needs_input_grad[0] else None
        if ctx.needs_input_grad[1] or ctx.needs_input_grad[2]:
            write_weight_grad(ctx.params, lambda dst, acc: linear_wgrad(dgu, x2, dst, acc))
        ctx.params = None
        return dx, None, None


# ------------------------------------------------------------------------------ RMSNorm
class RMSNormFn(Function):
    """RMSNorm; with ``sp_group`` (sequence parallelism) every rank normalises only its token
    shard, so the weight gradient is summed over that group before it is stored."""

    @staticmethod
    def forward(ctx, x, w, eps, sp_group=None):
        y, rstd = K.rmsnorm_fwd(x.contiguous(), w, eps)
        ctx.save_for_backward(x, w.detach(), rstd)
        ctx.param = w
        ctx.sp_group = sp_group
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        dx, dw = K.rmsnorm_bwd(dy.contiguous(), x.contiguous(), w, rstd)
        if ctx.needs_input_grad[1]:
            if ctx.sp_group is not None:
                dist.all_reduce(dw, group=ctx.sp_group)
            write_vector_grad(ctx.param, dw)
        ctx.param = None
        return dx, None, None, None


def rms_norm(x, w, eps, sp_group=None):
    return RMSNormFn.apply(x, w, eps, sp_group)


# ------------------------------------------------------------------------------ embedding
class EmbeddingFn(Function):
    """Vocab-parallel lookup: rows outside [vstart, vstart+V_local) give zeros (the TP
    reduction that completes them is applied by the caller)."""

    @staticmethod
    def forward(ctx, ids, weight, vstart):
        out = K.embed_fwd(ids, weight, vstart)
        ctx.save_for_backward(ids)
        ctx.param = weight
        ctx.vstart = vstart
        return out

    @staticmethod
    def backward(ctx, dout):
        (ids,) = ctx.saved_tensors
        weight = ctx.param
        ctx.param = None
        if ctx.needs_input_grad[1]:
            mg = getattr(weight, "main_grad", None)
            if mg is not None and mg.dtype == torch.float32 and ids.is_cuda:
                if getattr(weight, "grad_overwrite", False):
                    mg.zero_()
                    weight.grad_overwrite = False
                from .ext import native
                native().embed_bwd(ids.reshape(-1).contiguous(),
                                   dout.reshape(-1, dout.shape[-1]).contiguous(),
                                   mg.view(weight.shape), int(ctx.vstart))
                grad_ready(weight)
            else:
                write_vector_grad(weight, K.embed_bwd(ids, dout, weight.shape[0], ctx.vstart))
        return None, None, None


# ------------------------------------------------------------------------------ LM head + CE
class LMHeadCrossEntropyFn(Function):
    """loss = mean over non-ignored rows of CE(h @ W^T, labels), W the local vocab shard.

    The logits of the local shard are produced by one GEMM and reduced to per-row
    (max, sum-exp, target) partials; with tensor parallelism only these [T,4] partials cross
    the TP group (never the full-vocab logits).  The backward turns the saved logits into
    dlogits in place and runs the dgrad/wgrad GEMMs on them.
    """

    @staticmethod
    def forward(ctx, h, w, labels, vstart, tp_group, ignore_index):
        h2 = _as2d(h)
        logits = linear_fwd(h2, w)
        lab = labels.reshape(-1)
        stats = K.xent_stats(logits, lab, vstart)
        if tp_group is not None and dist.get_world_size(tp_group) > 1:
            ws = dist.get_world_size(tp_group)
            allst = torch.empty(ws * stats.shape[0], stats.shape[1], dtype=stats.dtype,
                                device=stats.device)
            dist.all_gather_into_tensor(allst, stats, group=tp_group)
            allst = allst.view(ws, *stats.shape)
            m = allst[..., 0].max(0).values
            s = (allst[..., 1] * torch.exp(allst[..., 0] - m)).sum(0)
            tgt = allst[..., 2].sum(0)
        else:
            m, s, tgt = stats[:, 0], stats[:, 1], stats[:, 2]
        lse = m + torch.log(s)
        valid = lab != ignore_index
        n_valid = valid.sum().to(torch.float32)
        loss = torch.where(valid, lse - tgt, torch.zeros_like(lse)).sum() / n_valid
        ctx.save_for_backward(h2, w.detach(), lab, lse, n_valid, logits)
        ctx.param = w
        ctx.meta = (vstart, ignore_index)
        ctx.hshape = h.shape
        return loss

    @staticmethod
    def backward(ctx, dloss):
        h2, w, lab, lse, n_valid, logits = ctx.saved_tensors
        vstart, ignore_index = ctx.meta
        scale = (dloss.float() / n_valid).reshape(1)
        dlogits = K.xent_bwd_(logits, lab, lse, scale, vstart, ignore_index)
        dh = linear_dgrad(dlogits, w).view(ctx.hshape) if ctx.needs_input_grad[0] else None
        if ctx.needs_input_grad[1]:
            write_weight_grad([ctx.param], lambda dst, acc: linear_wgrad(dlogits, h2, dst, acc))
        ctx.param = None
        return dh, None, None, None, None, None


def shift_labels(labels: torch.Tensor, ignore_index: int = -100) -> torch.Tensor:
    """labels[b, s+1] at position s; the last position of each sequence is ignored."""
    out = torch.full_like(labels, ignore_index)
    out[..., :-1] = labels[..., 1:]
    return out
