"""Per-op entry points: sm_100a kernels for CUDA tensors, PyTorch math for CPU tensors.

The CPU branches restate the kernels' math in plain PyTorch.  They run the gloo/CPU tests
and serve as the fp32 references of the GPU numerics tests; they are never used for CUDA
tensors.

Reference counterparts: the vocab-parallel embedding lookup
(femtotron/parallel/tensor_parallel/embedding.py:57-77), the gradient-norm sum of squares of
ClipGradNorm (femtotron/training/grad_transform.py:13-76), and ``torch.optim.AdamW`` inside
MixedPrecisionManager.step (femtotron/training/mixed_precision_manager.py:318-331).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .ext import native


# ------------------------------------------------------------------------------ RMSNorm
def rmsnorm_fwd(x: torch.Tensor, w: torch.Tensor, eps: float):
    """y = w * bf16(x * rsqrt(mean(x^2) + eps)); returns (y, rstd[fp32, rows])."""
    x2 = x.reshape(-1, x.shape[-1])
    if x.is_cuda:
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
        native().rmsnorm_fwd(x2, w, y, rstd, float(eps))
        return y.view_as(x), rstd
    xf = x2.float()
    rstd = torch.rsqrt(xf.pow(2).mean(-1) + eps)
    y = w.float() * (xf * rstd[:, None]).to(x.dtype).float()
    return y.to(x.dtype).view_as(x), rstd


def rmsnorm_bwd(dy: torch.Tensor, x: torch.Tensor, w: torch.Tensor, rstd: torch.Tensor):
    """Returns (dx, dw_fp32)."""
    H = x.shape[-1]
    x2, dy2 = x.reshape(-1, H), dy.reshape(-1, H)
    if x.is_cuda:
        dx = torch.empty_like(x2)
        dw = torch.zeros(H, dtype=torch.float32, device=x.device)
        native().rmsnorm_bwd(dy2.contiguous(), x2, w, rstd, dx, dw)
        return dx.view_as(x), dw
    xf, gf, wf = x2.float(), dy2.float(), w.float()
    n = xf * rstd[:, None]
    dn = gf * wf
    dot = (dn * n).mean(-1, keepdim=True)
    dx = rstd[:, None] * (dn - n * dot)
    dw = (gf * n.to(x.dtype).float()).sum(0)
    return dx.to(x.dtype).view_as(x), dw


# ------------------------------------------------------------------------------ RoPE
def rope_tables(head_dim: int, max_pos: int, theta: float, device, dtype=torch.bfloat16):
    """cos/sin tables [max_pos, head_dim/2], computed like the HF LLaMA rotary embedding
    (fp32 inv_freq and angles, then cast to the activation dtype)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    t = torch.arange(max_pos, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    return freqs.cos().to(dtype).to(device), freqs.sin().to(dtype).to(device)


def rope_(qk: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, nheads: int, head_dim: int,
          seq_len: int, inverse: bool = False, pos: torch.Tensor | None = None) -> torch.Tensor:
    """In-place rotate-half RoPE of the first `nheads` heads of each row of `qk` [T, ld].
    Row t has position pos[t] (or t % seq_len)."""
    if qk.is_cuda:
        native().rope_apply(qk, cos, sin, pos, nheads, head_dim, seq_len, inverse)
        return qk
    T = qk.shape[0]
    half = head_dim // 2
    p = pos.long() if pos is not None else torch.arange(T) % seq_len
    c = cos[p].float()[:, None, :]
    s = sin[p].float()[:, None, :]
    view = qk[:, : nheads * head_dim].view(T, nheads, head_dim)
    a = view[..., :half].float()
    b = view[..., half:].float()
    if not inverse:
        oa, ob = a * c - b * s, b * c + a * s
    else:
        oa, ob = a * c + b * s, b * c - a * s
    view[..., :half] = oa.to(qk.dtype)
    view[..., half:] = ob.to(qk.dtype)
    return qk


# ------------------------------------------------------------------------------ SwiGLU
def swiglu_fwd(gu: torch.Tensor, F_: int) -> torch.Tensor:
    if gu.is_cuda:
        h = torch.empty(gu.shape[0], F_, dtype=gu.dtype, device=gu.device)
        native().swiglu_fwd(gu, h, F_)
        return h
    g, u = gu[:, :F_].float(), gu[:, F_:2 * F_].float()
    return (F.silu(g) * u).to(gu.dtype)


def swiglu_bwd(dh: torch.Tensor, gu: torch.Tensor, F_: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Returns dGU [T, 2F] = [dgate | dup]."""
    if out is None:
        out = torch.empty(gu.shape[0], 2 * F_, dtype=gu.dtype, device=gu.device)
    if gu.is_cuda:
        native().swiglu_bwd(dh, gu, out, F_)
        return out
    # explicit copies: `out` may alias `gu`, and .float() does not copy fp32 inputs
    g, u, d = gu[:, :F_].float().clone(), gu[:, F_:2 * F_].float().clone(), dh.float()
    s = torch.sigmoid(g)
    out[:, :F_] = (d * u * s * (1 + g * (1 - s))).to(gu.dtype)
    out[:, F_:2 * F_] = (d * g * s).to(gu.dtype)
    return out


# ------------------------------------------------------------------------------ embedding
def embed_fwd(ids: torch.Tensor, table: torch.Tensor, vstart: int) -> torch.Tensor:
    flat = ids.reshape(-1)
    if ids.is_cuda:
        out = torch.empty(flat.numel(), table.shape[1], dtype=table.dtype, device=ids.device)
        native().embed_fwd(flat.contiguous(), table, out, int(vstart))
        return out.view(*ids.shape, table.shape[1])
    local = flat - vstart
    mask = (local < 0) | (local >= table.shape[0])
    out = F.embedding(local.masked_fill(mask, 0), table)
    out = out.masked_fill(mask[:, None], 0)
    return out.view(*ids.shape, table.shape[1])


def embed_bwd(ids: torch.Tensor, dout: torch.Tensor, vocab_local: int, vstart: int) -> torch.Tensor:
    """Returns the fp32 table gradient [vocab_local, H]."""
    H = dout.shape[-1]
    flat = ids.reshape(-1)
    d2 = dout.reshape(-1, H)
    dtable = torch.zeros(vocab_local, H, dtype=torch.float32, device=dout.device)
    if dout.is_cuda:
        native().embed_bwd(flat.contiguous(), d2.contiguous(), dtable, int(vstart))
        return dtable
    local = flat - vstart
    mask = (local >= 0) & (local < vocab_local)
    dtable.index_add_(0, local[mask], d2[mask].float())
    return dtable


# ------------------------------------------------------------------------------ cross-entropy
def xent_stats(logits: torch.Tensor, labels: torch.Tensor, vstart: int) -> torch.Tensor:
    """Per-row partials over the local vocab shard: [T, 4] = (max, sumexp, target, has)."""
    T = logits.shape[0]
    if logits.is_cuda:
        stats = torch.empty(T, 4, dtype=torch.float32, device=logits.device)
        native().xent_stats(logits, labels.contiguous(), stats, int(vstart))
        return stats
    x = logits.float()
    m = x.max(-1).values
    s = torch.exp(x - m[:, None]).sum(-1)
    V = x.shape[1]
    local = labels - vstart
    has = (local >= 0) & (local < V)
    tgt = torch.where(has, x.gather(1, local.clamp(0, V - 1)[:, None])[:, 0], torch.zeros_like(m))
    return torch.stack([m, s, tgt, has.float()], 1)


def xent_bwd_(logits: torch.Tensor, labels: torch.Tensor, lse: torch.Tensor,
              grad_scale: torch.Tensor, vstart: int, ignore_index: int = -100) -> torch.Tensor:
    """In place: logits <- (softmax - onehot) * grad_scale (0 for ignored rows)."""
    if logits.is_cuda:
        native().xent_bwd(logits, labels.contiguous(), lse.contiguous(), grad_scale, int(vstart),
                          int(ignore_index))
        return logits
    x = logits.float()
    p = torch.exp(x - lse[:, None])
    V = x.shape[1]
    local = labels - vstart
    has = (local >= 0) & (local < V)
    rows = torch.nonzero(has)[:, 0]
    p[rows, local[rows]] -= 1.0
    g = torch.where(labels == ignore_index, torch.zeros_like(lse), grad_scale.float().expand_as(lse))
    logits.copy_((p * g[:, None]).to(logits.dtype))
    return logits


# ------------------------------------------------------------------------------ optimizer
def adamw_multi(params, exp_avgs, exp_avg_sqs, grads, bf16_out, weight_decays, *, lr, beta1,
                beta2, eps, step, grad_scale: torch.Tensor | None = None):
    """Multi-tensor AdamW with torch.optim.AdamW semantics (decoupled weight decay, bias
    correction).  `bf16_out[i]` (optional) receives the updated parameter in bf16."""
    if not params:
        return
    if params[0].is_cuda:
        native().adamw_multi(list(params), list(exp_avgs), list(exp_avg_sqs), list(grads),
                             [t if t is not None else torch.empty(0, device=params[0].device)
                              for t in bf16_out] if bf16_out else [],
                             [float(w) for w in weight_decays], float(lr), float(beta1),
                             float(beta2), float(eps), int(step), grad_scale)
        return
    bc1 = 1 - beta1 ** step
    bc2s = (1 - beta2 ** step) ** 0.5
    gs = grad_scale.item() if grad_scale is not None else 1.0
    for i, p in enumerate(params):
        g = grads[i].float().reshape(p.shape) * gs
        p.mul_(1 - lr * weight_decays[i])
        exp_avgs[i].mul_(beta1).add_(g, alpha=1 - beta1)
        exp_avg_sqs[i].mul_(beta2).addcmul_(g, g, value=1 - beta2)
        denom = (exp_avg_sqs[i].sqrt() / bc2s).add_(eps)
        p.addcdiv_(exp_avgs[i], denom, value=-lr / bc1)
        if bf16_out and bf16_out[i] is not None:
            bf16_out[i].copy_(p.reshape(bf16_out[i].shape))


def sumsq_multi(tensors, slots, out: torch.Tensor) -> torch.Tensor:
    """out[slot] += sum(t^2) for each tensor t with its slot."""
    if not tensors:
        return out
    if out.is_cuda:
        native().sumsq_multi([t.contiguous() for t in tensors], [int(s) for s in slots], out)
        return out
    for t, s in zip(tensors, slots):
        out[s] += t.float().pow(2).sum()
    return out
