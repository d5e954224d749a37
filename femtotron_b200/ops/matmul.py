"""tcgen05 GEMM entry points and the three products of a linear layer.

These replace the cuBLAS GEMMs behind the reference's ``F.linear`` calls
(femtotron/parallel/tensor_parallel/linear.py:72 and :206) and their autograd backward.

``gemm`` computes ``D (op)= A @ B^T`` with A given as [M,K] (``a_mn=False``) or as its
transpose [K,M] (``a_mn=True``), and B as [N,K] or [K,N] (``b_mn``).  On CUDA it runs the
persistent tcgen05 kernel of ``csrc/gemm.cu``; on CPU the same contract is evaluated in
fp32 with PyTorch (the numerics oracle of the tests).

Epilogue modes:
  ``store_bf16`` / ``store_f32``  D = acc
  ``acc_f32`` / ``acc_bf16``      D += acc   (gradient accumulation in place)
  ``resid``                       D = acc + R (residual add of o_proj / down_proj)
  ``swiglu``                      B rows [0,N) gate, [off, off+N) up: D = silu(g)*u, GU = [g|u]
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .ext import error_flag, native

EPI_MODES = {"store_bf16": 0, "store_f32": 1, "acc_f32": 2, "acc_bf16": 3, "resid": 4, "swiglu": 5}


def gemm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, *, a_mn: bool = False,
         b_mn: bool = False, mode: str = "store_bf16", residual: torch.Tensor | None = None,
         gu: torch.Tensor | None = None, gate_up_off: int = 0) -> torch.Tensor:
    if a.is_cuda:
        native().gemm_tc(a, b, out, a_mn, b_mn, EPI_MODES[mode], residual, gu, gate_up_off,
                         error_flag(a.device))
        return out
    A = (a.t() if a_mn else a).float()
    B = (b.t() if b_mn else b).float()
    if mode == "swiglu":
        n = out.shape[1]
        g = A @ B[:n].t()
        u = A @ B[gate_up_off:gate_up_off + n].t()
        gb, ub = g.to(out.dtype), u.to(out.dtype)  # the kernel stores bf16 pre-activations
        gu[:, :n] = gb
        gu[:, gate_up_off:gate_up_off + n] = ub
        out.copy_(F.silu(gb.float()) * ub.float())
        return out
    acc = A @ B.t()
    if mode in ("store_bf16", "store_f32"):
        out.copy_(acc)
    elif mode in ("acc_f32", "acc_bf16"):
        out.copy_(out.float() + acc)
    elif mode == "resid":
        out.copy_(acc + residual.float())
    else:
        raise ValueError(mode)
    return out


def linear_fwd(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None = None,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """y[M,N] = x[M,K] @ w[N,K]^T (+ residual)."""
    if out is None:
        out = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
    return gemm(x, w, out, mode="resid" if residual is not None else "store_bf16",
                residual=residual)


def linear_dgrad(dy: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """dx[M,K] = dy[M,N] @ w[N,K]."""
    if out is None:
        out = torch.empty(dy.shape[0], w.shape[1], dtype=dy.dtype, device=dy.device)
    return gemm(dy, w, out, b_mn=True)


def linear_wgrad(dy: torch.Tensor, x: torch.Tensor, dw: torch.Tensor, accumulate: bool) -> torch.Tensor:
    """dw[N,K] (+)= dy[M,N]^T @ x[M,K]; fp32 or bf16 destination."""
    if dw.dtype == torch.float32:
        mode = "acc_f32" if accumulate else "store_f32"
    else:
        mode = "acc_bf16" if accumulate else "store_bf16"
    return gemm(dy, x, dw, a_mn=True, b_mn=True, mode=mode)
