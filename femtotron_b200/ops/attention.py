"""Causal GQA attention entry point.

``flash_attention`` runs the sm_100a flash-attention kernels (forward and backward) on a
packed [B*S, (nq+2nkv)*d] QKV projection.  Until those kernels are registered for a head
size, ``flash_available`` is False and the caller uses PyTorch SDPA.
"""
from __future__ import annotations

import torch

import os

from .ext import error_flag, has_native, native

# FT_ATTN=sdpa routes attention to torch SDPA (for A/B measurements against the library)
USE_NATIVE = os.environ.get("FT_ATTN", "native") != "sdpa"


def flash_available(head_dim: int, seq_len: int = 128) -> bool:
    """True when the native kernels cover this shape (head size 64/128, S a multiple of 128)."""
    if not has_native() or head_dim not in (64, 128) or seq_len % 128 != 0:
        return False
    m = native()
    return hasattr(m, "flash_fwd") and hasattr(m, "flash_bwd")


class FlashAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, B, S, nq, nkv, d):
        o = torch.empty(B * S, nq * d, dtype=qkv.dtype, device=qkv.device)
        lse = torch.empty(B, nq, S, dtype=torch.float32, device=qkv.device)
        native().flash_fwd(qkv, o, lse, B, S, nq, nkv, d, error_flag(qkv.device))
        ctx.save_for_backward(qkv, o, lse)
        ctx.meta = (B, S, nq, nkv, d)
        return o

    @staticmethod
    def backward(ctx, do):
        qkv, o, lse = ctx.saved_tensors
        B, S, nq, nkv, d = ctx.meta
        dqkv = torch.empty_like(qkv)
        native().flash_bwd(qkv, o, do.contiguous(), lse, dqkv, B, S, nq, nkv, d,
                          error_flag(qkv.device))
        return dqkv, None, None, None, None, None


def flash_attention(qkv, B, S, nq, nkv, d):
    return FlashAttnFn.apply(qkv, B, S, nq, nkv, d)
