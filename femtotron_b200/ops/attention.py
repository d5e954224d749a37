"""Causal GQA attention entry point.

``flash_attention`` runs the sm_100a flash-attention kernels (forward and backward) on a
packed [B*S, (nq+2nkv)*d] QKV projection.  They cover head sizes 64 and 128 with S a
multiple of 128; other shapes on a GPU use PyTorch SDPA, and every such call is counted in
``SDPA_FALLBACKS`` and announced once with a warning (FT_STRICT_ATTN=1 raises instead), so a
benchmark or a test can assert that the library never ran on its path.

Replaces the reference's attention, which runs inside Hugging Face ``LlamaDecoderLayer``
modules (femtotron/model/llama_partial_model.py:143-150) through PyTorch SDPA with GQA.
"""
from __future__ import annotations

import os
import warnings

import torch

from .ext import error_flag, has_native, native

# FT_ATTN=sdpa routes attention to torch SDPA (for A/B measurements against the library)
USE_NATIVE = os.environ.get("FT_ATTN", "native") != "sdpa"
STRICT = os.environ.get("FT_STRICT_ATTN") == "1"
# CUDA attention calls that went to PyTorch SDPA because the native kernels do not cover
# the shape (or FT_ATTN=sdpa)
SDPA_FALLBACKS = [0]


def note_fallback(head_dim: int, seq_len: int) -> None:
    """Record one CUDA attention call served by PyTorch SDPA."""
    if STRICT and USE_NATIVE:
        raise RuntimeError(f"native flash attention does not cover head_dim={head_dim}, "
                           f"seq_len={seq_len} (FT_STRICT_ATTN=1)")
    if SDPA_FALLBACKS[0] == 0 and USE_NATIVE:
        warnings.warn(f"attention on CUDA falls back to PyTorch SDPA for head_dim={head_dim}, "
                      f"seq_len={seq_len} (native kernels: head_dim 64/128, seq_len % 128 == 0)")
    SDPA_FALLBACKS[0] += 1


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
