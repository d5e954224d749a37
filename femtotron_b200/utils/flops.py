"""Model FLOPs per trained token, for MFU.

6 x (matmul parameters) for the forward and backward of every projection, plus
6 x layers x hidden x seq for causal attention (the score and value products, forward and
backward, with half the square masked).  Recomputation (activation checkpointing) is not
counted: MFU measures useful work."""
from __future__ import annotations


def llama_flops_per_token(cfg, seq_len: int) -> float:
    H, L, V = cfg.hidden_size, cfg.num_hidden_layers, cfg.vocab_size
    nq = cfg.num_attention_heads
    nkv = getattr(cfg, "num_key_value_heads", None) or nq
    d = getattr(cfg, "head_dim", None) or H // nq
    per_layer = H * nq * d + 2 * H * nkv * d + nq * d * H + 3 * H * cfg.intermediate_size
    n_matmul = L * per_layer + V * H
    return 6.0 * n_matmul + 6.0 * L * H * seq_len


# dense bf16 tensor-core peak of one B200 (NVIDIA's figure without 2:4 sparsity), TFLOP/s
B200_BF16_DENSE_TFLOPS = 2250.0
