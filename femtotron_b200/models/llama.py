"""LLaMA training model and builder (reference femtotron/model/llama.py:20-194).

``build_llama_model(cfg, ctx, use_pp_aware=False, layer_range=None)`` builds the model on the
meta device and swaps in tensor-parallel modules per the LLaMA plan; weights are then
materialised with :func:`femtotron_b200.models.materialize.materialize_model` (random init)
or a :class:`ModelLoader` (safetensors).
"""
from __future__ import annotations

import torch
from torch import nn

from .base import full_logits, lm_head_loss
from .llama_causal import LlamaForCausalLM
from .llama_partial_model import LlamaPartialModel
from .parallel_plan import get_llama_parallel_plan
from .parallelize_model import parallelize_model


class LlamaForTraining(nn.Module):
    """Full (non-PP) LLaMA: backbone + lm_head + shifted next-token loss.  With
    tie_word_embeddings the lm_head shares the embedding weight."""

    def __init__(self, model_config, parallel_ctx=None, device=None, dtype=None):
        super().__init__()
        self.config = model_config
        self.parallel_ctx = parallel_ctx
        self.model = LlamaPartialModel(model_config, parallel_ctx, device=device, dtype=dtype)
        self.lm_head = nn.Linear(model_config.hidden_size, model_config.vocab_size, bias=False,
                                 device=device, dtype=dtype)
        if getattr(model_config, "tie_word_embeddings", False):
            self.tie_weights()

    def tie_weights(self):
        self.lm_head.weight = self.model.embed_tokens.weight

    def forward(self, input_ids: torch.Tensor, labels: torch.Tensor | None = None,
                materialize_logits: bool | None = None) -> dict:
        hidden = self.model(input_ids)
        out: dict = {}
        if labels is not None:
            out["loss"] = lm_head_loss(self.lm_head, hidden, labels)
        want = materialize_logits if materialize_logits is not None else labels is None
        out["logits"] = full_logits(self.lm_head, hidden, tuple(input_ids.shape)) if want else None
        return out

    @property
    def is_first(self) -> bool:
        return True

    @property
    def is_last(self) -> bool:
        return True

    @property
    def hidden_size(self) -> int:
        return self.config.hidden_size


def build_llama_model(model_config, parallel_ctx, *, use_pp_aware: bool = False,
                      layer_range: range | None = None, sequence_parallel: bool = False) -> nn.Module:
    with torch.device("meta"):
        if use_pp_aware:
            model = LlamaForCausalLM(model_config, parallel_ctx, layer_range=layer_range)
        else:
            model = LlamaForTraining(model_config, parallel_ctx)
    parallelize_model(model, get_llama_parallel_plan(sequence_parallel), parallel_ctx)
    if sequence_parallel and parallel_ctx.tp_size > 1:
        from .layers import LlamaRMSNorm
        for m in model.modules():
            if isinstance(m, LlamaRMSNorm):
                m.sp_group = parallel_ctx.tp_group
    return model
