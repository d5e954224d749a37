"""PP-aware LLaMA causal LM (reference femtotron/model/llama_causal.py:14-48): backbone
LlamaPartialModel plus an lm_head on the last stage.  Tied embeddings are rejected, as in
the reference."""
from __future__ import annotations

from torch import nn

from .base import BaseCausalLMPipeline
from .llama_partial_model import LlamaPartialModel


class LlamaForCausalLM(BaseCausalLMPipeline):
    def __init__(self, config, parallel_ctx=None, layer_range: range | None = None, device=None, dtype=None):
        super().__init__()
        if getattr(config, "tie_word_embeddings", False):
            raise NotImplementedError("LlamaForCausalLM does not support tie_word_embeddings=True")
        self.config = config
        self.hidden_size = config.hidden_size
        self.model = LlamaPartialModel(config, parallel_ctx, layer_range=layer_range, device=device, dtype=dtype)
        self.is_first = self.model.is_first
        self.is_last = self.model.is_last
        if self.is_last:
            self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False, device=device, dtype=dtype)
