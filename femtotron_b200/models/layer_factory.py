"""Factory protocol for the non-decoder pieces of a model (embedding, final norm, lm_head),
the extension point the reference declares in femtotron/model/layer_factory.py:15-43.  The
default builds this package's modules; a subclass can substitute other implementations."""
from __future__ import annotations

from typing import Protocol

from torch import nn

from .layers import LlamaRMSNorm


class LayerFactory(Protocol):
    def make_embedding(self, config, parallel_ctx, *, dtype, device) -> nn.Module: ...
    def make_norm(self, config, *, dtype, device) -> nn.Module: ...
    def make_lm_head(self, config, parallel_ctx, *, tied_weight, dtype, device) -> nn.Module: ...


class DefaultLayerFactory:
    def make_embedding(self, config, parallel_ctx, *, dtype, device):
        from femtotron_b200.parallel.tensor_parallel import VocabParallelEmbedding
        tp = parallel_ctx.tp_size if parallel_ctx is not None else 1
        if tp > 1:
            return VocabParallelEmbedding(config.vocab_size // tp, config.hidden_size, parallel_ctx,
                                          device=device, dtype=dtype)
        return nn.Embedding(config.vocab_size, config.hidden_size, device=device, dtype=dtype)

    def make_norm(self, config, *, dtype, device):
        return LlamaRMSNorm(config.hidden_size, getattr(config, "rms_norm_eps", 1e-6), device=device, dtype=dtype)

    def make_lm_head(self, config, parallel_ctx, *, tied_weight=None, dtype=None, device=None):
        head = nn.Linear(config.hidden_size, config.vocab_size, bias=False, device=device, dtype=dtype)
        if tied_weight is not None:
            head.weight = tied_weight
        return head
