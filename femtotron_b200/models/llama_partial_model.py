"""PP-aware LLaMA backbone (the role of the reference's LlamaPartialModel,
femtotron/model/llama_partial_model.py:44-220).

Holds ``embed_tokens`` on the first stage, decoder ``layers`` keyed by GLOBAL layer index
in a ModuleDict, and the final ``norm`` on the last stage, so parameter names equal HF
LlamaModel's (``layers.{i}....``) on every stage.  ``forward`` returns hidden states
(normalised on the last stage).

Activation layout: the first stage takes input ids [B, S]; hidden states travel as
[B, S, H], or, under sequence parallelism, as the local token shard [B*S/tp, H] (the
embedding's TP reduction becomes a reduce-scatter over tokens).
"""
from __future__ import annotations

import torch
from torch import nn

from .layers import LlamaDecoderLayer, LlamaRMSNorm, LlamaRotaryEmbedding


class LlamaPartialModel(nn.Module):
    def __init__(self, model_config, parallel_ctx=None, layer_range: range | None = None,
                 is_first: bool | None = None, is_last: bool | None = None, device=None, dtype=None):
        super().__init__()
        n_layers = model_config.num_hidden_layers
        if layer_range is None:
            layer_range = range(n_layers)
        if not isinstance(layer_range, range):
            raise ValueError(f"layer_range must be a range, got {type(layer_range).__name__}")
        if layer_range.start < 0 or layer_range.stop > n_layers:
            raise ValueError(f"layer_range {layer_range} out of bounds for {n_layers} layers")
        if layer_range.step != 1:
            raise ValueError(f"layer_range must be contiguous (step=1), got step={layer_range.step}")
        self.config = model_config
        self.parallel_ctx = parallel_ctx
        self.layer_range = layer_range
        self.is_first = (layer_range.start == 0) if is_first is None else is_first
        self.is_last = (layer_range.stop == n_layers) if is_last is None else is_last
        if self.is_first:
            self.embed_tokens = nn.Embedding(model_config.vocab_size, model_config.hidden_size,
                                             padding_idx=getattr(model_config, "pad_token_id", None),
                                             device=device, dtype=dtype)
        self.layers = nn.ModuleDict({str(i): LlamaDecoderLayer(model_config, i, device=device, dtype=dtype)
                                     for i in layer_range})
        self.rotary_emb = LlamaRotaryEmbedding(model_config, device=device)
        if self.is_last:
            self.norm = LlamaRMSNorm(model_config.hidden_size,
                                     eps=float(getattr(model_config, "rms_norm_eps", 1e-6) or 1e-6),
                                     device=device, dtype=dtype)

    def _sequence_parallel(self) -> tuple[bool, int]:
        for layer in self.layers.values():
            q = layer.self_attn.q_proj
            sp = bool(getattr(q, "sequence_parallel", False))
            ws = int(getattr(q, "world_size", 1))
            return sp and ws > 1, ws
        return False, 1

    def forward(self, x: torch.Tensor, attention_mask: torch.Tensor | None = None,
                position_ids: torch.Tensor | None = None, batch_shape=None) -> torch.Tensor:
        if attention_mask is not None:
            raise NotImplementedError("only causal attention without padding masks is supported")
        sp, tp = self._sequence_parallel()
        if self.is_first:
            B, S = x.shape
            h = self.embed_tokens(x)
        else:
            h = x
            if batch_shape is not None:
                B, S = batch_shape
            elif h.dim() == 3:
                B, S = h.shape[0], h.shape[1]
            else:
                B, S = 1, h.shape[0] * (tp if sp else 1)
        if sp and h.dim() == 3:
            # a plain embedding (not vocab-parallel) was used: shard tokens here
            from femtotron_b200.parallel.tensor_parallel.comm_ops import scatter_to_tp
            h = scatter_to_tp(h.reshape(-1, h.shape[-1]), self.layers[next(iter(self.layers))].self_attn.q_proj.group, 0)
        cos, sin = self.rotary_emb(h, position_ids=position_ids, seq_len=S)
        pos = None
        if position_ids is not None:
            pos = position_ids.expand(B, S).reshape(-1).to(torch.int32).contiguous()
        pe = (cos, sin, pos)
        for layer in self.layers.values():
            h = layer(h, position_embeddings=pe, position_ids=position_ids, batch_shape=(B, S))
        if self.is_last:
            h = self.norm(h)
        return h
