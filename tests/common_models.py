"""Shared tiny configurations and builders for the CPU tests."""
from __future__ import annotations

import torch
from transformers import LlamaConfig


def tiny_config(**kw) -> LlamaConfig:
    base = dict(hidden_size=64, intermediate_size=160, num_attention_heads=4, num_key_value_heads=2,
                num_hidden_layers=2, vocab_size=256, max_position_embeddings=128, rms_norm_eps=1e-5,
                attn_implementation="sdpa")
    base.update(kw)
    return LlamaConfig(**base)


def hf_init(name, p):
    """Deterministic, well-conditioned init keyed by the parameter name (same values for
    every sharding of the same logical tensor are produced by slicing a full tensor)."""
    if p.dim() == 1:
        p.fill_(1.0)
    else:
        p.normal_(0, 0.05)


def full_state(cfg, seed=0):
    """A full fp32 state dict for the HF-named tiny model."""
    from femtotron_b200.models import LlamaForTraining, materialize_model
    torch.manual_seed(seed)
    with torch.device("meta"):
        m = LlamaForTraining(cfg)
    materialize_model(m, "cpu", dtype=torch.float32, init_fn=hf_init)
    return {k: v.detach().clone() for k, v in m.state_dict().items()}


def load_sharded(model, full_sd, ctx):
    """Copy this rank's TP slice of every tensor of `full_sd` into `model` (HF names)."""
    from femtotron_b200.models.model_loader import shard_for_rank
    from femtotron_b200.models.parallel_plan import get_llama_parallel_plan
    plan = get_llama_parallel_plan()
    with torch.no_grad():
        for name, p in model.named_parameters():
            src = full_sd[name]
            p.copy_(shard_for_rank(src, name, plan, ctx.tp_rank, ctx.tp_size))
