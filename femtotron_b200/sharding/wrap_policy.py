"""ZeRO-3 unit selection policies (reference femtotron/sharding/wrap_policy.py:6-35)."""
from __future__ import annotations

from torch import nn


def llama_wrap_policy(module: nn.Module) -> bool:
    """One unit per LLaMA decoder block (this package's block, or transformers' if present)."""
    from femtotron_b200.models.layers import LlamaDecoderLayer
    if isinstance(module, LlamaDecoderLayer):
        return True
    try:
        from transformers.models.llama.modeling_llama import LlamaDecoderLayer as HFLayer
        return isinstance(module, HFLayer)
    except ImportError:  # pragma: no cover
        return False


def make_class_wrap_policy(target_classes: tuple):
    def policy(module: nn.Module) -> bool:
        return isinstance(module, target_classes)
    return policy
