"""String presets for ZeRO-3 wrap policies and activation-checkpoint policies, as used by the
YAML config (reference femtotron/scripts/presets.py:19-62)."""
from __future__ import annotations

from typing import Callable

from torch import nn


def _llama_layer_policy() -> Callable[[nn.Module], bool]:
    from femtotron_b200.sharding.wrap_policy import llama_wrap_policy
    return llama_wrap_policy


WRAP_POLICY_PRESETS = {"llama_decoder_layer": _llama_layer_policy}
AC_POLICY_PRESETS = {"llama_decoder_layer": _llama_layer_policy,
                     "never": lambda: (lambda m: False)}


def get_wrap_policy(name: str):
    if name not in WRAP_POLICY_PRESETS:
        raise ValueError(f"unknown wrap_policy preset {name!r}; available: {list(WRAP_POLICY_PRESETS)}")
    return WRAP_POLICY_PRESETS[name]()


def get_ac_policy(name: str):
    if name not in AC_POLICY_PRESETS:
        raise ValueError(f"unknown ac_policy preset {name!r}; available: {list(AC_POLICY_PRESETS)}")
    return AC_POLICY_PRESETS[name]()
