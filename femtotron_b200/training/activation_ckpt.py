"""Activation checkpointing by module wrapping (reference
femtotron/training/activation_ckpt.py:34-235).

Selected modules are wrapped in :class:`ActivationCheckpointWrapper`, which runs the inner
module under ``torch.utils.checkpoint`` (non-reentrant by default).  State-dict hooks strip
and re-add the wrapper prefix, so checkpoints keep the unwrapped parameter names.  The
wrapped module object itself is reused, so hooks installed on it (e.g. ZeRO-3 unit hooks)
stay inside the checkpointed region and fire again during the recomputation."""
from __future__ import annotations

from typing import Any

import torch
from torch import nn
from torch.utils.checkpoint import checkpoint

_PREFIX = "_checkpoint_wrapped_module"


class ActivationCheckpointWrapper(nn.Module):
    def __init__(self, module: nn.Module, *, use_reentrant: bool = False,
                 preserve_rng_state: bool = True, debug: bool = False):
        super().__init__()
        self._checkpoint_wrapped_module = module
        self.use_reentrant = use_reentrant
        self.preserve_rng_state = preserve_rng_state
        self.debug = debug
        self._register_state_dict_hook(_post_state_dict_hook)
        self._register_load_state_dict_pre_hook(_pre_load_state_dict_hook, with_module=True)

    @property
    def inner_module(self) -> nn.Module:
        return self._checkpoint_wrapped_module

    def forward(self, *args: Any, **kwargs: Any) -> Any:
        if not torch.is_grad_enabled():
            return self._checkpoint_wrapped_module(*args, **kwargs)
        return checkpoint(self._checkpoint_wrapped_module, *args, use_reentrant=self.use_reentrant,
                          preserve_rng_state=self.preserve_rng_state, **kwargs)

    def __getattr__(self, name: str):
        try:
            return super().__getattr__(name)
        except AttributeError:
            return getattr(self._checkpoint_wrapped_module, name)

    def extra_repr(self) -> str:
        return f"use_reentrant={self.use_reentrant}, preserve_rng_state={self.preserve_rng_state}"


def apply_activation_checkpointing(model: nn.Module, policy, *, use_reentrant: bool = False,
                                   preserve_rng_state: bool = True, debug: bool = False) -> int:
    """Wrap every module selected by `policy` (outermost match wins, no nesting); returns
    the number of wrapped modules."""
    targets = _collect_wrap_targets(model, policy)
    for parent, attr, mod in targets:
        w = ActivationCheckpointWrapper(mod, use_reentrant=use_reentrant,
                                        preserve_rng_state=preserve_rng_state, debug=debug)
        if isinstance(parent, (nn.ModuleList, nn.Sequential)) and attr.isdigit():
            parent[int(attr)] = w
        elif isinstance(parent, nn.ModuleDict):
            parent[attr] = w
        else:
            setattr(parent, attr, w)
    return len(targets)


def remove_activation_checkpointing(model: nn.Module) -> int:
    n = 0
    for name, mod in list(model.named_modules()):
        for cname, child in list(mod.named_children()):
            if isinstance(child, ActivationCheckpointWrapper):
                inner = child.inner_module
                if isinstance(mod, nn.ModuleDict):
                    mod[cname] = inner
                elif isinstance(mod, (nn.ModuleList, nn.Sequential)) and cname.isdigit():
                    mod[int(cname)] = inner
                else:
                    setattr(mod, cname, inner)
                n += 1
    return n


def is_activation_checkpointed(module: nn.Module) -> bool:
    return isinstance(module, ActivationCheckpointWrapper)


def _collect_wrap_targets(model: nn.Module, policy):
    out = []

    def visit(mod: nn.Module):
        for cname, child in mod.named_children():
            if isinstance(child, ActivationCheckpointWrapper):
                continue
            if policy(child):
                out.append((mod, cname, child))
            else:
                visit(child)
    visit(model)
    return out


def _post_state_dict_hook(module, state_dict, prefix, *args):
    key = prefix + _PREFIX + "."
    for k in list(state_dict.keys()):
        if k.startswith(key):
            state_dict[prefix + k[len(key):]] = state_dict.pop(k)
    return state_dict


def _pre_load_state_dict_hook(module, state_dict, prefix, *args):
    for k in list(state_dict.keys()):
        if k.startswith(prefix) and not k.startswith(prefix + _PREFIX + "."):
            state_dict[prefix + _PREFIX + "." + k[len(prefix):]] = state_dict.pop(k)
