"""Swap modules for their tensor-parallel versions according to a ParallelPlan (reference
femtotron/model/parallelize_model.py:10-87).  Intended for models on the meta device: only
module types and parameter shapes change; weights are materialised afterwards."""
from __future__ import annotations

from torch import nn

from .parallel_module_builder import _BUILDER_REGISTRY


def parallelize_model(model: nn.Module, parallel_plan, parallel_ctx) -> nn.Module:
    replacements = []
    for name, module in model.named_modules():
        if not name:
            continue
        rule = parallel_plan.get_rule(name)
        if rule is None:
            continue
        parent, attr = _resolve_parent(model, name)
        replacements.append((parent, attr, module, rule))
    for parent, attr, old, rule in replacements:
        new = _resolve_builder(rule.parallel_type, type(old))(old, parallel_ctx, rule)
        if attr.isdigit() and isinstance(parent, (nn.ModuleList, nn.Sequential)):
            parent[int(attr)] = new
        else:
            setattr(parent, attr, new)
    return model


def _resolve_parent(root: nn.Module, qualified: str):
    parts = qualified.split(".")
    parent = root
    for p in parts[:-1]:
        if p.isdigit() and isinstance(parent, (nn.ModuleList, nn.Sequential)):
            parent = parent[int(p)]
        else:
            parent = getattr(parent, p)
    return parent, parts[-1]


def _resolve_builder(kind: str, source_type: type):
    b = _BUILDER_REGISTRY.get((kind, source_type))
    if b is not None:
        return b
    for base in source_type.__mro__[1:]:
        b = _BUILDER_REGISTRY.get((kind, base))
        if b is not None:
            return b
    raise ValueError(f"no builder registered for kind={kind!r}, source_type={source_type.__name__}")
