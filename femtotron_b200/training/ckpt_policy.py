"""Composable predicates selecting modules for activation checkpointing (reference
femtotron/training/ckpt_policy.py:25-142): by class, by class name, any_of / all_of /
not_of, and the constants never / always."""
from __future__ import annotations

from typing import Callable

from torch import nn

CheckpointPolicy = Callable[[nn.Module], bool]


def by_class(*classes: type) -> CheckpointPolicy:
    if not classes:
        raise ValueError("by_class needs at least one class")
    def policy(m: nn.Module) -> bool:
        return isinstance(m, classes)
    policy.__name__ = f"by_class({', '.join(c.__name__ for c in classes)})"
    return policy


def by_class_name(*names: str) -> CheckpointPolicy:
    if not names:
        raise ValueError("by_class_name needs at least one name")
    wanted = set(names)
    def policy(m: nn.Module) -> bool:
        return type(m).__name__ in wanted
    policy.__name__ = f"by_class_name({', '.join(names)})"
    return policy


def any_of(*policies: CheckpointPolicy) -> CheckpointPolicy:
    def policy(m): return any(p(m) for p in policies)
    policy.__name__ = f"any_of({', '.join(_name(p) for p in policies)})"
    return policy


def all_of(*policies: CheckpointPolicy) -> CheckpointPolicy:
    if not policies:
        raise ValueError("all_of needs at least one policy")
    def policy(m): return all(p(m) for p in policies)
    policy.__name__ = f"all_of({', '.join(_name(p) for p in policies)})"
    return policy


def not_of(p: CheckpointPolicy) -> CheckpointPolicy:
    def negated(m): return not p(m)
    negated.__name__ = f"not_of({_name(p)})"
    return negated


def never(m: nn.Module) -> bool:
    return False


def always(m: nn.Module) -> bool:
    return True


NEVER = never
ALWAYS = always


def _name(p) -> str:
    return getattr(p, "__name__", repr(p))
