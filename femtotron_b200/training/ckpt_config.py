"""Build a checkpoint policy from a plain dict (reference femtotron/training/ckpt_config.py:5-65):
{"type": "never"|"always"} | {"type": "class_name", "names": [...]} |
{"type": "any_of"|"all_of", "policies": [...]} | {"type": "not_of", "policy": {...}}."""
from __future__ import annotations

from typing import Any

from . import ckpt_policy as P


def policy_from_config(config: dict[str, Any] | None):
    if config is None:
        return P.never
    t = config.get("type")
    if t == "never":
        return P.never
    if t == "always":
        return P.always
    if t == "class_name":
        names = config.get("names") or []
        if not names:
            raise ValueError("class_name policy needs non-empty 'names'")
        return P.by_class_name(*names)
    if t in ("any_of", "all_of"):
        subs = [policy_from_config(c) for c in config.get("policies", [])]
        return P.any_of(*subs) if t == "any_of" else P.all_of(*subs)
    if t == "not_of":
        return P.not_of(policy_from_config(config["policy"]))
    raise ValueError(f"unknown checkpoint policy type {t!r}")
