"""What a forward pass keeps for its backward: a debugging aid for activation checkpointing
and for forwards that should be identical but are not (the reference ships the same idea as a
test-side script, femtotron/test/integration/diagnose_mismatch.py:18-91).

    with SavedTensorLog("no-ac") as a:
        loss = model(ids, labels=ids)["loss"]
    with SavedTensorLog("ac") as b:
        loss2 = model_ac(ids, labels=ids)["loss"]
    print(a.summary(), b.summary())
    print(format_diff(diff_saved(a, b)))

Each saved tensor is recorded with its shape, dtype, byte size and the innermost frames of
the caller's own code (frames inside torch and site-packages are skipped), so a difference
points at the line that saved it.  Tensors are passed through unchanged.
"""
from __future__ import annotations

import os
import traceback
from collections import Counter
from dataclasses import dataclass, field

import torch


@dataclass
class SavedTensorLog:
    name: str
    frames: int = 3
    entries: list = field(default_factory=list)

    def _where(self) -> str:
        stack = traceback.extract_stack()[:-2]
        own = [f for f in stack if f"{os.sep}torch{os.sep}" not in f.filename
               and "site-packages" not in f.filename]
        chosen = (own or stack)[-self.frames:]
        return " <- ".join(f"{os.path.basename(f.filename)}:{f.lineno}" for f in reversed(chosen))

    def _pack(self, t: torch.Tensor):
        self.entries.append((tuple(t.shape), str(t.dtype).replace("torch.", ""),
                             t.numel() * t.element_size(), self._where()))
        return t

    @staticmethod
    def _unpack(t):
        return t

    def __enter__(self):
        self._hooks = torch.autograd.graph.saved_tensors_hooks(self._pack, self._unpack)
        self._hooks.__enter__()
        return self

    def __exit__(self, *exc):
        self._hooks.__exit__(*exc)
        return False

    @property
    def saved_bytes(self) -> int:
        return sum(e[2] for e in self.entries)

    def summary(self) -> str:
        return f"[{self.name}] {len(self.entries)} tensors saved, {self.saved_bytes / 2 ** 20:.1f} MiB"


def diff_saved(a: SavedTensorLog, b: SavedTensorLog) -> dict:
    """Multiset difference of (shape, dtype, location) between two logs (order ignored):
    {"only_a": {key: count}, "only_b": {key: count}}; both empty when the saves agree."""
    ka = Counter((e[0], e[1], e[3]) for e in a.entries)
    kb = Counter((e[0], e[1], e[3]) for e in b.entries)
    return {"only_a": dict(ka - kb), "only_b": dict(kb - ka)}


def format_diff(d: dict, a_name: str = "a", b_name: str = "b") -> str:
    if not d["only_a"] and not d["only_b"]:
        return "saved tensors agree"
    lines = []
    for side, name in (("only_a", a_name), ("only_b", b_name)):
        for (shape, dtype, where), n in d[side].items():
            lines.append(f"only in {name}: {n}x shape={shape} dtype={dtype} at {where}")
    return "\n".join(lines)
