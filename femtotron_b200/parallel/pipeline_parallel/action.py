"""Immutable pipeline actions (reference femtotron/parallel/pipeline_parallel/action.py:26-123).
Schedules are lists of these; the runner dispatches on their type.  Compact reprs
(F(0), SFRB(1,0), ...) make schedules easy to print and assert on."""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class PPAction:
    pass


@dataclass(frozen=True, repr=False)
class Forward(PPAction):
    mb_id: int

    def __repr__(self): return f"F({self.mb_id})"


@dataclass(frozen=True, repr=False)
class Backward(PPAction):
    mb_id: int

    def __repr__(self): return f"B({self.mb_id})"


@dataclass(frozen=True, repr=False)
class SendForward(PPAction):
    mb_id: int

    def __repr__(self): return f"SF({self.mb_id})"


@dataclass(frozen=True, repr=False)
class RecvForward(PPAction):
    mb_id: int

    def __repr__(self): return f"RF({self.mb_id})"


@dataclass(frozen=True, repr=False)
class SendBackward(PPAction):
    mb_id: int

    def __repr__(self): return f"SB({self.mb_id})"


@dataclass(frozen=True, repr=False)
class RecvBackward(PPAction):
    mb_id: int

    def __repr__(self): return f"RB({self.mb_id})"


@dataclass(frozen=True, repr=False)
class SendForwardRecvBackward(PPAction):
    fwd_mb: int
    bwd_mb: int

    def __repr__(self): return f"SFRB({self.fwd_mb},{self.bwd_mb})"


@dataclass(frozen=True, repr=False)
class SendBackwardRecvForward(PPAction):
    bwd_mb: int
    fwd_mb: int

    def __repr__(self): return f"SBRF({self.bwd_mb},{self.fwd_mb})"
