"""NVTX ranges for timeline profilers (Nsight Systems, ncu's NVTX filters).

Enabled by FT_NVTX=1; otherwise every helper returns immediately, so the ranges can stay on
the hot path.  Ranges annotate: each decoder layer's forward (``layer<i>``, also during the
activation-checkpoint recompute), the trainer's phases (``phase:fwd``, ``phase:bwd``,
``phase:optimizer``) and every point where the compute stream waits on communication
(``wait:<kind>``, the same places the exposed-communication timer measures).  The reference
has no tracing of its own (it prints host-timed tokens/s, femtotron/training/trainer.py:241-250).
"""
from __future__ import annotations

import os
from contextlib import contextmanager

import torch

ENABLED = os.environ.get("FT_NVTX") == "1"


def _on() -> bool:
    return ENABLED and torch.cuda.is_available()


@contextmanager
def nvtx_range(name: str):
    """Push an NVTX range around the body (no-op unless FT_NVTX=1 on a CUDA build)."""
    if not _on():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


class PhaseRanges:
    """Consecutive, non-nested NVTX ranges: ``switch(label)`` closes the open range (if any)
    and opens ``label`` (None only closes)."""

    def __init__(self):
        self._open = False

    def switch(self, label: str | None) -> None:
        if not _on():
            return
        if self._open:
            torch.cuda.nvtx.range_pop()
            self._open = False
        if label is not None:
            torch.cuda.nvtx.range_push(label)
            self._open = True


PHASES = PhaseRanges()
