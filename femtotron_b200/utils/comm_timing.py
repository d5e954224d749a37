"""Exposed-communication timer: how long the compute stream is blocked on communication.

Every place where the compute stream waits for a communication stream or runs a collective
inline is wrapped in ``TIMER.wait(kind)``: a CUDA event is recorded on the compute stream
right before and right after the wait, and since nothing else is enqueued between the two,
their distance is device time the compute stream spent blocked.  Enabled by
FT_COMM_TIMING=1 (otherwise the context manager does nothing).  The reference has no such
measurement (it prints host-timed tokens/s only, femtotron/training/trainer.py:241-250).
"""
from __future__ import annotations

import os
from collections import defaultdict
from contextlib import contextmanager

import torch

from femtotron_b200.utils.tracing import PHASES, nvtx_range


class CommWaitTimer:
    def __init__(self):
        self.enabled = os.environ.get("FT_COMM_TIMING") == "1"
        self._pending: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []
        self._marks: list[tuple[str | None, torch.cuda.Event]] = []

    @contextmanager
    def wait(self, kind: str):
        if not self.enabled or not torch.cuda.is_available():
            with nvtx_range("wait:" + kind):
                yield
            return
        a = torch.cuda.Event(enable_timing=True)
        a.record()
        with nvtx_range("wait:" + kind):
            yield
        b = torch.cuda.Event(enable_timing=True)
        b.record()
        self._pending.append((kind, a, b))

    def mark(self, label: str | None) -> None:
        """Phase mark on the current stream: the device time until the next mark is added to
        ``phase:<label>`` (label None only closes the previous phase).  The same marks
        delimit NVTX ranges when FT_NVTX=1."""
        PHASES.switch(None if label is None else "phase:" + label)
        if not self.enabled or not torch.cuda.is_available():
            return
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self._marks.append((label, e))

    def collect(self) -> dict:
        """Milliseconds blocked per kind, and per phase, since the last call (synchronises on
        the events)."""
        out: dict[str, float] = defaultdict(float)
        for kind, a, b in self._pending:
            b.synchronize()
            out[kind] += a.elapsed_time(b)
        self._pending.clear()
        for (label, a), (_, b) in zip(self._marks, self._marks[1:]):
            if label is not None:
                b.synchronize()
                out["phase:" + label] += a.elapsed_time(b)
        self._marks = self._marks[-1:] if self._marks and self._marks[-1][0] is not None else []
        return dict(out)


TIMER = CommWaitTimer()
