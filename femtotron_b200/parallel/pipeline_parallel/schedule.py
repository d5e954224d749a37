"""Pipeline schedules as pure functions returning action lists.

GPipe: every micro-batch forward (recv -> F -> send), then every backward in reverse.
1F1B (Megatron; reference femtotron/parallel/pipeline_parallel/schedule.py:78-174): stage r of
P runs min(P-1-r, N) warm-up forwards, then N-warmup steady iterations of one forward and one
backward, then drains the warm-up backwards.  In the steady phase the send of a forward
output is paired with the receive of a gradient (SFRB) and vice versa (SBRF) so neighbouring
stages never block on each other.  The exact action lists are part of the contract (unit
tests compare them verbatim)."""
from __future__ import annotations

from .action import (Backward, Forward, PPAction, RecvBackward, RecvForward, SendBackward,
                     SendBackwardRecvForward, SendForward, SendForwardRecvBackward)


def gpipe_schedule(num_microbatches: int, is_first: bool, is_last: bool) -> list[PPAction]:
    if num_microbatches < 1:
        raise ValueError(f"num_microbatches must be >= 1, got {num_microbatches}")
    out: list[PPAction] = []
    for mb in range(num_microbatches):
        if not is_first:
            out.append(RecvForward(mb))
        out.append(Forward(mb))
        if not is_last:
            out.append(SendForward(mb))
    for mb in range(num_microbatches - 1, -1, -1):
        if not is_last:
            out.append(RecvBackward(mb))
        out.append(Backward(mb))
        if not is_first:
            out.append(SendBackward(mb))
    return out


def one_f_one_b_schedule(num_microbatches: int, pp_size: int, pp_rank: int) -> list[PPAction]:
    if num_microbatches < 1:
        raise ValueError(f"num_microbatches must be >= 1, got {num_microbatches}")
    if pp_size < 1:
        raise ValueError(f"pp_size must be >= 1, got {pp_size}")
    if not 0 <= pp_rank < pp_size:
        raise ValueError(f"pp_rank must be in [0, {pp_size}), got {pp_rank}")
    first, last = pp_rank == 0, pp_rank == pp_size - 1
    warm = min(pp_size - 1 - pp_rank, num_microbatches)
    steady = num_microbatches - warm
    out: list[PPAction] = []
    for j in range(warm):
        if not first:
            out.append(RecvForward(j))
        out.append(Forward(j))
        if not last:
            out.append(SendForward(j))
    for k in range(steady):
        f, b = warm + k, k
        if k == 0 and not first:
            out.append(RecvForward(f))
        out.append(Forward(f))
        if not last:
            out.append(SendForwardRecvBackward(f, b))
        out.append(Backward(b))
        if not first:
            out.append(SendBackward(b) if k == steady - 1 else SendBackwardRecvForward(b, f + 1))
    for j in range(warm):
        b = steady + j
        if not last:
            out.append(RecvBackward(b))
        out.append(Backward(b))
        if not first:
            out.append(SendBackward(b))
    return out
