"""Point-to-point activation/gradient transport between neighbouring pipeline stages.

NCCL (or gloo on CPU) ``batch_isend_irecv``.  On CUDA the operations are issued from a
dedicated communication stream that first waits on the compute stream (so the sent tensor
is ready), and the compute stream waits on the communication stream only when a received
tensor is consumed — the host never blocks, so transfers overlap with compute already
queued.  Combined send+recv operations are submitted together so neighbours can never
deadlock in 1F1B's steady state.  Devices come from the parallel context (one process per
local GPU), not from the global rank as in the reference (single-node only there).

Reference: ``PipelineComm`` (femtotron/parallel/pipeline_parallel/comm_ops.py:33-198), which
issues ``batch_isend_irecv`` on the compute stream and waits on the host (:187-198)."""
from __future__ import annotations

from typing import Optional, Sequence

import torch
import torch.distributed as dist
from torch.distributed import P2POp


class PipelineComm:
    def __init__(self, parallel_ctx, seqlen: int, hidden_size: int, dtype: torch.dtype,
                 device: torch.device | None = None):
        self.ctx = parallel_ctx
        self._act_shape = (seqlen, hidden_size)
        self._dtype = dtype
        self._device = device if device is not None else parallel_ctx.device
        self._stream = torch.cuda.Stream(device=self._device) if self._device.type == "cuda" else None

    @property
    def is_first_stage(self) -> bool:
        return self.ctx.pp_prev_rank is None

    @property
    def is_last_stage(self) -> bool:
        return self.ctx.pp_next_rank is None

    @property
    def act_shape(self):
        return self._act_shape

    @property
    def dtype(self):
        return self._dtype

    def send_forward(self, act: torch.Tensor) -> None:
        if not self.is_last_stage:
            self._batch([(dist.isend, act, self.ctx.pp_next_rank)])

    def recv_forward(self, out: Optional[torch.Tensor] = None):
        if self.is_first_stage:
            return None
        buf = self._buf(out)
        self._batch([(dist.irecv, buf, self.ctx.pp_prev_rank)])
        return buf

    def send_backward(self, grad: torch.Tensor) -> None:
        if not self.is_first_stage:
            self._batch([(dist.isend, grad, self.ctx.pp_prev_rank)])

    def recv_backward(self, out: Optional[torch.Tensor] = None):
        if self.is_last_stage:
            return None
        buf = self._buf(out)
        self._batch([(dist.irecv, buf, self.ctx.pp_next_rank)])
        return buf

    def send_forward_recv_backward(self, act, out=None):
        if self.is_last_stage:
            return None
        buf = self._buf(out)
        self._batch([(dist.isend, act, self.ctx.pp_next_rank), (dist.irecv, buf, self.ctx.pp_next_rank)])
        return buf

    def send_backward_recv_forward(self, grad, out=None):
        if self.is_first_stage:
            return None
        buf = self._buf(out)
        self._batch([(dist.isend, grad, self.ctx.pp_prev_rank), (dist.irecv, buf, self.ctx.pp_prev_rank)])
        return buf

    def _buf(self, out):
        if out is None:
            return torch.empty(self._act_shape, dtype=self._dtype, device=self._device)
        if out.dtype != self._dtype:
            raise ValueError(f"out buffer dtype {out.dtype} != expected {self._dtype}")
        if out.device != self._device:
            raise ValueError(f"out buffer device {out.device} != expected {self._device}")
        return out

    def _batch(self, specs: Sequence[tuple]) -> None:
        tensors = [t.contiguous() if not t.is_contiguous() else t for _, t, _ in specs]
        ops = [P2POp(fn, t, peer, self.ctx.pp_group) for (fn, _, peer), t in zip(specs, tensors)]
        if self._stream is None:
            for r in dist.batch_isend_irecv(ops):
                r.wait()
            return
        cur = torch.cuda.current_stream(self._device)
        self._stream.wait_stream(cur)
        with torch.cuda.stream(self._stream):
            reqs = dist.batch_isend_irecv(ops)
            for r in reqs:
                r.wait()  # stream-ordered: makes the comm stream wait, not the host
        for t in tensors:
            t.record_stream(self._stream)
        # Only a receive has a consumer on the compute stream; a pure send lets the compute
        # stream run on (the caching allocator keeps the sent tensor alive through
        # record_stream, and sent activations / gradients are not modified in place).
        if any(fn is dist.irecv for fn, _, _ in specs):
            cur.wait_stream(self._stream)
