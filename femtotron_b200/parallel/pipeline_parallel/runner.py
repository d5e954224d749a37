"""Stateless pipeline dispatcher: executes a schedule's actions against a stage and a comm
object (reference femtotron/parallel/pipeline_parallel/runner.py:28-199)."""
from __future__ import annotations

import torch

from .action import (Backward, Forward, PPAction, RecvBackward, RecvForward, SendBackward,
                     SendBackwardRecvForward, SendForward, SendForwardRecvBackward)
from .microbatch import split_microbatches
from .schedule import gpipe_schedule, one_f_one_b_schedule


class PipelineRunner:
    def __init__(self, stage, comm, *, schedule_name: str = "1f1b", num_microbatches: int = 1,
                 recv_shape: tuple, recv_dtype: torch.dtype = torch.bfloat16):
        self.stage = stage
        self.comm = comm
        self.num_microbatches = num_microbatches
        self.recv_shape = tuple(recv_shape)
        self.recv_dtype = recv_dtype
        self.actions = self._build_actions(schedule_name)
        self._device = next(stage.model.parameters()).device

    def run_step(self, batch: dict) -> dict[int, torch.Tensor]:
        inputs = labels = None
        if self.stage.is_first:
            inputs = dict(enumerate(split_microbatches(batch["input_ids"], self.num_microbatches)))
        if self.stage.is_last:
            labels = dict(enumerate(split_microbatches(batch["labels"], self.num_microbatches)))
        return self.run(self.actions, recv_shape=self.recv_shape, recv_dtype=self.recv_dtype,
                        microbatch_inputs=inputs, microbatch_labels=labels)

    def run(self, actions, *, recv_shape, recv_dtype, microbatch_inputs=None, microbatch_labels=None):
        if self.stage.is_first and microbatch_inputs is None:
            raise ValueError("first stage requires microbatch_inputs")
        for a in actions:
            self._dispatch(a, microbatch_inputs, microbatch_labels, recv_shape, recv_dtype)
        losses = self.stage.pop_all_losses()
        self.stage.assert_clean()
        return losses

    def _empty(self, shape, dtype):
        return torch.empty(shape, dtype=dtype, device=self._device)

    def _dispatch(self, a: PPAction, inputs, labels, shape, dtype) -> None:
        st, cm = self.stage, self.comm
        if isinstance(a, Forward):
            if st.is_first:
                if a.mb_id not in inputs:
                    raise RuntimeError(f"first stage missing input for micro-batch {a.mb_id}")
                st.stage_input(a.mb_id, inputs[a.mb_id])
            if st.is_last and labels is not None and a.mb_id in labels:
                st.stage_labels(a.mb_id, labels[a.mb_id])
            st.forward(a.mb_id)
        elif isinstance(a, Backward):
            st.backward(a.mb_id)
        elif isinstance(a, RecvForward):
            buf = self._empty(shape, dtype)
            cm.recv_forward(out=buf)
            st.stage_input(a.mb_id, buf)
        elif isinstance(a, SendForward):
            cm.send_forward(st.get_output(a.mb_id))
        elif isinstance(a, RecvBackward):
            buf = self._empty(shape, dtype)
            cm.recv_backward(out=buf)
            st.stage_grad(a.mb_id, buf)
        elif isinstance(a, SendBackward):
            cm.send_backward(st.get_input_grad(a.mb_id))
        elif isinstance(a, SendForwardRecvBackward):
            buf = self._empty(shape, dtype)
            cm.send_forward_recv_backward(st.get_output(a.fwd_mb), out=buf)
            st.stage_grad(a.bwd_mb, buf)
        elif isinstance(a, SendBackwardRecvForward):
            buf = self._empty(shape, dtype)
            cm.send_backward_recv_forward(st.get_input_grad(a.bwd_mb), out=buf)
            st.stage_input(a.fwd_mb, buf)
        else:
            raise NotImplementedError(f"unsupported action {type(a).__name__}")

    @property
    def is_first_stage(self):
        return self.stage.is_first

    @property
    def is_last_stage(self):
        return self.stage.is_last

    def _build_actions(self, name: str):
        ctx = self.stage.parallel_ctx
        if name == "gpipe":
            return gpipe_schedule(self.num_microbatches, self.stage.is_first, self.stage.is_last)
        if name == "1f1b":
            return one_f_one_b_schedule(self.num_microbatches, ctx.pp_size, ctx.pp_rank)
        raise ValueError(f"unknown schedule {name!r}")
