"""Per-rank pipeline execution unit holding per-micro-batch tensors.

Same lifecycle and invariants as the reference stage
(femtotron/parallel/pipeline_parallel/stage.py:46-361): every cached entry has exactly one
owner that pops it; calling the methods out of order raises with the micro-batch id;
``assert_clean`` detects schedule bugs at the end of a step; ``reset`` recovers after an
exception.  The last stage scales its loss by ``loss_scale`` (1/num_microbatches for
gradient-accumulation equivalence) before the backward."""
from __future__ import annotations

import torch
from torch import nn


class PipelineStage:
    def __init__(self, model: nn.Module, parallel_ctx, *, loss_scale: float = 1.0):
        for attr in ("is_first", "is_last"):
            if not hasattr(model, attr):
                raise TypeError(f"model must expose '{attr}' (pipeline causal-LM protocol)")
        if not callable(getattr(model, "forward", None)):
            raise TypeError("model must have a callable forward")
        self.model = model
        self.parallel_ctx = parallel_ctx
        self.loss_scale = float(loss_scale)
        self.is_first = bool(model.is_first)
        self.is_last = bool(model.is_last)
        self._inputs: dict[int, torch.Tensor] = {}
        self._outputs: dict[int, torch.Tensor] = {}
        self._labels: dict[int, torch.Tensor] = {}
        self._pending_grad_outputs: dict[int, torch.Tensor] = {}
        self._input_grads: dict[int, torch.Tensor] = {}
        self._loss_values: dict[int, torch.Tensor] = {}

    def stage_input(self, mb_id: int, x: torch.Tensor) -> None:
        if mb_id in self._inputs:
            raise RuntimeError(f"stage_input({mb_id}): input already staged")
        if not self.is_first:
            if x.grad_fn is not None:
                raise RuntimeError(f"stage_input({mb_id}): non-first stage expects a leaf tensor")
            if not x.dtype.is_floating_point:
                raise TypeError(f"stage_input({mb_id}): non-first stage expects float hidden states, got {x.dtype}")
            x = x.detach().requires_grad_(True)
        self._inputs[mb_id] = x

    def stage_labels(self, mb_id: int, labels: torch.Tensor) -> None:
        if not self.is_last:
            raise RuntimeError(f"stage_labels({mb_id}): only the last stage takes labels")
        if mb_id in self._labels:
            raise RuntimeError(f"stage_labels({mb_id}): labels already staged")
        self._labels[mb_id] = labels

    def forward(self, mb_id: int) -> None:
        if mb_id not in self._inputs:
            raise RuntimeError(f"forward({mb_id}): no input staged")
        if mb_id in self._outputs:
            raise RuntimeError(f"forward({mb_id}): output already exists (duplicate forward?)")
        labels = None
        if self.is_last:
            if mb_id not in self._labels:
                raise RuntimeError(f"forward({mb_id}): last stage requires labels")
            labels = self._labels[mb_id]
        out = self.model(self._inputs[mb_id], labels=labels)
        if self.is_last:
            self._labels.pop(mb_id)
            if labels is not None:
                loss = out["loss"]
                self._outputs[mb_id] = loss * self.loss_scale if self.loss_scale != 1.0 else loss
            else:
                self._outputs[mb_id] = out["logits"]
        else:
            self._outputs[mb_id] = out["hidden_states"]

    def get_output(self, mb_id: int) -> torch.Tensor:
        if mb_id not in self._outputs:
            raise RuntimeError(f"get_output({mb_id}): no output cached")
        return self._outputs[mb_id]

    def stage_grad(self, mb_id: int, grad: torch.Tensor) -> None:
        if self.is_last:
            raise RuntimeError(f"stage_grad({mb_id}): the last stage starts backward from its loss")
        if mb_id in self._pending_grad_outputs:
            raise RuntimeError(f"stage_grad({mb_id}): grad already staged")
        self._pending_grad_outputs[mb_id] = grad

    def backward(self, mb_id: int) -> None:
        if mb_id not in self._outputs:
            raise RuntimeError(f"backward({mb_id}): no output")
        if mb_id not in self._inputs:
            raise RuntimeError(f"backward({mb_id}): input missing but output exists")
        if not self.is_last and mb_id not in self._pending_grad_outputs:
            raise RuntimeError(f"backward({mb_id}): non-last stage requires grad_output")
        output = self._outputs.pop(mb_id)
        inp = self._inputs.pop(mb_id)
        if self.is_last:
            self._loss_values[mb_id] = output.detach()
            output.backward()
        else:
            output.backward(self._pending_grad_outputs.pop(mb_id))
        if not self.is_first:
            if inp.grad is None:
                raise RuntimeError(f"backward({mb_id}): input.grad is None on a non-first stage")
            self._input_grads[mb_id] = inp.grad
            inp.grad = None

    def get_input_grad(self, mb_id: int) -> torch.Tensor:
        if self.is_first:
            raise RuntimeError(f"get_input_grad({mb_id}): first stage has no upstream")
        if mb_id not in self._input_grads:
            raise RuntimeError(f"get_input_grad({mb_id}): no input grad cached")
        return self._input_grads.pop(mb_id)

    def pop_all_losses(self) -> dict[int, torch.Tensor]:
        out, self._loss_values = self._loss_values, {}
        return out

    def assert_clean(self) -> None:
        left = [f"  {n}: mb_ids={sorted(d)}" for n, d in (
            ("_inputs", self._inputs), ("_outputs", self._outputs), ("_labels", self._labels),
            ("_pending_grad_outputs", self._pending_grad_outputs), ("_input_grads", self._input_grads)) if d]
        if left:
            raise RuntimeError("PipelineStage has leftover per-microbatch state:\n" + "\n".join(left))

    def reset(self) -> None:
        for d in (self._inputs, self._outputs, self._labels, self._pending_grad_outputs,
                  self._input_grads, self._loss_values):
            d.clear()
