"""PP-aware causal-LM base (reference femtotron/model/base.py:7-31): subclasses provide
``self.model`` (backbone) and ``self.lm_head``; this class runs the head and the loss.

The loss is the mean next-token cross-entropy over positions whose shifted label is not
-100, like the reference's ``F.cross_entropy(logits[..., :-1, :], labels[..., 1:])``, but
computed by the fused vocab-parallel LM-head kernel path: the logits of each vocab shard are
consumed in place and never gathered.  ``logits`` are materialised (and gathered across TP)
only when no labels are given or ``materialize_logits=True``.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from femtotron_b200.ops.functional import LMHeadCrossEntropyFn, shift_labels
from femtotron_b200.parallel.tensor_parallel import comm_ops as C
from femtotron_b200.parallel.tensor_parallel.linear import ColumnParallelLinear


def lm_head_loss(lm_head: nn.Module, hidden: torch.Tensor, labels: torch.Tensor,
                 ignore_index: int = -100) -> torch.Tensor:
    lab = shift_labels(labels, ignore_index)
    if isinstance(lm_head, ColumnParallelLinear) and lm_head.bias is None:
        group = lm_head.group if lm_head.world_size > 1 else None
        h = hidden.reshape(-1, hidden.shape[-1])
        if group is not None:
            h = C.gather_from_sp(h, group) if lm_head.sequence_parallel or h.shape[0] != lab.numel() \
                else C.copy_to_tp(h, group)
        vstart = lm_head.rank * lm_head.out_features
        return LMHeadCrossEntropyFn.apply(h, lm_head.weight, lab, vstart, group, ignore_index)
    if type(lm_head) is nn.Linear and lm_head.bias is None:
        h = hidden.reshape(-1, hidden.shape[-1])
        return LMHeadCrossEntropyFn.apply(h, lm_head.weight, lab, 0, None, ignore_index)
    logits = lm_head(hidden)
    return F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), lab.reshape(-1),
                           ignore_index=ignore_index)


def full_logits(lm_head: nn.Module, hidden: torch.Tensor, batch_shape) -> torch.Tensor:
    h = hidden
    if isinstance(lm_head, ColumnParallelLinear) and lm_head.sequence_parallel and lm_head.world_size > 1:
        h = C.gather_from_sp(h.reshape(-1, h.shape[-1]), lm_head.group)
    logits = lm_head(h)
    return logits.reshape(*batch_shape, logits.shape[-1])


class BaseCausalLMPipeline(nn.Module):
    is_first: bool
    is_last: bool
    hidden_size: int

    def forward(self, x, labels=None, materialize_logits: bool | None = None) -> dict:
        hidden = self.model(x)
        if not self.is_last:
            return {"loss": None, "logits": None, "hidden_states": hidden}
        batch_shape = tuple(labels.shape) if labels is not None else tuple(x.shape[:2])
        loss = lm_head_loss(self.lm_head, hidden, labels) if labels is not None else None
        want = materialize_logits if materialize_logits is not None else labels is None
        logits = full_logits(self.lm_head, hidden, batch_shape) if want else None
        return {"loss": loss, "logits": logits, "hidden_states": None}
