"""Data-parallel gradient averaging for replicated (ZeRO-0) training.

Where the reference all-reduces every gradient tensor separately
(femtotron/parallel/data_parallel/ddp.py:43-61), this flattens the gradients into buckets of
about ``bucket_mb`` megabytes and all-reduces each bucket once (AVG), then copies back."""
from __future__ import annotations

from contextlib import contextmanager

import torch
import torch.distributed as dist
from torch._utils import _flatten_dense_tensors, _unflatten_dense_tensors

from femtotron_b200.training.param_group import local_grad


class DataParallelGradSync:
    def __init__(self, groups, parallel_ctx, bucket_mb: int = 256):
        self.groups = groups
        self.parallel_ctx = parallel_ctx
        self.dp_group = parallel_ctx.dp_group
        self.bucket_bytes = bucket_mb << 20
        self._sync_enabled = True

    @contextmanager
    def no_sync(self):
        prev = self._sync_enabled
        self._sync_enabled = False
        try:
            yield
        finally:
            self._sync_enabled = prev

    def sync_gradients(self) -> None:
        if not self._sync_enabled or self.parallel_ctx.dp_size <= 1:
            return
        grads = [g for g in (local_grad(pg.compute) for pg in self.groups) if g is not None]
        by_dtype: dict = {}
        for g in grads:
            by_dtype.setdefault(g.dtype, []).append(g)
        for ts in by_dtype.values():
            bucket, size = [], 0
            for t in ts:
                bucket.append(t)
                size += t.numel() * t.element_size()
                if size >= self.bucket_bytes:
                    self._reduce(bucket)
                    bucket, size = [], 0
            if bucket:
                self._reduce(bucket)

    def _reduce(self, bucket) -> None:
        flat = _flatten_dense_tensors(bucket)
        dist.all_reduce(flat, op=dist.ReduceOp.AVG, group=self.dp_group)
        for t, r in zip(bucket, _unflatten_dense_tensors(flat, bucket)):
            t.copy_(r)

    def state_dict(self) -> dict:
        return {}

    def load_state_dict(self, sd: dict) -> None:
        pass
