"""Data-parallel gradient averaging for replicated (ZeRO-0) training.

Where the reference all-reduces every gradient tensor separately
(femtotron/parallel/data_parallel/ddp.py:43-61), this packs the gradients into buckets of
about ``bucket_mb`` megabytes and all-reduces each bucket once (AVG), then copies back.  On
GPUs with NVLS multicast (and FT_NVLS not 0) a bucket is packed straight into a multicast
buffer and reduced in the switch (``parallel/nvls.py``); otherwise NCCL all-reduces it."""
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
        self._nvls = None
        self._nvls_tried = False

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

    def _nvls_for(self, bucket):
        """The NVLS buffer (created on first use, sized for the largest bucket), or None."""
        t0 = bucket[0]
        if not self._nvls_tried:
            self._nvls_tried = True
            from femtotron_b200.parallel.nvls import NVLSAllReduce, nvls_available
            if nvls_available(t0.device):
                # a bucket closes at the first tensor that makes it reach bucket_bytes
                largest = max([g.numel() * g.element_size() for g in
                               (local_grad(pg.compute) for pg in self.groups) if g is not None] or [0])
                self._nvls = NVLSAllReduce(self.dp_group, self.bucket_bytes + largest, t0.device)
        nv = self._nvls
        if nv is None or t0.dtype not in (torch.float32, torch.bfloat16):
            return None
        if sum(t.numel() * t.element_size() for t in bucket) > nv.data_bytes:
            return None
        return nv

    def _reduce(self, bucket) -> None:
        nv = self._nvls_for(bucket) if bucket[0].is_cuda else None
        if nv is not None:
            nv.all_reduce_many_(bucket, average=True)
            return
        flat = _flatten_dense_tensors(bucket)
        dist.all_reduce(flat, op=dist.ReduceOp.AVG, group=self.dp_group)
        for t, r in zip(bucket, _unflatten_dense_tensors(flat, bucket)):
            t.copy_(r)

    def close(self) -> None:
        """Release the NVLS buffer on every rank together (a later sync creates a new one)."""
        if self._nvls is not None:
            self._nvls.close()
            self._nvls = None
        self._nvls_tried = False

    def state_dict(self) -> dict:
        return {}

    def load_state_dict(self, sd: dict) -> None:
        pass
