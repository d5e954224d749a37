"""Fused tensor-parallel communication for sequence parallelism on NVLink (one process per
GPU): all-gather -> GEMM and GEMM -> reduce-scatter driven by this library's kernels.

All-gather (AG) of a token-sharded activation x_local [Tl, H] into x_full [T = tp*Tl, H]:
  1. after a bounded wait for every peer's DONE flag of two epochs ago (they finished reading
     this slot), the rank stages x_local in its symmetric slot and writes epoch e into every
     peer's READY[me] flag (stream memory write, system-scope fence first);
  2. every chunk is brought into x_full on its own stream, one stream per rank in ring order
     starting with this rank: a one-warp kernel waits (bounded) for the owner's READY flag,
     the copy engines pull the chunk over NVLink (so several engines run at once and no SM
     moves bytes), and a stream write sets the chunk's flag to e; once every chunk is in, a
     stream writes DONE[me] = e into every peer (FT_TP_AG=sm instead runs ``ag_pull``, a pull
     kernel on the SMs the GEMM leaves free, which bumps per-chunk counters);
  3. the consuming GEMM runs on the compute stream at once, leaving two SMs to the flag waits:
     its TMA producer waits (bounded) until the flag of every chunk its tile rows touch has
     reached e, its tiles start at this rank's own rows and follow the ring order, so MMAs on
     the local chunk start immediately and peer rows are consumed as they land; every remote
     row crosses NVLink exactly once.
Reduce-scatter (RS) of a row-parallel GEMM's partial output over tokens:
  1. after a bounded wait for every peer's CONS flag of two epochs ago, the GEMM stores its
     full partial [T, N] into this rank's symmetric slot (local stores) and the stream writes
     PART[me] = e into every peer;
  2. the owner of rows [me*Tl, (me+1)*Tl) runs ``rs_pull``: it waits (bounded) for every
     PART flag, sums those rows of every peer's slot in fp32 over NVLink, adds the residual,
     writes bf16, and then the stream writes CONS[me] = e into every peer.
These paths replace the reference's TP collectives around the column- and row-parallel
linears (femtotron/parallel/tensor_parallel/linear.py:66-77, :194-210): the backward
all-reduce of ``CopyToTPRegion`` and the forward all-reduce of ``ReduceFromTPRegion``
(femtotron/parallel/tensor_parallel/comm_ops.py:33, :117), which the reference issues with no
sequence parallelism.

Slots are double-buffered per direction; epochs increase monotonically and every rank makes
the same sequence of calls, so stale flags are never mistaken for fresh ones.

Every wait is a kernel with a time limit (FT_COMM_TIMEOUT_MS, default 30 s): a peer that never
publishes makes the waiting rank record an error code (200 + flag-kind offset + peer) and
continue, and the host raises KernelTimeoutError at its next ``check_kernel_errors``.  The
gated GEMM leaves SMs free for the kernels that release it (two for the flag waits of the
copy-engine mode, ``gate_reserved_sms()`` for the pull kernel), so they always run side by
side.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from femtotron_b200.ops.ext import error_flag, native
from femtotron_b200.parallel.symm import SymmetricAllocator, SymmetricHeap

KINDS = ("READY", "DONE", "PART", "CONS", "CHUNK")
NSLOTS = 2
# bound of every cross-rank flag wait; a peer that late has failed
COMM_TIMEOUT_MS = int(os.environ.get("FT_COMM_TIMEOUT_MS", "30000"))
# error code base per waited flag kind (code = base + index of the first missing peer)
WAIT_CODES = {"READY": 200, "DONE": 220, "PART": 240, "CONS": 260}
# SMs a gated GEMM leaves to the one-warp flag waits of the copy-engine all-gather
CE_RESERVED_SMS = 2


class TPFusedComm:
    def __init__(self, group, rank: int, world: int, rows_local: int, cols: int, device):
        self.group, self.rank, self.world = group, rank, world
        self.rows_local, self.cols = rows_local, cols
        self.device = device
        self.slot_elems = rows_local * cols
        sb = self.slot_elems * 2
        a = SymmetricAllocator()
        self.off_ag = a.reserve("ag", NSLOTS * sb)              # this rank's staged shard
        self.off_rs = a.reserve("rs", NSLOTS * world * sb)      # this rank's full partial
        self.off_flags = a.reserve("flags", len(KINDS) * 64 * 4)
        self.heap = SymmetricHeap(group, None, a.size, device)
        self.cs = torch.cuda.Stream(device=device)
        # all-gather mover: copy engines, one stream per chunk ("ce"), or the SM pull kernel
        self.ag_mode = os.environ.get("FT_TP_AG", "ce")
        if self.ag_mode == "sm":
            self.ctas = int(native().gate_reserved_sms())
        else:
            self.ctas = CE_RESERVED_SMS
            self.pull_streams = [torch.cuda.Stream(device=device) for _ in range(world)]
        self.ag_epoch = 0
        self.rs_epoch = 0

    # ------------------------------------------------------------------ flags
    def _flag_off(self, kind: str, idx: int) -> int:
        return self.off_flags + (KINDS.index(kind) * 64 + idx) * 4

    def local_flag(self, kind: str, idx: int) -> int:
        return self.heap.peer_ptr(self.rank, self._flag_off(kind, idx))

    def peer_flag(self, owner: int, kind: str, idx: int) -> int:
        return self.heap.peer_ptr(owner, self._flag_off(kind, idx))

    def wait_all(self, kind: str, epoch: int) -> None:
        """Bounded wait, on the current stream, until every rank's `kind` flag here >= epoch."""
        native().wait_flags_geq([self.local_flag(kind, r) for r in range(self.world)], epoch,
                                error_flag(self.device), COMM_TIMEOUT_MS, WAIT_CODES[kind])

    def publish(self, kind: str, epoch: int) -> None:
        """Write epoch into every rank's `kind`[me] flag once the current stream's work is done."""
        C = native()
        for r in range(self.world):
            C.stream_write(self.peer_flag(r, kind, self.rank), epoch)

    def fits(self, rows_local: int, cols: int) -> bool:
        return rows_local * cols <= self.slot_elems

    # ------------------------------------------------------------------ all-gather
    def all_gather(self, x_local: torch.Tensor):
        """Start gathering x_local [Tl, H] (bf16, contiguous); returns (x_full, epoch).  The
        rows of rank r are valid once CHUNK[r] >= epoch x CTAs (gate the consuming GEMM on
        it); work queued on the current stream after ``after_gated`` sees x_full complete."""
        Tl, H = x_local.shape
        e = self.ag_epoch = self.ag_epoch + 1
        s = e % NSLOTS
        cur = torch.cuda.current_stream(self.device)
        if e > NSLOTS:
            self.wait_all("DONE", e - NSLOTS)
        slot_off = self.off_ag + s * self.slot_elems * 2
        self.heap.view(slot_off, Tl * H, torch.bfloat16).copy_(x_local.reshape(-1))
        self.publish("READY", e)
        full = torch.empty(self.world * Tl, H, dtype=torch.bfloat16, device=self.device)
        C = native()
        if self.ag_mode == "sm":
            self.cs.wait_stream(cur)
            with torch.cuda.stream(self.cs):
                C.ag_pull([self.heap.peer_ptr(r, slot_off) for r in range(self.world)],
                          [self.local_flag("READY", r) for r in range(self.world)],
                          full, Tl * H * 2, self.local_flag("CHUNK", 0), self.rank, e,
                          self.ctas, error_flag(self.device), COMM_TIMEOUT_MS)
                self.publish("DONE", e)
            full.record_stream(self.cs)
            return full, e
        nb = Tl * H * 2
        for k in range(self.world):
            r = (self.rank + k) % self.world
            st = self.pull_streams[k]
            st.wait_stream(cur)
            with torch.cuda.stream(st):
                if r != self.rank:
                    C.wait_flags_geq([self.local_flag("READY", r)], e, error_flag(self.device),
                                     COMM_TIMEOUT_MS, WAIT_CODES["READY"] + r)
                C.copy_from_ptrs([full.data_ptr() + r * nb], [self.heap.peer_ptr(r, slot_off)], [nb])
                C.stream_write(self.local_flag("CHUNK", r), e)
            full.record_stream(st)
            self.cs.wait_stream(st)
        with torch.cuda.stream(self.cs):
            self.publish("DONE", e)      # every peer's slot read: the owners may reuse it
        return full, e

    def gate(self, epoch: int, rows_local: int, cols: int) -> dict:
        """Operand gate of the consuming GEMM.  Its tiles start at this rank's own rows, the
        chunk the pull kernel copies first, and follow the ring order of the pulls."""
        rot = self.rank * rows_local
        target = epoch * self.ctas if self.ag_mode == "sm" else epoch   # counters or epochs
        return dict(gate_flags=self.local_flag("CHUNK", 0), gate_op=1, gate_epoch=target,
                    gate_off=0, gate_row_elems=cols, gate_chunk_elems=rows_local * cols,
                    gate_rot_rows=rot if rot % 256 == 0 else 0, gate_reserved=self.ctas)

    def after_gated(self) -> None:
        """Order later work on the current stream after every chunk's transfer."""
        torch.cuda.current_stream(self.device).wait_stream(self.cs)

    # ------------------------------------------------------------------ reduce-scatter
    def rs_begin(self, rows_local: int, cols: int):
        """Returns (epoch, partial): the [T, cols] buffer the row-parallel GEMM stores into."""
        e = self.rs_epoch = self.rs_epoch + 1
        s = e % NSLOTS
        if e > NSLOTS:
            self.wait_all("CONS", e - NSLOTS)
        T = self.world * rows_local
        off = self.off_rs + s * self.world * self.slot_elems * 2
        return e, self.heap.view(off, T * cols, torch.bfloat16).view(T, cols)

    def rs_publish(self, e: int) -> None:
        """Tell every peer that this rank's partial of epoch e is complete."""
        self.publish("PART", e)

    def rs_finish(self, e: int, rows_local: int, cols: int, residual: torch.Tensor | None,
                  published: bool = False):
        """This rank's rows of the sum over ranks of the partials (+ residual)."""
        if not published:
            self.rs_publish(e)
        s = e % NSLOTS
        n = rows_local * cols
        base = self.off_rs + s * self.world * self.slot_elems * 2 + self.rank * n * 2
        out = torch.empty(rows_local, cols, dtype=torch.bfloat16, device=self.device)
        native().rs_pull([self.heap.peer_ptr(r, base) for r in range(self.world)],
                         [self.local_flag("PART", r) for r in range(self.world)],
                         residual.reshape(-1) if residual is not None else None, out, n, e,
                         error_flag(self.device), COMM_TIMEOUT_MS)
        self.publish("CONS", e)
        return out

    def close(self):
        torch.cuda.synchronize(self.device)
        self.heap.close()


def fused_gemm(a, b, out, *, a_mn=False, b_mn=False, mode="store_bf16", residual=None, gu=None,
               gate_up_off=0, gate: dict | None = None, scatter=None):
    """GEMM with an optional operand gate and scatter epilogue (CUDA only)."""
    from femtotron_b200.ops.matmul import EPI_MODES
    g = gate or {}
    ptrs, rows = (scatter if scatter is not None else ([], 0))
    m = 6 if scatter is not None else EPI_MODES[mode]
    native().gemm_tc_fused(a, b, out, a_mn, b_mn, m, residual, gu, gate_up_off, error_flag(a.device),
                           g.get("gate_flags", 0), g.get("gate_op", 0), g.get("gate_epoch", 0),
                           g.get("gate_off", 0), g.get("gate_row_elems", 1), g.get("gate_chunk_elems", 1),
                           list(ptrs), rows, g.get("gate_rot_rows", 0), g.get("gate_reserved", 0))
    return out


_COMMS: dict = {}


def tp_fused_comm(group, rows_local: int, cols: int, device) -> TPFusedComm | None:
    """The fused-communication object of a TP group, (re)created for the needed size."""
    if group is None or not torch.cuda.is_available() or device.type != "cuda":
        return None
    key = (id(group), device.index)
    c = _COMMS.get(key)
    if c is None or not c.fits(rows_local, cols):
        if c is not None:
            c.close()
        c = TPFusedComm(group, dist.get_rank(group), dist.get_world_size(group), rows_local, cols, device)
        _COMMS[key] = c
    return c


# ------------------------------------------------------------------------------ autograd
from torch.autograd import Function  # noqa: E402

from femtotron_b200.ops import kernels as K  # noqa: E402
from femtotron_b200.ops.functional import cat_rows_view, write_weight_grad  # noqa: E402
from femtotron_b200.ops.matmul import gemm, linear_wgrad  # noqa: E402


def _dgrad_rs(comm, d, W, Tl, H):
    """Start dx_local [Tl, H] = reduce-scatter over tokens of d [T, N] @ W [N, H]: the dgrad
    GEMM stores the partial into the symmetric slot and the peers are told at once."""
    e, part = comm.rs_begin(Tl, H)
    gemm(d, W, part, b_mn=True)
    comm.rs_publish(e)
    return e


class SPColumnFn(Function):
    """Column-parallel projection of a token-sharded input under sequence parallelism:
    fused all-gather -> GEMM forward, fused GEMM -> reduce-scatter backward.
    kind: "linear" | "qkv_rope" (args: cos, sin, pos, n_rot, head_dim, seq) | "swiglu"."""

    @staticmethod
    def forward(ctx, x_local, comm, kind, rope_args, *weights):
        x2 = x_local.reshape(-1, x_local.shape[-1]).contiguous()
        Tl, H = x2.shape
        full, e = comm.all_gather(x2)
        gate = comm.gate(e, Tl, H)
        W = cat_rows_view(weights)
        T = full.shape[0]
        if kind == "swiglu":
            F_ = weights[0].shape[0]
            out = torch.empty(T, F_, dtype=x2.dtype, device=x2.device)
            gu = torch.empty(T, 2 * F_, dtype=x2.dtype, device=x2.device)
            fused_gemm(full, W, out, mode="swiglu", gu=gu, gate_up_off=F_, gate=gate)
            comm.after_gated()
            ctx.save_for_backward(full, gu, *[w.detach() for w in weights])
        else:
            out = torch.empty(T, W.shape[0], dtype=x2.dtype, device=x2.device)
            fused_gemm(full, W, out, gate=gate)
            comm.after_gated()
            if kind == "qkv_rope":
                cos, sin, pos, n_rot, hd, S = rope_args
                K.rope_(out, cos, sin, n_rot, hd, S, pos=pos)
            ctx.save_for_backward(full, *[w.detach() for w in weights])
        ctx.comm, ctx.kind, ctx.rope_args, ctx.params = comm, kind, rope_args, weights
        ctx.Tl, ctx.H, ctx.xshape = Tl, H, x_local.shape
        return out

    @staticmethod
    def backward(ctx, dout):
        comm, kind = ctx.comm, ctx.kind
        if kind == "swiglu":
            full, gu, *ws = ctx.saved_tensors
            d = K.swiglu_bwd(dout.contiguous(), gu, ws[0].shape[0], out=gu)
        else:
            full, *ws = ctx.saved_tensors
            d = dout.contiguous()
            if kind == "qkv_rope":
                cos, sin, pos, n_rot, hd, S = ctx.rope_args
                d = K.rope_(d.clone(), cos, sin, n_rot, hd, S, inverse=True, pos=pos)
        W = cat_rows_view(ws)
        e = _dgrad_rs(comm, d, W, ctx.Tl, ctx.H)
        write_weight_grad(ctx.params, lambda dst, acc: linear_wgrad(d, full, dst, acc))
        dx = comm.rs_finish(e, ctx.Tl, ctx.H, None, published=True)
        ctx.params = None
        return (dx.view(ctx.xshape), None, None, None) + (None,) * len(ws)


class SPRowFn(Function):
    """Row-parallel projection under sequence parallelism: GEMM into the symmetric partial
    slot, owner-side pull and sum of the partials plus the residual (fused GEMM ->
    reduce-scatter); backward gathers the output gradient with the fused all-gather."""

    @staticmethod
    def forward(ctx, h, residual, comm, *weights):
        h2 = h.reshape(-1, h.shape[-1]).contiguous()
        W = cat_rows_view(weights)
        T, N = h2.shape[0], W.shape[0]
        Tl = T // comm.world
        e, part = comm.rs_begin(Tl, N)
        gemm(h2, W, part)
        res = residual.reshape(-1, N).contiguous() if residual is not None else None
        out = comm.rs_finish(e, Tl, N, res)
        ctx.save_for_backward(h2, *[w.detach() for w in weights])
        ctx.comm, ctx.params, ctx.has_res, ctx.Tl, ctx.hshape = comm, weights, residual is not None, Tl, h.shape
        return out

    @staticmethod
    def backward(ctx, dout):
        comm = ctx.comm
        h2, *ws = ctx.saved_tensors
        W = cat_rows_view(ws)
        d2 = dout.reshape(-1, dout.shape[-1]).contiguous()
        Tl, N = d2.shape
        dfull, e = comm.all_gather(d2)
        dh = torch.empty(dfull.shape[0], W.shape[1], dtype=h2.dtype, device=h2.device)
        fused_gemm(dfull, W, dh, b_mn=True, gate=comm.gate(e, Tl, N))
        comm.after_gated()
        write_weight_grad(ctx.params, lambda dst, acc: linear_wgrad(dfull, h2, dst, acc))
        ctx.params = None
        return (dh.view(ctx.hshape), dout if ctx.has_res else None, None) + (None,) * len(ws)
