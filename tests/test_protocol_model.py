"""Model check, on the CPU, of the cross-GPU flag protocols that order this library's NVLink
traffic: the sequence-parallel all-gather -> GEMM and GEMM -> reduce-scatter of
``parallel/tensor_parallel/fused.py`` (both all-gather movers) and the ZeRO-3 gradient
reduce-scatter of ``sharding/param_group_cluster.py::_reduce_symm`` and the in-switch (NVLS)
all-reduce of ``parallel/nvls.py``.

The real Python code of those classes runs for every simulated rank; only the device is
replaced.  Each CUDA stream becomes a FIFO of operations, and each native call becomes the
operation it enqueues: a bounded flag wait, a stream flag write, a copy or pull from a peer's
symmetric slot, a gated GEMM, the fused reduce-scatter + AdamW.  ``wait_stream`` becomes a
wait for the other stream's position.  A scheduler then runs all ranks' streams in random
interleavings, with random per-stream speeds so that some ranks or streams lag far behind.
Every interleaving must

* finish (no rank waits for a flag that is never written: the device waits would time out);
* read every peer slot while it holds the epoch the reader expects (not stale, not already
  overwritten by a later epoch);
* overwrite a slot only after every rank has read its previous content;
* start a gated GEMM only when every chunk of its all-gather is in place;
* never move a flag backwards.

Negative controls remove one ordering at a time (the GEMM's operand gate, the flag wait
before a chunk copy, the wait for partials before the pull-and-sum, the wait for the peers'
DONE flags before a slot is restaged, the wait for peers' gradient flags, the step barrier),
and the checker must report a violation for each, so its silence on the real protocol means
something.  (In the training step's order every all-gather is consumed by a gated GEMM on the
compute stream before the next one starts, which already orders slot reuse; the DONE flags
matter for all-gathers issued back to back, which a separate program checks.)

The host programs replay the call order of the training step: ``SPColumnFn`` / ``SPRowFn``
forward and backward per decoder block, and per step the ZeRO-3 units' backward, their
reduce-scatters, ``wait_comm`` (compute stream waits for the reduce stream) and the
``post_step`` barrier (one all-reduce on the compute stream).
"""
from __future__ import annotations

import contextlib
import random
from collections import defaultdict

import pytest
import torch

import femtotron_b200.ops.ext as ext
import femtotron_b200.parallel.tensor_parallel.fused as fused
from femtotron_b200.sharding.param_group_cluster import ParamGroupCluster

SHIFT = 40


def addr(rank: int, off: int) -> int:
    return ((rank + 1) << SHIFT) | off


def decode(a: int) -> tuple[int, int]:
    return (a >> SHIFT) - 1, a & ((1 << SHIFT) - 1)


class Violation(AssertionError):
    pass


class Deadlock(AssertionError):
    pass


class Op:
    __slots__ = ("what", "run", "ready")

    def __init__(self, what, run=None, ready=None):
        self.what = what
        self.run = run or (lambda: None)
        self.ready = ready or (lambda: True)


class FakeStream:
    def __init__(self, sim, rank: int, name: str):
        self.sim, self.rank, self.name = sim, rank, name
        self.ops: list[Op] = []
        self.pos = 0
        sim.streams.append(self)

    def put(self, op: Op) -> None:
        self.ops.append(op)

    def wait_stream(self, other: "FakeStream") -> None:
        n = len(other.ops)
        self.put(Op(f"wait_stream({other.name} to {n})", ready=lambda: other.pos >= n))

    def __repr__(self):
        return self.name


class Sim:
    """Flags, slot contents and streams of `world` simulated GPUs."""

    def __init__(self, world: int):
        self.world = world
        self.flags: dict[int, int] = defaultdict(int)
        self.streams: list[FakeStream] = []
        self.cur: dict[int, FakeStream] = {}
        self.rank = 0                      # rank whose host program is being recorded
        self.version: dict = {}            # slot key -> epoch it holds
        self.readers = defaultdict(set)    # (slot key, epoch) -> ranks that read it
        self.chunks = defaultdict(set)     # (rank, gather buffer) -> {(chunk, epoch)}
        self.arrivals = defaultdict(set)   # collective instance -> ranks arrived
        self.n_coll = defaultdict(int)
        self.locate = None                 # offset -> (region, index) of a symmetric slot
        self._names = defaultdict(int)

    # --------------------------------------------------------------- recording
    def new_stream(self, rank=None) -> FakeStream:
        r = self.rank if rank is None else rank
        k = self._names[r]
        self._names[r] += 1
        return FakeStream(self, r, f"r{r}.s{k}")

    def put(self, op: Op) -> None:
        self.cur[self.rank].put(op)

    def key(self, a: int):
        owner, off = decode(a)
        return (owner,) + self.locate(off)

    def write_slot(self, key, epoch, writer: int, needed=None) -> Op:
        """Stream write of `epoch` into a slot; `needed(old)`: the ranks that must have read
        the old content first (default: every rank)."""
        def run():
            old = self.version.get(key)
            if old is not None and old != epoch:
                must = set(range(self.world)) if needed is None else needed(old)
                missing = must - self.readers[(key, old)]
                if missing:
                    raise Violation(f"rank {writer} overwrote {key} with epoch {epoch} before "
                                    f"ranks {sorted(missing)} read epoch {old}")
            self.version[key] = epoch
        return Op(f"write {key} <- {epoch}", run)

    def read_slot(self, key, expect: int, reader: int) -> None:
        v = self.version.get(key)
        if v != expect:
            raise Violation(f"rank {reader} read {key} holding epoch {v}, expected {expect}")
        self.readers[(key, v)].add(reader)

    def barrier(self) -> None:
        """A collective on the current stream: done once every rank's stream reached it."""
        r = self.rank
        inst = self.n_coll[r]
        self.n_coll[r] += 1

        def ready():
            self.arrivals[inst].add(r)
            return len(self.arrivals[inst]) == self.world
        self.put(Op(f"barrier {inst}", ready=ready))

    # --------------------------------------------------------------- execution
    def run(self, rng: random.Random) -> None:
        speed = {s.name: 10 ** rng.uniform(-2.5, 0) for s in self.streams}
        while True:
            ready = [s for s in self.streams if s.pos < len(s.ops) and s.ops[s.pos].ready()]
            if not ready:
                left = [s for s in self.streams if s.pos < len(s.ops)]
                if not left:
                    return
                raise Deadlock("; ".join(f"{s.name} at {s.ops[s.pos].what}" for s in left[:8]))
            s = rng.choices(ready, weights=[speed[x.name] for x in ready])[0]
            op = s.ops[s.pos]
            op.run()
            s.pos += 1


class FakeView:
    """A symmetric-heap view: writing into it is a stream-ordered slot write."""

    def __init__(self, sim, rank, off, epoch_of):
        self.sim, self.rank, self.off, self.epoch_of = sim, rank, off, epoch_of

    def view(self, *shape):
        return self

    def copy_(self, src):
        self.sim.put(self.sim.write_slot((self.rank,) + self.sim.locate(self.off),
                                         self.epoch_of(), self.rank))
        return self


class FakeNative:
    """The native entry points the protocols call, as stream operations."""

    def __init__(self, sim: Sim):
        self.sim = sim
        self.comms = {}              # rank -> TPFusedComm (for the epoch of an all-gather copy)
        self.skip_wait_codes = set()  # negative controls: waits that are dropped
        self.ungated = False

    def gate_reserved_sms(self):
        return 16

    def wait_flags_geq(self, addrs, value, err, timeout_ms, code):
        if any(code >= c and code < c + 20 for c in self.skip_wait_codes):
            return
        fl, addrs = self.sim.flags, list(addrs)
        self.sim.put(Op(f"wait code {code} >= {value}",
                        ready=lambda: all(fl[a] >= value for a in addrs)))

    def stream_write(self, a, value):
        sim = self.sim

        def run():
            if sim.flags[a] > value:
                raise Violation(f"flag {decode(a)} moved back from {sim.flags[a]} to {value}")
            sim.flags[a] = value
        sim.put(Op(f"flag {decode(a)} = {value}", run))

    def copy_from_ptrs(self, dsts, srcs, sizes):
        sim, me = self.sim, self.sim.rank
        e = self.comms[me].ag_epoch

        def run():
            for d, s, n in zip(dsts, srcs, sizes):
                owner = decode(s)[0]
                sim.read_slot(sim.key(s), e, me)
                sim.chunks[(me, d - owner * n)].add((owner, e))
        sim.put(Op(f"copy epoch {e}", run))

    def ag_pull(self, src_ptrs, ready_ptrs, dst, chunk_bytes, counter, me, epoch, ctas, err,
                timeout_ms):
        sim, W = self.sim, self.sim.world
        skip = any(200 <= c < 220 for c in self.skip_wait_codes)
        for k in range(W):             # every CTA walks the chunks in ring order
            r = (me + k) % W

            def run(r=r):
                sim.read_slot(sim.key(src_ptrs[r]), epoch, me)
                sim.chunks[(me, dst.data_ptr())].add((r, epoch))
                sim.flags[counter + 4 * r] += ctas
            ready = (lambda: True) if skip else (lambda r=r: sim.flags[ready_ptrs[r]] >= epoch)
            sim.put(Op(f"ag_pull chunk {r} epoch {epoch}", run, ready))

    def gemm_tc_fused(self, a, b, out, a_mn, b_mn, mode, residual, gu, gate_up_off, err,
                      gate_flags, gate_op, gate_epoch, gate_off, gate_row_elems,
                      gate_chunk_elems, scatter_ptrs, scatter_rows, rot_rows, reserved):
        sim, me, W = self.sim, self.sim.rank, self.sim.world
        assert gate_op == 1
        c = self.comms[me]
        e = gate_epoch // c.ctas if c.ag_mode == "sm" else gate_epoch   # the gather's epoch
        flags = [gate_flags + 4 * r for r in range(W)]

        def run():
            have = sim.chunks[(me, a.data_ptr())]
            missing = [r for r in range(W) if (r, e) not in have]
            if missing:
                raise Violation(f"rank {me}: gated GEMM of epoch {e} ran before chunks {missing}")
        ready = (lambda: True) if self.ungated else \
            (lambda: all(sim.flags[f] >= gate_epoch for f in flags))
        sim.put(Op(f"gated GEMM epoch {e}", run, ready))

    def rs_pull(self, src_ptrs, part_ptrs, resid, out, n, e, err, timeout_ms):
        sim, me = self.sim, self.sim.rank
        skip = any(240 <= c < 260 for c in self.skip_wait_codes)

        def run():
            for s in src_ptrs:
                sim.read_slot(sim.key(s), e, me)
        ready = (lambda: True) if skip else (lambda: all(sim.flags[p] >= e for p in part_ptrs))
        sim.put(Op(f"rs_pull epoch {e}", run, ready))

    def rs_adamw(self, srcs, base, n, src_f32, scale, accumulate, grad_shard, store, master,
                 m, v, p16, segments, beta1, beta2, eps, step, expect=None):
        sim, me = self.sim, self.sim.rank
        ep = self.zero_epoch()

        def run():
            for s in srcs:
                sim.read_slot(sim.key(s), ep, me)
        sim.put(Op(f"rs_adamw epoch {ep}", run))


class FakeHeap:
    def __init__(self, sim, rank, epoch_of):
        self.sim, self.rank, self.epoch_of = sim, rank, epoch_of

    def peer_ptr(self, r, off):
        return addr(r, off)

    def view(self, off, numel, dtype):
        return FakeView(self.sim, self.rank, off, lambda: self.epoch_of(off))

    def close(self):
        pass


class FakeGroup:
    def __init__(self, rank):
        self.rank = rank


def patch_device(monkeypatch, sim: Sim, nat: FakeNative):
    @contextlib.contextmanager
    def stream_ctx(st):
        prev = sim.cur[sim.rank]
        sim.cur[sim.rank] = st
        try:
            yield
        finally:
            sim.cur[sim.rank] = prev

    monkeypatch.setattr(torch.cuda, "Stream", lambda device=None, **k: sim.new_stream())
    monkeypatch.setattr(torch.cuda, "current_stream", lambda device=None: sim.cur[sim.rank])
    monkeypatch.setattr(torch.cuda, "stream", stream_ctx)
    monkeypatch.setattr(torch.Tensor, "record_stream", lambda self, s: None)
    monkeypatch.setattr(fused, "native", lambda: nat)
    monkeypatch.setattr(fused, "error_flag", lambda dev: None)
    monkeypatch.setattr(ext, "native", lambda: nat)
    monkeypatch.setattr(ext, "error_flag", lambda dev: None)


# =============================================================== tensor parallel (SP)
def build_tp(monkeypatch, world: int, mode: str, rows_local=4, cols=8):
    sim = Sim(world)
    nat = FakeNative(sim)
    patch_device(monkeypatch, sim, nat)
    monkeypatch.setenv("FT_TP_AG", mode)
    comms = []
    for r in range(world):
        sim.rank = r
        sim.cur[r] = sim.new_stream()

        def heap_factory(group, _unused, size, device, r=r):
            def epoch_of(off, r=r):
                c = nat.comms[r]
                return c.ag_epoch if sim.locate(off)[0] == "ag" else c.rs_epoch
            return FakeHeap(sim, r, epoch_of)
        monkeypatch.setattr(fused, "SymmetricHeap", heap_factory)
        c = fused.TPFusedComm(FakeGroup(r), r, world, rows_local, cols, torch.device("cpu"))
        nat.comms[r] = c
        comms.append(c)
    c0 = comms[0]
    sb = c0.slot_elems * 2

    def locate(off):
        if c0.off_ag <= off < c0.off_ag + fused.NSLOTS * sb:
            return ("ag", (off - c0.off_ag) // sb)
        if c0.off_rs <= off < c0.off_rs + fused.NSLOTS * world * sb:
            return ("rs", (off - c0.off_rs) // (world * sb))
        raise AssertionError(f"offset {off} is in no slot")
    sim.locate = locate
    return sim, nat, comms


def tp_program(sim: Sim, comm, layers: int, keep: list):
    """The communication calls of `layers` sequence-parallel decoder layers, forward then
    backward, in the order SPColumnFn / SPRowFn make them (two blocks per layer: attention
    and MLP, each a column-parallel and a row-parallel projection)."""
    Tl, H = comm.rows_local, comm.cols
    x = torch.zeros(Tl, H, dtype=torch.bfloat16)
    W = torch.zeros(H, H, dtype=torch.bfloat16)

    def gemm_into(part):            # the row-parallel / dgrad GEMM stores its partial
        part.copy_(None)

    for _ in range(layers):
        for _block in range(2):
            full, e = comm.all_gather(x)                       # SPColumnFn.forward
            out = torch.empty(full.shape[0], H, dtype=x.dtype)
            fused.fused_gemm(full, W, out, gate=comm.gate(e, Tl, H))
            comm.after_gated()
            keep += [full, out]
            e2, part = comm.rs_begin(Tl, H)                    # SPRowFn.forward
            gemm_into(part)
            comm.rs_finish(e2, Tl, H, None)
    for _ in range(layers):
        for _block in range(2):
            dfull, e = comm.all_gather(x)                      # SPRowFn.backward
            dh = torch.empty(dfull.shape[0], H, dtype=x.dtype)
            fused.fused_gemm(dfull, W, dh, b_mn=True, gate=comm.gate(e, Tl, H))
            comm.after_gated()
            keep += [dfull, dh]
            e2, part = comm.rs_begin(Tl, H)                    # SPColumnFn.backward
            gemm_into(part)
            comm.rs_publish(e2)
            comm.rs_finish(e2, Tl, H, None, published=True)


def back_to_back_program(sim: Sim, comm, rounds: int, keep: list):
    """Three all-gathers issued before any of them is consumed, so the third restages the
    first one's slot while peers may still be copying it: only the DONE flags order that."""
    Tl, H = comm.rows_local, comm.cols
    x = torch.zeros(Tl, H, dtype=torch.bfloat16)
    W = torch.zeros(H, H, dtype=torch.bfloat16)
    for _ in range(rounds):
        gathered = [comm.all_gather(x) for _ in range(3)]
        for full, e in gathered:
            out = torch.empty(full.shape[0], H, dtype=x.dtype)
            fused.fused_gemm(full, W, out, gate=comm.gate(e, Tl, H))
            keep += [full, out]
        comm.after_gated()


def run_tp(monkeypatch, world, mode, seed, layers=2, control=None, program=tp_program):
    sim, nat, comms = build_tp(monkeypatch, world, mode)
    if control == "ungated":
        nat.ungated = True
    elif control == "no_ready_wait":
        nat.skip_wait_codes.add(fused.WAIT_CODES["READY"])
    elif control == "no_part_wait":
        nat.skip_wait_codes.add(fused.WAIT_CODES["PART"])
    elif control == "no_done_wait":
        nat.skip_wait_codes.add(fused.WAIT_CODES["DONE"])
    keep = []
    for r, c in enumerate(comms):
        sim.rank = r
        program(sim, c, layers, keep)
    sim.run(random.Random(seed))
    # every all-gather and reduce-scatter slot content was read by every rank
    for (key, ep), readers in list(sim.readers.items()):
        assert readers == set(range(world)), (key, ep, readers)
    return sim


@pytest.mark.parametrize("mode", ["ce", "sm"])
@pytest.mark.parametrize("world,seeds", [(2, 40), (3, 25), (4, 20), (8, 6)])
def test_tp_protocol_is_race_and_deadlock_free(monkeypatch, mode, world, seeds):
    for seed in range(seeds):
        sim = run_tp(monkeypatch, world, mode, seed)
        # slots cycled through several epochs (the double buffering was exercised)
        assert max(v for k, v in sim.version.items() if k[1] == "ag") >= 8
        monkeypatch.undo()


@pytest.mark.parametrize("mode,control", [("ce", "ungated"), ("sm", "ungated"),
                                          ("ce", "no_ready_wait"), ("sm", "no_ready_wait"),
                                          ("ce", "no_part_wait")])
def test_tp_checker_catches_a_missing_ordering(monkeypatch, mode, control):
    found = None
    for seed in range(60):
        try:
            run_tp(monkeypatch, 4, mode, seed, control=control)
        except Violation as e:
            found = e
            break
        finally:
            monkeypatch.undo()
    assert found is not None, f"{control}: no interleaving showed the missing ordering"


# =============================================================== ZeRO-3 reduce-scatter
def build_zero(monkeypatch, world: int, units: int, early: bool):
    sim = Sim(world)
    nat = FakeNative(sim)
    patch_device(monkeypatch, sim, nat)
    UNIT, FLAGS = 1 << 20, 1 << 30      # grad buffer offsets and flag arrays per unit
    sim.locate = lambda off: ("grad", off // UNIT) if off < FLAGS else ("flags", 0)
    ranks = []
    for r in range(world):
        sim.rank = r
        cur = sim.cur[r] = sim.new_stream()
        rs = sim.new_stream()
        heap = FakeHeap(sim, r, None)
        cl = []
        for u in range(units):
            c = object.__new__(ParamGroupCluster)
            c.__dict__.update(
                name=f"unit{u}", device=torch.device("cpu"), direct=False, dp_size=world,
                dp_rank=r, symm=(heap,), flag_offset=FLAGS + u * 4 * 64, grad_offset=u * UNIT,
                shard_size=16, grad_dtype=torch.float32, rs_stream=rs, comm_stream=None,
                _rs_epoch=0, _flat_grad_shard=torch.zeros(16), updated_early=False,
                master=torch.zeros(16), flat_param_shard=torch.zeros(16, dtype=torch.bfloat16),
                early_update=None)
            if early:
                c.early_update = lambda c: dict(exp_avg=torch.zeros(16), exp_avg_sq=torch.zeros(16),
                                                segments=torch.zeros(1, 4, dtype=torch.float64),
                                                beta1=0.9, beta2=0.95, eps=1e-8, step=1)
            cl.append(c)
        ranks.append((cur, rs, cl))
    return sim, nat, ranks


def zero_program(sim: Sim, nat: FakeNative, cur, rs, clusters, steps: int, barrier=True,
                 order_rng=None):
    """Per step: the units' backward (last unit first, or a per-rank random order with
    `order_rng`), each followed by its reduce-scatter (``_reduce_symm``, the real method), then
    ``wait_comm`` and the ``post_step`` barrier."""
    r = sim.rank
    for _step in range(steps):
        order = list(reversed(clusters))
        if order_rng is not None:
            order_rng.shuffle(order)
        for c in order:
            # the backward writes this rank's unsharded gradient buffer of the unit
            sim.put(sim.write_slot((r, "grad", c.grad_offset >> 20), c._rs_epoch + 1, r))
            nat.zero_epoch = lambda c=c: c._rs_epoch
            c._reduce_symm(object(), accumulate=False)
        cur.wait_stream(rs)          # wait_comm
        if barrier:
            sim.barrier()            # post_step: one all-reduce on the compute stream


def run_zero(monkeypatch, world, seed, units=3, steps=3, early=False, control=None,
             shuffled=False):
    sim, nat, ranks = build_zero(monkeypatch, world, units, early)
    if control == "no_flag_wait":
        from femtotron_b200.sharding.param_group_cluster import RS_WAIT_CODE
        nat.skip_wait_codes.add(RS_WAIT_CODE)
    for r, (cur, rs, cl) in enumerate(ranks):
        sim.rank = r
        zero_program(sim, nat, cur, rs, cl, steps, barrier=control != "no_barrier",
                     order_rng=random.Random(seed * 97 + r) if shuffled else None)
    sim.run(random.Random(seed))
    for (cur, rs, cl) in ranks:
        assert all(c._rs_epoch == steps for c in cl)
    return sim


@pytest.mark.parametrize("early", [False, True])
@pytest.mark.parametrize("world,seeds", [(2, 60), (4, 40), (8, 15)])
def test_zero3_reduce_scatter_protocol_is_race_and_deadlock_free(monkeypatch, world, seeds, early):
    for seed in range(seeds):
        run_zero(monkeypatch, world, seed, early=early)
        monkeypatch.undo()


def test_zero3_reduce_scatter_does_not_depend_on_a_common_unit_order(monkeypatch):
    """Every unit has its own flags and epochs, and the flags are published from the compute
    stream, which never waits for the reduce stream before the step's end: ranks whose
    gradient-ready callbacks fire in different orders still finish."""
    for seed in range(40):
        run_zero(monkeypatch, 4, seed, units=5, shuffled=True)
        monkeypatch.undo()


@pytest.mark.parametrize("control", ["no_flag_wait", "no_barrier"])
def test_zero3_checker_catches_a_missing_ordering(monkeypatch, control):
    found = None
    for seed in range(80):
        try:
            run_zero(monkeypatch, 4, seed, control=control)
        except Violation as e:
            found = e
            break
        finally:
            monkeypatch.undo()
    assert found is not None, f"{control}: no interleaving showed the missing ordering"


@pytest.mark.parametrize("mode", ["ce", "sm"])
def test_tp_back_to_back_all_gathers_reuse_slots_safely(monkeypatch, mode):
    for seed in range(30):
        run_tp(monkeypatch, 4, mode, seed, layers=3, program=back_to_back_program)
        monkeypatch.undo()
    found = None
    for seed in range(60):
        try:
            run_tp(monkeypatch, 4, mode, seed, layers=3, control="no_done_wait",
                   program=back_to_back_program)
        except Violation as e:
            found = e
            break
        finally:
            monkeypatch.undo()
    assert found is not None, "no interleaving showed the missing DONE ordering"
    assert "overwrote" in str(found) or "holding" in str(found), found


# =============================================================== NVLS all-reduce
class FakeTensor:
    """A user tensor handed to the NVLS all-reduce: copying into it reads this rank's copy of
    the multicast buffer (every slice must hold the round's reduced result)."""
    dtype = torch.float32

    def __init__(self, sim, ar, numel):
        self.sim, self.ar, self._n = sim, ar, numel

    def is_contiguous(self):
        return True

    def numel(self):
        return self._n

    def element_size(self):
        return 4

    def reshape(self, *shape):
        return self

    def view(self, *shape):
        return self

    def copy_(self, src):
        sim, ar, me = self.sim, self.ar, self.sim.rank
        k = ar.epoch // 2          # after the round's two barriers

        def run():
            for j in range(sim.world):
                sim.read_slot((me, "copy", j), ("out", k), me)
        sim.put(Op(f"copy out round {k}", run))
        return self


class FakeBuf:
    """This rank's copy of the multicast buffer: writing into it stages the round's input."""

    def __init__(self, sim, ar):
        self.sim, self.ar = sim, ar

    def __getitem__(self, idx):
        return self

    def view(self, dtype):
        return self

    def copy_(self, src):
        sim, ar, me = self.sim, self.ar, self.sim.rank
        k = ar.epoch // 2 + 1      # before the round's first barrier
        for j in range(sim.world):
            # the old input of slice j must have been reduced by rank j, an old result read
            # back by this rank
            sim.put(sim.write_slot((me, "copy", j), ("in", k), me,
                                   needed=lambda old, j=j: {j} if old[0] == "in" else {me}))
        return self


def build_nvls(monkeypatch, world: int, control=None):
    from femtotron_b200.parallel import nvls
    sim = Sim(world)
    nat = FakeNative(sim)
    patch_device(monkeypatch, sim, nat)
    monkeypatch.setattr(nvls, "native", lambda: nat)
    monkeypatch.setattr(nvls, "error_flag", lambda dev: None)
    ars = []
    for r in range(world):
        sim.rank = r
        sim.cur[r] = sim.new_stream()
        ar = object.__new__(nvls.NVLSAllReduce)
        ar.__dict__.update(group=None, rank=r, world=world, device=torch.device("cpu"),
                           size=1 << 20, data_bytes=(1 << 20) - 4096, flag_off=(1 << 20) - 4096,
                           uc=addr(r, 0), mc=0, epoch=0, closed=False)
        ar.buf = FakeBuf(sim, ar)
        ars.append(ar)
    skipped = {"no_first_barrier": 1, "no_second_barrier": 0}.get(control)

    def nvls_barrier(uc, mc, flag_off, target, err, code, timeout_ms):
        me = sim.rank
        ar = ars[me]

        def arrive():                   # multimem.red.add of 1 into every rank's counter
            for a in range(world):
                sim.flags[("ctr", a)] += 1
        sim.put(Op(f"barrier arrive {target}", arrive))
        if skipped is not None and ar.epoch % 2 == skipped:
            return                      # negative control: arrive without waiting
        sim.put(Op(f"barrier wait {target}", ready=lambda: sim.flags[("ctr", me)] >= target))

    def nvls_reduce_slice(mc, nbytes, rank, world_, f32, scale):
        k = (ars[rank].epoch + 1) // 2

        def run():                      # multimem.ld_reduce of slice `rank`, multimem.st back
            for a in range(world):
                sim.read_slot((a, "copy", rank), ("in", k), rank)
            for a in range(world):
                sim.write_slot((a, "copy", rank), ("out", k), rank,
                               needed=lambda old: {rank}).run()
        sim.put(Op(f"reduce slice {rank} round {k}", run))
    nat.nvls_barrier = nvls_barrier
    nat.nvls_reduce_slice = nvls_reduce_slice
    return sim, ars


def run_nvls(monkeypatch, world, seed, rounds=6, control=None):
    sim, ars = build_nvls(monkeypatch, world, control)
    kinds = random.Random(1000 + seed).choices(["one", "many"], k=rounds)  # same on every rank
    for r, ar in enumerate(ars):
        sim.rank = r
        for kind in kinds:
            if kind == "one":
                ar.all_reduce_(FakeTensor(sim, ar, 1024))
            else:
                ar.all_reduce_many_([FakeTensor(sim, ar, 256), FakeTensor(sim, ar, 512)],
                                    average=True)
    sim.run(random.Random(seed))
    assert all(ar.epoch == 2 * rounds for ar in ars)
    return sim


@pytest.mark.parametrize("world,seeds", [(2, 60), (4, 40), (8, 15)])
def test_nvls_all_reduce_protocol_is_race_and_deadlock_free(monkeypatch, world, seeds):
    for seed in range(seeds):
        run_nvls(monkeypatch, world, seed)
        monkeypatch.undo()


@pytest.mark.parametrize("control", ["no_first_barrier", "no_second_barrier"])
def test_nvls_checker_catches_a_missing_barrier(monkeypatch, control):
    found = None
    for seed in range(80):
        try:
            run_nvls(monkeypatch, 4, seed, control=control)
        except Violation as e:
            found = e
            break
        finally:
            monkeypatch.undo()
    assert found is not None, f"{control}: no interleaving showed the missing barrier"
