"""Pure unit tests (no process group): pipeline actions/schedules/partition/micro-batches,
ZeRO-3 cluster layout, sampler, LR schedule, parameter groups, activation checkpointing."""
import pytest
import torch
from torch import nn

from femtotron_b200.parallel.pipeline_parallel import (Backward, Forward, RecvBackward, RecvForward,
                                                       SendBackward, SendBackwardRecvForward,
                                                       SendForward, SendForwardRecvBackward,
                                                       gpipe_schedule, one_f_one_b_schedule,
                                                       partition_layers, split_microbatches)
from femtotron_b200.sharding import compute_cluster_layout


# ------------------------------------------------------------------ actions / schedules
def test_actions_are_frozen_hashable_and_compact():
    a = SendForwardRecvBackward(1, 0)
    assert repr(a) == "SFRB(1,0)" and repr(Forward(3)) == "F(3)" and repr(SendBackwardRecvForward(0, 2)) == "SBRF(0,2)"
    assert Forward(1) == Forward(1) and hash(Forward(1)) == hash(Forward(1))
    with pytest.raises(Exception):
        Forward(1).mb_id = 2


def test_gpipe_lists():
    assert repr(gpipe_schedule(2, True, True)) == "[F(0), F(1), B(1), B(0)]"
    assert repr(gpipe_schedule(2, True, False)) == "[F(0), SF(0), F(1), SF(1), RB(1), B(1), RB(0), B(0)]"
    assert repr(gpipe_schedule(2, False, True)) == "[RF(0), F(0), RF(1), F(1), B(1), SB(1), B(0), SB(0)]"


def test_1f1b_two_stage_lists():
    assert repr(one_f_one_b_schedule(3, 2, 0)) == \
        "[F(0), SF(0), F(1), SFRB(1,0), B(0), F(2), SFRB(2,1), B(1), RB(2), B(2)]"
    assert repr(one_f_one_b_schedule(3, 2, 1)) == \
        "[RF(0), F(0), B(0), SBRF(0,1), F(1), B(1), SBRF(1,2), F(2), B(2), SB(2)]"
    assert repr(one_f_one_b_schedule(2, 1, 0)) == "[F(0), B(0), F(1), B(1)]"


@pytest.mark.parametrize("P", [1, 2, 3, 4])
@pytest.mark.parametrize("N", [1, 2, 3, 4, 8])
def test_1f1b_invariants(P, N):
    for r in range(P):
        acts = one_f_one_b_schedule(N, P, r)
        f = [a.mb_id for a in acts if isinstance(a, Forward)]
        b = [a.mb_id for a in acts if isinstance(a, Backward)]
        assert sorted(f) == list(range(N)) and sorted(b) == list(range(N))
        for m in range(N):
            assert acts.index(Forward(m)) < acts.index(Backward(m))
        # in-flight forwards never exceed the warm-up depth + 1
        live = peak = 0
        for a in acts:
            live += isinstance(a, Forward) - isinstance(a, Backward)
            peak = max(peak, live)
        assert peak <= min(P - r, N)
        if r == 0:
            assert not any(isinstance(a, (RecvForward, SendBackward, SendBackwardRecvForward)) for a in acts)
        if r == P - 1:
            assert not any(isinstance(a, (SendForward, RecvBackward, SendForwardRecvBackward)) for a in acts)


def test_schedule_argument_validation():
    with pytest.raises(ValueError):
        one_f_one_b_schedule(0, 2, 0)
    with pytest.raises(ValueError):
        one_f_one_b_schedule(2, 2, 2)
    with pytest.raises(ValueError):
        gpipe_schedule(0, True, True)


def test_partition_layers():
    assert partition_layers(10, 4) == [range(0, 3), range(3, 6), range(6, 8), range(8, 10)]
    assert partition_layers(8, 2, "manual", layer_counts=[5, 3]) == [range(0, 5), range(5, 8)]
    with pytest.raises(ValueError):
        partition_layers(2, 3)
    with pytest.raises(ValueError):
        partition_layers(8, 2, "manual", layer_counts=[4, 3])
    with pytest.raises(NotImplementedError):
        partition_layers(8, 2, "balanced")


def test_split_microbatches_views():
    x = torch.arange(24).view(6, 4)
    parts = split_microbatches(x, 3)
    assert len(parts) == 3 and parts[1].data_ptr() == x[2:4].data_ptr()
    with pytest.raises(ValueError):
        split_microbatches(x, 4)


# ------------------------------------------------------------------ ZeRO-3 layout
def test_cluster_layout_cross_boundary():
    numels = [10, 7, 5]
    shapes = [torch.Size([10]), torch.Size([7]), torch.Size([5])]
    dts = [torch.bfloat16] * 3
    lay0, shard, pad = compute_cluster_layout(numels, shapes, dts, 0, 4)
    assert shard == 6 and pad == 2
    assert lay0[0].has_local_view and lay0[0].local_numel == 6 and not lay0[1].has_local_view
    lay1, _, _ = compute_cluster_layout(numels, shapes, dts, 1, 4)
    assert lay1[0].local_offset == 0 and lay1[0].local_numel == 4
    assert lay1[1].local_offset == 4 and lay1[1].local_numel == 2 and lay1[1].is_partially_local
    lay3, _, _ = compute_cluster_layout(numels, shapes, dts, 3, 4)
    assert lay3[2].local_numel == 4 and lay3[2].global_offset == 17
    total = sum(l.local_numel for r in range(4) for l in compute_cluster_layout(numels, shapes, dts, r, 4)[0])
    assert total == sum(numels)


# ------------------------------------------------------------------ sampler / LR / groups
class _Ctx:
    def __init__(self, r, n):
        self.dp_rank, self.dp_size = r, n


def test_sampler_shards_and_resumes():
    from femtotron_b200.data import DistributedSampler
    s0, s1 = DistributedSampler(10, _Ctx(0, 2), seed=1), DistributedSampler(10, _Ctx(1, 2), seed=1)
    a, b = list(s0), list(s1)
    assert len(a) == len(b) == 5 and not set(a) & set(b)
    s0.advance(2)
    st = s0.state_dict()
    s2 = DistributedSampler(10, _Ctx(0, 2), seed=1)
    s2.load_state_dict(st)
    assert list(s2) == a[2:]
    s2.set_epoch(1)
    assert list(s2) != a


def test_lr_schedule_shape():
    from femtotron_b200.training import create_lr_schedule
    p = nn.Parameter(torch.zeros(1))
    opt = torch.optim.SGD([p], lr=1.0)
    sch = create_lr_schedule(opt, warmup_steps=4, total_steps=10, min_lr_ratio=0.1)
    lrs = []
    for _ in range(12):
        lrs.append(opt.param_groups[0]["lr"])
        opt.step()
        sch.step()
    assert lrs[0] == pytest.approx(0.25) and lrs[3] == pytest.approx(1.0)
    assert lrs[-1] == pytest.approx(0.1) and all(a >= b for a, b in zip(lrs[3:], lrs[4:]))


def test_param_groups_decay_rule():
    from femtotron_b200.training import get_param_groups
    m = nn.ModuleDict({"embed_tokens": nn.Embedding(4, 4), "lin": nn.Linear(4, 4), "norm": nn.LayerNorm(4)})
    g = get_param_groups(m, 0.1)
    decay = {id(p) for p in g[0]["params"]}
    assert id(m["lin"].weight) in decay and id(m["lin"].bias) not in decay
    assert id(m["embed_tokens"].weight) not in decay and id(m["norm"].weight) not in decay


# ------------------------------------------------------------------ activation checkpointing
def test_activation_checkpointing_wraps_and_keeps_names():
    from femtotron_b200.training import (apply_activation_checkpointing, is_activation_checkpointed,
                                         remove_activation_checkpointing)
    from femtotron_b200.training.ckpt_policy import all_of, any_of, by_class, by_class_name, not_of
    m = nn.Sequential(nn.Linear(4, 4), nn.ReLU(), nn.Sequential(nn.Linear(4, 4)))
    names = set(m.state_dict().keys())
    x = torch.randn(3, 4, requires_grad=True)
    ref = m(x).sum()
    ref.backward()
    g_ref = m[0].weight.grad.clone()
    m.zero_grad()
    n = apply_activation_checkpointing(m, by_class(nn.Linear))
    assert n == 2 and is_activation_checkpointed(m[0]) and is_activation_checkpointed(m[2][0])
    assert set(m.state_dict().keys()) == names
    m(x).sum().backward()
    assert torch.allclose(m[0].inner_module.weight.grad, g_ref)
    m.load_state_dict({k: v for k, v in m.state_dict().items()})
    assert remove_activation_checkpointing(m) == 2 and not is_activation_checkpointed(m[0])
    p = any_of(by_class_name("ReLU"), not_of(by_class(nn.Module)))
    assert p(nn.ReLU()) and not p(nn.Linear(1, 1))
    assert all_of(by_class(nn.Linear), by_class_name("Linear"))(nn.Linear(1, 1))


def test_policy_from_config():
    from femtotron_b200.training.ckpt_config import policy_from_config
    pol = policy_from_config({"type": "any_of", "policies": [{"type": "class_name", "names": ["ReLU"]},
                                                             {"type": "never"}]})
    assert pol(nn.ReLU()) and not pol(nn.Linear(1, 1))
    with pytest.raises(ValueError):
        policy_from_config({"type": "bogus"})


def test_nvtx_helpers_are_noops_when_disabled():
    from femtotron_b200.utils import tracing
    from femtotron_b200.utils.comm_timing import TIMER
    with tracing.nvtx_range("x"):
        pass
    tracing.PHASES.switch("phase:a")
    tracing.PHASES.switch(None)
    with TIMER.wait("k"):
        pass
    TIMER.mark("fwd")
    TIMER.mark(None)


def test_saved_tensor_log_diff_and_activation_checkpointing():
    import torch
    from common_models import tiny_config
    from femtotron_b200.models import LlamaForTraining, materialize_model
    from femtotron_b200.models.layers import LlamaDecoderLayer
    from femtotron_b200.training import apply_activation_checkpointing
    from femtotron_b200.training.ckpt_policy import by_class
    from femtotron_b200.utils.saved_tensors import SavedTensorLog, diff_saved, format_diff
    cfg = tiny_config()
    with torch.device("meta"):
        m = LlamaForTraining(cfg)
    materialize_model(m, "cpu", dtype=torch.float32, init_std=0.02)
    ids = torch.randint(0, cfg.vocab_size, (2, 32), generator=torch.Generator().manual_seed(0))
    logs = []
    for name in ("first", "second"):   # same call site: locations compare equal
        with SavedTensorLog(name) as log:
            m(ids, labels=ids)["loss"]
        logs.append(log)
    a, b = logs
    assert len(a.entries) > 0 and format_diff(diff_saved(a, b)) == "saved tensors agree"
    apply_activation_checkpointing(m, by_class(LlamaDecoderLayer), use_reentrant=False)
    with SavedTensorLog("ac") as c:
        m(ids, labels=ids)["loss"].backward()
    d = diff_saved(a, c)
    assert d["only_a"] and c.saved_bytes < a.saved_bytes, (a.summary(), c.summary())
    assert "only in a:" in format_diff(d)


def test_schedules_equal_the_reference_action_lists(ref_root):
    """The pipeline schedules are pure data: for every (P, rank, N) they must produce the same
    action sequence (compared by compact repr, e.g. F(0), SFRB(1,0)) as the reference's
    gpipe_schedule / one_f_one_b_schedule ."""
    import os
    import sys
    import pytest
    root = ref_root
    sys.path.insert(0, root)
    try:
        from femtotron.parallel.pipeline_parallel import schedule as R
    finally:
        sys.path.remove(root)
    from femtotron_b200.parallel.pipeline_parallel import schedule as O
    for P in range(1, 5):
        for rank in range(P):
            for N in range(1, 9):
                mine = [repr(a) for a in O.one_f_one_b_schedule(N, P, rank)]
                theirs = [repr(a) for a in R.one_f_one_b_schedule(N, P, rank)]
                assert mine == theirs, (P, rank, N, mine, theirs)
                first, last = rank == 0, rank == P - 1
                assert [repr(a) for a in O.gpipe_schedule(N, first, last)] == \
                    [repr(a) for a in R.gpipe_schedule(N, first, last)], (P, rank, N)


def test_cluster_layout_equals_the_reference(ref_root):
    """compute_cluster_layout keeps the reference's flat, padded-to-dp layout (so ZeRO-3
    shards and checkpoints line up): every field of every parameter's spec, the shard size and
    the padding agree for assorted parameter lists and DP sizes."""
    import os
    import random
    import sys
    import pytest
    import torch
    root = ref_root
    sys.path.insert(0, root)
    try:
        from femtotron.sharding.cluster_sharding_spec import compute_cluster_layout as ref_layout
    finally:
        sys.path.remove(root)
    from femtotron_b200.sharding.cluster_sharding_spec import compute_cluster_layout
    rng = random.Random(0)
    fields = ("global_offset", "numel", "original_shape", "original_dtype", "has_local_view",
              "local_offset", "local_numel")
    for trial in range(40):
        shapes = [torch.Size([rng.randint(1, 40)] + ([rng.randint(1, 9)] if rng.random() < 0.6 else []))
                  for _ in range(rng.randint(1, 7))]
        numels = [s.numel() for s in shapes]
        dtypes = [torch.float32] * len(shapes)
        dp = rng.randint(1, 8)
        for rank in range(dp):
            a = compute_cluster_layout(numels, shapes, dtypes, rank, dp)
            b = ref_layout(numels, shapes, dtypes, rank, dp)
            assert a[1:] == tuple(b[1:]), (trial, rank, a[1:], b[1:])
            for x, y in zip(a[0], b[0]):
                assert all(getattr(x, f) == getattr(y, f) for f in fields), (trial, rank, x, y)


def test_lr_schedule_and_param_groups_equal_the_reference(ref_root):
    """The LR multiplier (linear warm-up with the reference's current_step+1 shift, cosine to
    min_lr_ratio) and the weight-decay grouping equal the reference's for the same inputs
    ."""
    import os
    import sys
    import pytest
    import torch
    from common_models import tiny_config
    root = ref_root
    sys.path.insert(0, root)
    try:
        from femtotron.training.lr_schedule import create_lr_schedule as ref_lr
        from femtotron.training.optimizer import get_param_groups as ref_groups
    finally:
        sys.path.remove(root)
    from femtotron_b200.models import LlamaForTraining, materialize_model
    from femtotron_b200.training import create_lr_schedule, get_param_groups
    for warm, total, mn in ((0, 10, 0.1), (3, 20, 0.0), (10, 10, 0.5), (5, 100, 0.1)):
        curves = []
        for make in (create_lr_schedule, ref_lr):
            opt = torch.optim.SGD([torch.nn.Parameter(torch.zeros(1))], lr=1.0)
            sch = make(opt, warm, total, mn)
            lrs = []
            for _ in range(total + 3):
                lrs.append(opt.param_groups[0]["lr"])
                opt.step()
                sch.step()
            curves.append(lrs)
        assert curves[0] == pytest.approx(curves[1], abs=1e-12), (warm, total, mn)
    with torch.device("meta"):
        m = LlamaForTraining(tiny_config())
    materialize_model(m, "cpu", dtype=torch.float32, init_std=0.02)
    names = {id(p): n for n, p in m.named_parameters()}
    for a, b in zip(get_param_groups(m, 0.03), ref_groups(m, 0.03)):
        assert a["weight_decay"] == b["weight_decay"]
        assert [names[id(p)] for p in a["params"]] == [names[id(p)] for p in b["params"]]


def test_reference_import_paths_and_public_names_exist(ref_root):
    """Every module of the reference package has a same-path module here
    (femtotron.X.Y -> femtotron_b200.X.Y), and every public top-level class and function of the
    reference module exists in it, so code written against the reference's imports resolves.
    The reference's names are read from its source (no import)."""
    import ast
    import importlib
    import os
    root = ref_root
    pkg = os.path.join(root, "femtotron")
    missing = []
    for dirpath, _, files in os.walk(pkg):
        if f"{os.sep}test" in dirpath[len(pkg):]:
            continue
        for fn in files:
            if not fn.endswith(".py"):
                continue
            rel = os.path.relpath(os.path.join(dirpath, fn), root)[:-3].replace(os.sep, ".")
            rel = rel[:-len(".__init__")] if rel.endswith(".__init__") else rel
            with open(os.path.join(dirpath, fn)) as f:
                tree = ast.parse(f.read())
            names = [n.name for n in tree.body if isinstance(n, (ast.FunctionDef, ast.ClassDef))
                     and not n.name.startswith("_")]
            try:
                ours = importlib.import_module("femtotron_b200" + rel[len("femtotron"):])
            except ImportError:
                missing.append(rel)
                continue
            missing += [f"{rel}.{n}" for n in names if not hasattr(ours, n)]
    assert not missing, missing


def test_preprocess_local_jsonl_with_byte_tokenizer(tmp_path):
    """Offline preprocessing: a local .jsonl corpus, the byte tokenizer (UTF-8 bytes, EOS 256),
    documents packed into full rows each followed by EOS; PackedDataset reads the result."""
    import json
    import torch
    from femtotron_b200.data import PackedDataset
    from femtotron_b200.data.preprocess import BYTES_EOS, pack_tokens, preprocess
    docs = ["hello world", "packed rows of tokens", "é ✓"]
    src = tmp_path / "corpus.jsonl"
    src.write_text("\n".join(json.dumps({"text": d}) for d in docs) + "\n")
    out = tmp_path / "packed" / "data.pt"
    data = preprocess(str(src), "bytes", str(out), seq_len=8)
    stream = []
    for d in docs:
        stream += list(d.encode("utf-8")) + [BYTES_EOS]
    n = len(stream) // 8
    assert data.shape == (n, 8) and data.dtype == torch.int32
    assert data.reshape(-1).tolist() == stream[:n * 8]
    ds = PackedDataset(str(out))
    assert len(ds) == n and ds.seq_len == 8
    assert pack_tokens([[1, 2], [3]], eos=0, seq_len=3).tolist() == [[1, 2, 0]]


def test_sampler_data_order_equals_the_reference(ref_root):
    """Data order is an interface: for the same seed, epoch and DP layout the sampler yields
    the reference sampler's index sequence, including after a resume offset."""
    import os
    import sys
    from types import SimpleNamespace
    import pytest
    root = ref_root
    sys.path.insert(0, root)
    try:
        from femtotron.data.distributed_sampler import DistributedSampler as Ref
    finally:
        sys.path.remove(root)
    from femtotron_b200.data import DistributedSampler
    for size in (7, 64, 101):
        for dp in (1, 2, 3, 8):
            for shuffle in (True, False):
                for drop_last in (True, False):
                    for r in range(dp):
                        ctx = SimpleNamespace(dp_rank=r, dp_size=dp)
                        a = DistributedSampler(size, ctx, seed=5, shuffle=shuffle, drop_last=drop_last)
                        b = Ref(size, ctx, seed=5, shuffle=shuffle, drop_last=drop_last)
                        for epoch in (0, 3):
                            a.set_epoch(epoch)
                            b.set_epoch(epoch)
                            assert list(a) == list(b) and len(a) == len(b), (size, dp, r, epoch)
                        if len(a) > 2:
                            a.advance(2)
                            b.advance(2)
                            assert list(a) == list(b), (size, dp, r, "resume")


def test_parallel_context_groups_match_coordinate_enumeration():
    """Every group of every dimension holds exactly the ranks whose row-major coordinates
    differ from this rank's only along that dimension, in coordinate order (tp innermost);
    prev/next ranks are the neighbours in that order."""
    from collections import OrderedDict
    from femtotron_b200.parallel_context import SUPPORTED_PARALLEL_DIMS, ParallelContext
    for dims in [dict(pp=2, dp=2, tp=2), dict(dp=4), dict(pp=3, dp=2, tp=4), dict(tp=8),
                 dict(pp=2, cp=2, tp=2), dict(pp=2, dp=3)]:
        sizes = [dims.get(n, 1) for n in SUPPORTED_PARALLEL_DIMS]
        world = 1
        for s in sizes:
            world *= s
        for rank in range(world):
            ctx = ParallelContext(OrderedDict(dims), world_size=world, world_rank=rank)
            coord, r = [], rank
            for s in reversed(sizes):
                coord.append(r % s)
                r //= s
            coord.reverse()
            assert ctx.local_coord == coord
            for d, name in enumerate(SUPPORTED_PARALLEL_DIMS):
                want = []
                for pos in range(sizes[d]):
                    c = list(coord)
                    c[d] = pos
                    idx = 0
                    for s, x in zip(sizes, c):
                        idx = idx * s + x
                    want.append(idx)
                assert ctx.get_ranks_in_group(name) == want
                assert ctx.get_rank(name) == coord[d]
                i = want.index(rank)
                assert ctx.get_prev_rank_in(name) == (want[i - 1] if i > 0 else None)
                assert ctx.get_next_rank_in(name) == (want[i + 1] if i + 1 < len(want) else None)


def test_fused_adamw_flat_moments_survive_a_checkpoint_round_trip():
    """The moments of parameters updated by the fused reduce-scatter + AdamW live in one flat
    buffer per ZeRO unit; a saved and reloaded optimizer state lands back in those buffers."""
    import io
    import torch
    from femtotron_b200.training.optimizer import FusedAdamW
    torch.manual_seed(0)
    p1, p2 = torch.nn.Parameter(torch.randn(10)), torch.nn.Parameter(torch.randn(6))
    opt = FusedAdamW([p1, p2], lr=1e-2)
    m, v = torch.zeros(16), torch.zeros(16)
    opt.bind_state(p1, m[:10], v[:10])
    opt.bind_state(p2, m[10:], v[10:])
    for _ in range(3):
        p1.grad, p2.grad = torch.randn(10), torch.randn(6)
        opt.step()
    buf = io.BytesIO()
    torch.save(opt.state_dict(), buf)
    buf.seek(0)
    q1, q2 = torch.nn.Parameter(p1.detach().clone()), torch.nn.Parameter(p2.detach().clone())
    opt2 = FusedAdamW([q1, q2], lr=1e-2)
    m2, v2 = torch.zeros(16), torch.zeros(16)
    opt2.bind_state(q1, m2[:10], v2[:10])
    opt2.bind_state(q2, m2[10:], v2[10:])
    opt2.load_state_dict(torch.load(buf))
    assert torch.equal(m2, m) and torch.equal(v2, v)
    assert opt2.state[q1]["exp_avg"].data_ptr() == m2.data_ptr()
    assert float(opt2.state[q2]["step"]) == 3.0
    # an early (fused) update advances the step and is skipped by the next step()
    assert opt2.mark_updated([q1, q2]) == 4
    before = q1.detach().clone()
    q1.grad, q2.grad = torch.randn(10), torch.randn(6)
    opt2.step()
    assert torch.equal(q1.detach(), before) and float(opt2.state[q1]["step"]) == 4.0
