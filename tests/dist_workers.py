"""Bodies of the multi-rank CPU (gloo) tests; module-level so spawned ranks can import them."""
from __future__ import annotations

import os
from collections import OrderedDict

import torch
import torch.distributed as dist
from torch import nn

from common_models import full_state, hf_init, load_sharded, tiny_config


def ctx_of(**dims):
    from femtotron_b200.parallel_context import ParallelContext
    return ParallelContext(OrderedDict(dims))


# ----------------------------------------------------------------------------- topology
def w_parallel_context(rank, world):
    c = ctx_of(pp=2, dp=1, tp=2)
    out = {"coord": c.local_coord, "tp": c.get_ranks_in_group("tp"), "pp": c.get_ranks_in_group("pp"),
           "prev": c.pp_prev_rank, "next": c.pp_next_rank, "tp_rank": c.tp_rank, "pp_rank": c.pp_rank}
    c2 = ctx_of(dp=2, tp=2)
    out["dp_ranks"] = c2.get_ranks_in_group("dp")
    t = torch.ones(1) * rank
    dist.all_reduce(t, group=c2.tp_group)
    out["tp_sum"] = t.item()
    return out


# ----------------------------------------------------------------------------- TP layers
def w_tp_layers(rank, world, sequence_parallel):
    from femtotron_b200.parallel.tensor_parallel import (ColumnParallelLinear, RowParallelLinear,
                                                         VocabParallelEmbedding)
    c = ctx_of(tp=world)
    torch.manual_seed(0)
    T, H, F = 16, 32, 48
    lin1, lin2 = nn.Linear(H, F, bias=False), nn.Linear(F, H, bias=False)
    emb = nn.Embedding(64, H)
    x = torch.randn(T, H)
    ids = torch.randint(0, 64, (T,))
    # reference
    xr = x.clone().requires_grad_(True)
    yr = lin2(torch.relu(lin1(xr) + emb(ids)[:, :1]))
    yr.pow(2).sum().backward()
    col = ColumnParallelLinear.from_linear_temp(lin1, c, sequence_parallel=sequence_parallel)
    row = RowParallelLinear.from_linear_temp(lin2, c, sequence_parallel=sequence_parallel)
    vemb = VocabParallelEmbedding.from_embedding_temp(emb, c)
    chunk = T // world
    if sequence_parallel:
        xl = x[rank * chunk:(rank + 1) * chunk].clone().requires_grad_(True)
    else:
        xl = x.clone().requires_grad_(True)
    h = col(xl)
    e = vemb(ids)[:, :1]
    y = row(torch.relu(h + e))
    y.pow(2).sum().backward() if sequence_parallel else (y.pow(2).sum()).backward()
    if sequence_parallel:
        ref_y = yr.detach()[rank * chunk:(rank + 1) * chunk]
        ref_dx = xr.grad[rank * chunk:(rank + 1) * chunk]
    else:
        ref_y, ref_dx = yr.detach(), xr.grad
    fo = F // world
    ok = {
        "y": torch.allclose(y.detach(), ref_y, atol=1e-5, rtol=1e-5),
        "dx": torch.allclose(xl.grad, ref_dx, atol=1e-5, rtol=1e-5),
        "dw1": torch.allclose(col.weight.grad, lin1.weight.grad[rank * fo:(rank + 1) * fo], atol=1e-5, rtol=1e-5),
        "dw2": torch.allclose(row.weight.grad, lin2.weight.grad[:, rank * fo:(rank + 1) * fo], atol=1e-5, rtol=1e-5),
    }
    return ok


# ----------------------------------------------------------------------------- TP model
def _single_model(cfg, sd):
    from femtotron_b200.models import LlamaForTraining, materialize_model
    with torch.device("meta"):
        m = LlamaForTraining(cfg)
    materialize_model(m, "cpu", dtype=torch.float32, init_std=None)
    m.load_state_dict(sd)
    return m


def w_tp_model(rank, world, sequence_parallel):
    from femtotron_b200.models import build_llama_model, materialize_model
    cfg = tiny_config()
    sd = full_state(cfg)
    c = ctx_of(tp=world)
    m = build_llama_model(cfg, c, sequence_parallel=sequence_parallel)
    materialize_model(m, "cpu", dtype=torch.float32, init_std=None)
    load_sharded(m, sd, c)
    torch.manual_seed(1)
    ids = torch.randint(0, cfg.vocab_size, (2, 32))
    loss = m(ids, labels=ids)["loss"]
    loss.backward()
    ref = _single_model(cfg, sd)
    lr = ref(ids, labels=ids)["loss"]
    lr.backward()
    from femtotron_b200.models.model_loader import shard_for_rank
    from femtotron_b200.models.parallel_plan import get_llama_parallel_plan
    plan = get_llama_parallel_plan()
    rp = dict(ref.named_parameters())
    worst = 0.0
    for n, p in m.named_parameters():
        g_ref = shard_for_rank(rp[n].grad, n, plan, c.tp_rank, c.tp_size)
        worst = max(worst, ((p.grad - g_ref).norm() / (g_ref.norm() + 1e-12)).item())
    return {"loss": loss.item(), "ref": lr.item(), "worst": worst}


# ----------------------------------------------------------------------------- ZeRO 0..3
def _inject_delays(model, seed, max_s=0.02):
    """Host-side random sleeps before every decoder layer's forward and backward on this
    rank: the ranks reach their collectives (ZeRO gathers / reduce-scatters) at shifted
    times, which shakes out ordering assumptions between ranks."""
    import random
    import time
    from femtotron_b200.models.layers import LlamaDecoderLayer
    rng = random.Random(seed)

    def nap(*_):
        time.sleep(rng.uniform(0.0, max_s))
    for mod in model.modules():
        if isinstance(mod, LlamaDecoderLayer):
            mod.register_forward_pre_hook(nap)
            mod.register_full_backward_pre_hook(nap)


def _build_trainer(cfg, sd, ctx, stage, steps, mb, ga, seed_data, lr=5e-3, clip=None, ckpt=None,
                   ac=False, delay_seed=None, check_finite=False, dtype=torch.float32):
    from femtotron_b200.data import DistributedDataLoader, SyntheticTokens, simple_pretrain_collator
    from femtotron_b200.models import build_llama_model, get_llama_parallel_plan, materialize_model
    from femtotron_b200.parallel.data_parallel import create_grad_synchronizer
    from femtotron_b200.sharding import ZeROConfig, create_sharding_strategy, llama_wrap_policy
    from femtotron_b200.training import (ClipGradNorm, FusedAdamW, MixedPrecisionManager, TrainConfig,
                                         Trainer, apply_activation_checkpointing, create_lr_schedule,
                                         get_param_groups)
    from femtotron_b200.training.ckpt_policy import by_class
    from femtotron_b200.models.layers import LlamaDecoderLayer
    m = build_llama_model(cfg, ctx)
    materialize_model(m, "cpu", dtype=dtype, init_std=None)
    load_sharded(m, sd, ctx)
    if delay_seed is not None:
        _inject_delays(m, delay_seed)
    tc = TrainConfig(train_steps=steps, grad_accum_steps=ga, master_dtype=torch.float32,
                     param_dtype=dtype, log_interval=10 ** 6,
                     checkpoint_interval=ckpt[1] if ckpt else 10 ** 6,
                     checkpoint_dir=ckpt[0] if ckpt else "ckpt", warmup_steps=1, min_lr_ratio=0.1)
    st = create_sharding_strategy(ctx, ZeROConfig(stage=stage, wrap_policy=llama_wrap_policy))
    transforms = [ClipGradNorm(clip, ctx, dp_sharded=st.grads_are_dp_sharded())] if clip else None
    mp = MixedPrecisionManager(m, ctx, get_llama_parallel_plan(), tc, FusedAdamW,
                               dict(lr=lr, betas=(0.9, 0.95), eps=1e-8), get_param_groups(m, 0.01),
                               grad_transforms=transforms, sharding_strategy=st)
    if ac:
        apply_activation_checkpointing(m, by_class(LlamaDecoderLayer))
    sch = create_lr_schedule(mp.inner, 1, steps)
    ds = SyntheticTokens(64, 32, cfg.vocab_size, seed=seed_data)
    dl = DistributedDataLoader(ds, ctx, mb, simple_pretrain_collator, num_workers=0, pin_memory=False)
    return Trainer(m, mp, sch, dl, create_grad_synchronizer(mp.groups, ctx, st), ctx, tc,
                   check_finite=check_finite)


def _train(cfg, sd, ctx, stage, steps, mb, ga, seed_data, lr=5e-3, clip=None, ckpt=None,
           resume=None, ac=False, delay_seed=None):
    tr = _build_trainer(cfg, sd, ctx, stage, steps, mb, ga, seed_data, lr=lr, clip=clip, ckpt=ckpt,
                        ac=ac, delay_seed=delay_seed)
    if resume:
        tr._load_checkpoint(resume)
    hist = tr.train()
    return [h["loss"] for h in hist]


def w_zero(rank, world, stage, ac):
    cfg = tiny_config()
    sd = full_state(cfg)
    ctx = ctx_of(dp=world)
    losses = _train(cfg, sd, ctx, stage, steps=4, mb=2, ga=2, seed_data=3, ac=ac)
    t = torch.tensor(losses)
    dist.all_reduce(t)
    return (t / world).tolist()


def w_zero_delayed(rank, world, stage):
    """Same run as w_zero with random host delays on rank 1 only."""
    cfg = tiny_config()
    sd = full_state(cfg)
    ctx = ctx_of(dp=world)
    losses = _train(cfg, sd, ctx, stage, steps=4, mb=2, ga=2, seed_data=3,
                    delay_seed=100 + rank if rank == 1 else None)
    t = torch.tensor(losses)
    dist.all_reduce(t)
    return (t / world).tolist()


def w_zero_clip(rank, world, stage):
    cfg = tiny_config()
    sd = full_state(cfg)
    ctx = ctx_of(dp=world)
    losses = _train(cfg, sd, ctx, stage, steps=4, mb=2, ga=1, seed_data=3, clip=0.05)
    t = torch.tensor(losses)
    dist.all_reduce(t)
    return (t / world).tolist()


def w_resume(rank, world, stage, tmpdir):
    cfg = tiny_config()
    sd = full_state(cfg)
    ctx = ctx_of(dp=world)
    full = _train(cfg, sd, ctx, stage, steps=4, mb=2, ga=1, seed_data=5, ckpt=(tmpdir, 2))
    part = _train(cfg, sd, ctx, stage, steps=4, mb=2, ga=1, seed_data=5,
                  resume=os.path.join(tmpdir, "step_2"))
    return {"full": full, "resumed": part}


# ----------------------------------------------------------------------------- pipeline
def w_pipeline(rank, world, schedule):
    from femtotron_b200.models import build_llama_model, materialize_model
    from femtotron_b200.parallel.pipeline_parallel import (PipelineComm, PipelineRunner, PipelineStage,
                                                           partition_layers)
    cfg = tiny_config(num_hidden_layers=4)
    sd = full_state(cfg)
    ctx = ctx_of(pp=world)
    rng = partition_layers(cfg.num_hidden_layers, world)[ctx.pp_rank]
    m = build_llama_model(cfg, ctx, use_pp_aware=True, layer_range=rng)
    materialize_model(m, "cpu", dtype=torch.float32, init_std=None)
    with torch.no_grad():
        for n, p in m.named_parameters():
            p.copy_(sd[n])
    nmb, mb, S = 4, 2, 16
    torch.manual_seed(7)
    ids = torch.randint(0, cfg.vocab_size, (nmb * mb, S))
    stage = PipelineStage(m, ctx, loss_scale=1.0 / nmb)
    comm = PipelineComm(ctx, S, cfg.hidden_size, torch.float32, device=torch.device("cpu"))
    runner = PipelineRunner(stage, comm, schedule_name=schedule, num_microbatches=nmb,
                            recv_shape=(mb, S, cfg.hidden_size), recv_dtype=torch.float32)
    losses = runner.run_step({"input_ids": ids, "labels": ids})
    # single-rank reference: mean of micro-batch losses
    ref = _single_model(cfg, sd)
    tot = 0.0
    for i in range(nmb):
        l = ref(ids[i * mb:(i + 1) * mb], labels=ids[i * mb:(i + 1) * mb])["loss"] / nmb
        l.backward()
        tot += l.item()
    rp = dict(ref.named_parameters())
    worst = max(((p.grad - rp[n].grad).norm() / (rp[n].grad.norm() + 1e-12)).item()
                for n, p in m.named_parameters())
    mine = sum(v.item() for v in losses.values()) if losses else None
    return {"loss": mine, "ref": tot, "worst": worst, "is_last": stage.is_last}


# ----------------------------------------------------------------------------- faults
def w_failure_modes(rank, world, tmpdir):
    """Host-side fault injection on gloo ranks:
    * an exception inside a ZeRO-3 unit's forward, recovered by force_reshard_all, after which
      training continues exactly as an undisturbed run;
    * a checkpoint without its _SUCCESS marker, and one whose shard file is truncated: both
      refuse to load;
    * a NaN in a parameter: the trainer's finite-loss check aborts the step on every rank."""
    from femtotron_b200.models.layers import LlamaDecoderLayer
    cfg = tiny_config()
    sd = full_state(cfg)
    ctx = ctx_of(dp=world)
    out = {}
    # -- exception inside a unit, then recovery
    clean = _build_trainer(cfg, sd, ctx, 3, steps=2, mb=2, ga=1, seed_data=9)
    clean.dataloader.set_epoch(0)
    ref = clean.train_step(iter(clean.dataloader))["loss"]
    tr = _build_trainer(cfg, sd, ctx, 3, steps=2, mb=2, ga=1, seed_data=9)
    layer = [m for m in tr.model.modules() if isinstance(m, LlamaDecoderLayer)][1]
    fired = []

    def boom(*_):
        if not fired:
            fired.append(1)
            raise RuntimeError("injected failure inside a ZeRO-3 unit")
    h = layer.register_forward_pre_hook(boom)
    tr.dataloader.set_epoch(0)
    try:
        tr.train_step(iter(tr.dataloader))
        out["raised"] = False
    except RuntimeError as e:
        out["raised"] = "injected" in str(e)
    h.remove()
    tr.mp_manager.strategy.force_reshard_all()
    out["all_resharded"] = all(c._full_buffer is None and c._prefetch is None
                               for c in tr.mp_manager.strategy.clusters)
    tr.dataloader.set_epoch(0)
    out["recovered_loss_matches"] = abs(tr.train_step(iter(tr.dataloader))["loss"] - ref) < 1e-6
    # -- incomplete checkpoints
    ck = os.path.join(tmpdir, "ck")
    tr.train_config.checkpoint_dir = ck
    tr.global_step = 1
    d = tr._save_checkpoint()
    dist.barrier()
    if rank == 0:
        os.remove(os.path.join(d, "_SUCCESS"))
    dist.barrier()
    try:
        tr._load_checkpoint(d)
        out["missing_success_refused"] = False
    except RuntimeError as e:
        out["missing_success_refused"] = "_SUCCESS" in str(e)
    dist.barrier()
    if rank == 0:
        with open(os.path.join(d, "_SUCCESS"), "w") as f:
            f.write("ok")
    shard = os.path.join(d, tr._shard_name())
    with open(shard, "r+b") as f:
        f.truncate(max(1, os.path.getsize(shard) // 2))
    dist.barrier()
    try:
        tr._load_checkpoint(d)
        out["truncated_refused"] = False
    except Exception:
        out["truncated_refused"] = True
    dist.barrier()
    # -- NaN abort
    nan_tr = _build_trainer(cfg, sd, ctx, 3, steps=2, mb=2, ga=1, seed_data=9, check_finite=True)
    with torch.no_grad():
        # under ZeRO-3 the embedding is sharded like every other parameter: its storage is
        # this rank's slice of its cluster, gathered at the next forward
        owner = [c for c in nan_tr.mp_manager.clusters
                 if any(pg.name.endswith("embed_tokens.weight") for pg in c.param_groups)]
        if owner:
            owner[0].flat_param_shard.fill_(float("nan"))
        else:
            nan_tr.model.model.embed_tokens.weight.fill_(float("nan"))
    nan_tr.dataloader.set_epoch(0)
    try:
        nan_tr.train_step(iter(nan_tr.dataloader))
        out["nan_aborted"] = False
    except FloatingPointError:
        out["nan_aborted"] = True
    return out


def w_rank_failure(rank, world):
    """Rank 1 dies between steps; rank 0's next collective must fail with an error (process
    group timeout), not hang."""
    import time
    ctx = ctx_of(dp=world)
    t = torch.ones(4)
    dist.all_reduce(t, group=ctx.dp_group)
    if rank == 1:
        return {"left": True}  # leaves between steps, nothing in flight
    t0 = time.time()
    try:
        dist.all_reduce(t, group=ctx.dp_group)
    except Exception as e:  # gloo raises on timeout / peer loss
        return {"raised": True, "elapsed": time.time() - t0, "msg": str(e)[:100]}
    return {"raised": False}


# ----------------------------------------------------------------------------- model loading
def w_model_loading(rank, world, tmpdir):
    """Reference test_model_loading: rank 0 writes an HF LlamaForCausalLM with save_pretrained
    (safetensors), every rank loads its TP slices with ModelLoader; the sharded model's loss and
    its weight-gradient slices must match the HF model's."""
    from transformers import LlamaForCausalLM
    from femtotron_b200.models import build_llama_model, materialize_model
    from femtotron_b200.models.model_loader import ModelLoader, shard_for_rank
    from femtotron_b200.models.parallel_plan import get_llama_parallel_plan
    cfg = tiny_config()
    torch.manual_seed(11)
    hf = LlamaForCausalLM(cfg).float()
    path = os.path.join(tmpdir, "hf")
    if rank == 0:
        hf.save_pretrained(path, safe_serialization=True)
    dist.barrier()
    ctx = ctx_of(tp=world)
    m = build_llama_model(cfg, ctx)
    materialize_model(m, "cpu", dtype=torch.float32, init_std=0.02)
    ModelLoader(ctx).load_and_distribute(m, path, device="cpu")
    ids = torch.randint(0, cfg.vocab_size, (2, 32), generator=torch.Generator().manual_seed(3))
    loss = m(input_ids=ids, labels=ids)["loss"]
    loss.backward()
    ref = hf(input_ids=ids, labels=ids).loss
    ref.backward()
    plan = get_llama_parallel_plan()
    hfp = dict(hf.named_parameters())
    worst_w = worst_g = 0.0
    for name, p in m.named_parameters():
        key = name.replace("._checkpoint_wrapped_module", "")
        w_ref = shard_for_rank(hfp[key].detach(), key, plan, ctx.tp_rank, ctx.tp_size)
        g_ref = shard_for_rank(hfp[key].grad, key, plan, ctx.tp_rank, ctx.tp_size)
        worst_w = max(worst_w, (p.detach() - w_ref).abs().max().item())
        g = p.main_grad if getattr(p, "main_grad", None) is not None else p.grad
        worst_g = max(worst_g, ((g - g_ref).norm() / (g_ref.norm() + 1e-12)).item())
    return {"loss": loss.item(), "ref": ref.item(), "worst_w": worst_w, "worst_g": worst_g}


# ----------------------------------------------------------------------------- DP x TP splits
def _global_batches(cfg, steps, gb, seq=32, seed=21):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, cfg.vocab_size, (gb, seq), generator=g) for _ in range(steps)]


def _run_split(cfg, sd, ctx, stage, steps, mb, ga, seed=21, ac=False):
    """Train `steps` optimizer steps where global step s consumes the fixed global batch G_s
    (dp x ga x mb rows): DP rank r, micro-batch k takes rows [(r*ga + k)*mb, ... + mb).
    Returns the loss curve averaged over all ranks (= the global-batch mean)."""
    gb = ctx.dp_size * ga * mb
    batches = _global_batches(cfg, steps, gb, seed=seed)
    tr = _build_trainer(cfg, sd, ctx, stage, steps=steps, mb=mb, ga=ga, seed_data=1, ac=ac)
    r = ctx.dp_rank
    losses = []
    for s in range(steps):
        def it(s=s):
            for k in range(ga):
                x = batches[s][(r * ga + k) * mb:(r * ga + k + 1) * mb]
                yield {"input_ids": x, "labels": x}
        losses.append(tr.train_step(it())["loss"])
    t = torch.tensor(losses, dtype=torch.float64)
    dist.all_reduce(t)
    return (t / dist.get_world_size()).tolist()


def w_dp_tp_split(rank, world, dp, tp, stage, ac=False):
    """Reference test_dp_training: the same global batches under every legal (DP, TP) split
    (optionally with ZeRO and activation checkpointing)."""
    cfg = tiny_config(num_key_value_heads=4)
    sd = full_state(cfg)
    return _run_split(cfg, sd, ctx_of(dp=dp, tp=tp), stage, steps=3, mb=8 // dp, ga=1, ac=ac)


def w_grad_accum(rank, world, mb, ga):
    """Reference test_gradient_accum: (micro-batch, accumulation) pairs with the same global
    batch give the same loss curve."""
    cfg = tiny_config()
    sd = full_state(cfg)
    return _run_split(cfg, sd, ctx_of(dp=world), 1, steps=3, mb=mb, ga=ga)


# ----------------------------------------------------------------------------- pipeline stage
def w_stage_errors(rank, world):
    """Reference test_pipeline_stage (error handling / state management) on a one-stage
    pipeline (first and last): out-of-order calls raise with the micro-batch id, leftover
    state is reported by assert_clean, reset recovers, and a full micro-batch matches a direct
    forward/backward of the model."""
    from femtotron_b200.models import build_llama_model, materialize_model
    from femtotron_b200.parallel.pipeline_parallel import PipelineStage
    cfg = tiny_config()
    ctx = ctx_of(pp=1)
    m = build_llama_model(cfg, ctx, use_pp_aware=True, layer_range=range(cfg.num_hidden_layers))
    materialize_model(m, "cpu", dtype=torch.float32, init_std=0.02)
    st = PipelineStage(m, ctx, loss_scale=0.5)
    ids = torch.randint(0, cfg.vocab_size, (2, 16), generator=torch.Generator().manual_seed(2))
    out = {}

    def raises(fn, text):
        try:
            fn()
        except RuntimeError as e:
            return text in str(e)
        return False
    out["forward_without_input"] = raises(lambda: st.forward(0), "forward(0): no input staged")
    out["backward_without_output"] = raises(lambda: st.backward(3), "backward(3): no output")
    st.stage_input(0, ids)
    out["double_input"] = raises(lambda: st.stage_input(0, ids), "input already staged")
    out["forward_without_labels"] = raises(lambda: st.forward(0), "last stage requires labels")
    st.stage_labels(0, ids)
    out["leftover_reported"] = raises(st.assert_clean, "leftover per-microbatch state")
    st.reset()
    st.assert_clean()
    out["reset_clean"] = True
    # one micro-batch through the stage == direct loss * loss_scale, same gradients
    st.stage_input(1, ids)
    st.stage_labels(1, ids)
    st.forward(1)
    out["double_forward"] = raises(lambda: st.forward(1), "output already exists")
    st.backward(1)
    loss = st.pop_all_losses()[1].item()
    st.assert_clean()

    def grad_of(p):
        return p.main_grad if getattr(p, "main_grad", None) is not None else p.grad
    g_stage = {n: grad_of(p).clone() for n, p in m.named_parameters()}
    for p in m.parameters():
        p.grad = None
        if getattr(p, "main_grad", None) is not None:
            p.main_grad.zero_()
    ref = m(ids, labels=ids)["loss"] * 0.5
    ref.backward()
    out["loss_matches"] = abs(loss - ref.item()) < 1e-6
    out["grads_match"] = all(torch.allclose(g_stage[n], grad_of(p), atol=1e-6, rtol=1e-5)
                             for n, p in m.named_parameters())
    return out


# ----------------------------------------------------------------------------- clipping
def w_clip_norm_vs_torch(rank, world, tp):
    """Reference test_mixed_precision (clipping): the global gradient norm that ClipGradNorm
    reports equals torch.nn.utils.clip_grad_norm_'s total norm of the same gradients, for
    DP-replicated (ZeRO-0), DP-sharded (ZeRO-1/2/3, including ZeRO-3's unsharded free
    parameters) and TP-sharded gradients."""
    cfg = tiny_config()
    sd = full_state(cfg)
    dp = world // tp
    x = _global_batches(cfg, 1, 4 * dp, seed=5)[0]
    out = {}
    for stage in (0, 1, 2, 3):
        ctx = ctx_of(dp=dp, tp=tp)
        tr = _build_trainer(cfg, sd, ctx, stage, steps=1, mb=4, ga=1, seed_data=1, clip=0.05)
        r = ctx.dp_rank
        mine = x[r * 4:(r + 1) * 4]
        info = tr.train_step(iter([{"input_ids": mine, "labels": mine}]))
        out[f"zero{stage}"] = info["grad_norm"]
    # reference: one process, the same batches (mean of the DP ranks' losses)
    ref = _single_model(cfg, sd)
    loss = sum(ref(x[r * 4:(r + 1) * 4], labels=x[r * 4:(r + 1) * 4])["loss"] for r in range(dp)) / dp
    loss.backward()
    out["torch"] = torch.nn.utils.clip_grad_norm_(list(ref.parameters()), max_norm=1e9).item()
    return out


# ----------------------------------------------------------------------------- reference parity
def _load_reference(ref_root):
    import sys
    if ref_root not in sys.path:
        sys.path.insert(0, ref_root)
    from femtotron.parallel_context import ParallelContext as RCtx
    from femtotron.model.llama import build_llama_model as rbuild
    return RCtx, rbuild


def w_reference_parity(rank, world, ref_root, steps):
    """BASELINE configuration 1 against the reference's own modules on the same gloo ranks:
    tiny LLaMA (4 layers, hidden 256, 8/4 heads, FFN 688, vocab 2048), TP=2, fp32, seq 128,
    micro-batch 4, uniform token ids from seed 0, identical initial weights, `steps` steps.  Both sides run
    forward + backward of their own model and an identical AdamW update of the full
    parameters, so the loss curves must agree."""
    from collections import OrderedDict
    from transformers import LlamaConfig
    from femtotron_b200.models import build_llama_model, materialize_model
    from femtotron_b200.models.model_loader import shard_for_rank
    from femtotron_b200.models.parallel_plan import get_llama_parallel_plan
    RCtx, rbuild = _load_reference(ref_root)
    cfg = LlamaConfig(hidden_size=256, intermediate_size=688, num_attention_heads=8,
                      num_key_value_heads=4, num_hidden_layers=4, vocab_size=2048,
                      max_position_embeddings=512, rms_norm_eps=1e-5, rope_theta=10000.0,
                      tie_word_embeddings=False, attn_implementation="sdpa")
    cfg.use_cache = False
    sd = full_state(cfg)
    plan = get_llama_parallel_plan()
    g = torch.Generator().manual_seed(0)
    batches = [torch.randint(0, 2048, (4, 128), generator=g) for _ in range(steps)]

    ctx = ctx_of(tp=world)
    ours = build_llama_model(cfg, ctx)
    materialize_model(ours, "cpu", dtype=torch.float32, init_std=None)
    load_sharded(ours, sd, ctx)

    rctx = RCtx(OrderedDict([("pp", 1), ("dp", 1), ("tp", world)]))
    ref = rbuild(cfg, rctx).to_empty(device="cpu")
    with torch.no_grad():
        for name, p in ref.named_parameters():
            p.copy_(shard_for_rank(sd[name], name, plan, rctx.tp_rank, rctx.tp_size))
        rot = ref.model.rotary_emb   # the reference's own tests recompute inv_freq after to_empty
        d = cfg.hidden_size // cfg.num_attention_heads
        theta = (getattr(cfg, "rope_parameters", None) or {}).get("rope_theta", 10000.0)
        inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
        rot.inv_freq.copy_(inv)
        if hasattr(rot, "original_inv_freq"):
            rot.original_inv_freq.copy_(inv)

    def run(model, grad_of):
        opt = torch.optim.AdamW(list(model.parameters()), lr=3e-4, betas=(0.9, 0.95), eps=1e-8,
                                weight_decay=0.0)
        losses = []
        for x in batches:
            opt.zero_grad(set_to_none=True)
            for p in model.parameters():
                if getattr(p, "main_grad", None) is not None:
                    p.main_grad.zero_()
            loss = model(x, labels=x)["loss"]
            loss.backward()
            for p in model.parameters():
                gr = grad_of(p)
                if gr is not p.grad:
                    p.grad = gr.clone()
            opt.step()
            losses.append(loss.item())
        return losses

    mine = run(ours, lambda p: p.main_grad if getattr(p, "main_grad", None) is not None else p.grad)
    theirs = run(ref, lambda p: p.grad)
    return {"ours": mine, "reference": theirs}


def w_reference_zero_parity(rank, world, ref_root, stage, steps):
    """Full-framework parity with the reference on CPU gloo ranks: the reference's own
    MixedPrecisionManager (ZeRO `stage`, torch AdamW), LR schedule, parameter groups and
    Trainer step against this package's, on the same weights and the same per-rank batches
    (DP=world, fp32 compute and master weights)."""
    from collections import OrderedDict
    from femtotron_b200.models.model_loader import shard_for_rank
    from femtotron_b200.models.parallel_plan import get_llama_parallel_plan
    RCtx, rbuild = _load_reference(ref_root)
    from femtotron.model.parallel_plan import get_llama_parallel_plan as rplan
    from femtotron.training.train_config import TrainConfig as RTC
    from femtotron.training.optimizer import get_param_groups as rgroups
    from femtotron.training.mixed_precision_manager import MixedPrecisionManager as RMP
    from femtotron.training.lr_schedule import create_lr_schedule as rlr
    from femtotron.sharding.factory import create_sharding_strategy as rstrat
    from femtotron.sharding.zero_config import ZeROConfig as RZ
    from femtotron.scripts.presets import get_wrap_policy
    from femtotron.parallel.data_parallel.gradient_synchronizer import create_grad_synchronizer as rsync
    cfg = tiny_config()
    cfg.use_cache = False
    sd = full_state(cfg)
    batches = _global_batches(cfg, steps, 2 * world, seed=13)
    mine = [b[rank * 2:(rank + 1) * 2] for b in batches]

    def it():
        for x in mine:
            yield {"input_ids": x, "labels": x}

    # ours: same hyper-parameters as _build_trainer (AdamW 5e-3, betas 0.9/0.95, wd 0.01,
    # warm-up 1 step, cosine to 0.1)
    tr = _build_trainer(cfg, sd, ctx_of(dp=world), stage, steps=steps, mb=2, ga=1, seed_data=1)
    gi = it()
    ours = [tr.train_step(gi)["loss"] for _ in range(steps)]

    rctx = RCtx(OrderedDict([("pp", 1), ("dp", world), ("tp", 1)]))
    ref = rbuild(cfg, rctx).to_empty(device="cpu")
    plan = get_llama_parallel_plan()
    with torch.no_grad():
        for name, p in ref.named_parameters():
            p.copy_(shard_for_rank(sd[name], name, plan, 0, 1))
        rot = ref.model.rotary_emb
        d = cfg.hidden_size // cfg.num_attention_heads
        theta = (getattr(cfg, "rope_parameters", None) or {}).get("rope_theta", 10000.0)
        inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
        rot.inv_freq.copy_(inv)
        if hasattr(rot, "original_inv_freq"):
            rot.original_inv_freq.copy_(inv)
    tc = RTC(master_dtype=torch.float32, param_dtype=torch.float32, grad_clip=None,
             train_steps=steps, log_interval=10 ** 6, checkpoint_interval=10 ** 6, warmup_steps=1,
             min_lr_ratio=0.1, lr=5e-3)
    wrap = get_wrap_policy("llama_decoder_layer") if stage == 3 else None
    strategy = rstrat(rctx, RZ(stage=stage, wrap_policy=wrap))
    mp = RMP(model=ref, sharding_strategy=strategy, parallel_ctx=rctx, parallel_plan=rplan(),
             config=tc, inner_optimizer_cls=torch.optim.AdamW,
             inner_optimizer_kwargs={"lr": 5e-3, "betas": (0.9, 0.95), "eps": 1e-8},
             compute_param_groups=rgroups(ref, weight_decay=0.01))
    sched = rlr(mp.inner, warmup_steps=1, total_steps=steps, min_lr_ratio=0.1)
    gs = rsync(mp.groups, rctx, strategy)
    mp.strategy.prepare_for_backward(mp.groups)
    # the reference Trainer pins cuda:{current_device} in its constructor, so its standard
    # step (femtotron/training/trainer.py:157-190, grad_accum_steps=1) is replayed here with
    # its own components; the optimizer step runs under no_grad (ZeRO-1/2 weight gathers
    # modify views in place, which autograd rejects on CPU)
    theirs = []
    for x in mine:
        loss = ref(input_ids=x, labels=x)["loss"]
        loss.backward()
        gs.sync_gradients()
        with torch.no_grad():
            mp.step()
        sched.step()
        theirs.append(loss.item())
    return {"ours": ours, "reference": theirs}


def w_reference_state_dict_interchange(rank, world, ref_root):
    """The model part of a checkpoint (HF parameter names, TP-sliced) is interchangeable with
    the reference's: same keys and shapes per TP rank, and a state dict of this package's
    model loads strictly into the reference model and reproduces its loss."""
    from collections import OrderedDict
    RCtx, rbuild = _load_reference(ref_root)
    from femtotron_b200.models import build_llama_model, materialize_model
    cfg = tiny_config()
    cfg.use_cache = False
    sd = full_state(cfg)
    ctx = ctx_of(tp=world)
    ours = build_llama_model(cfg, ctx)
    materialize_model(ours, "cpu", dtype=torch.float32, init_std=None)
    load_sharded(ours, sd, ctx)
    rctx = RCtx(OrderedDict([("pp", 1), ("dp", 1), ("tp", world)]))
    ref = rbuild(cfg, rctx).to_empty(device="cpu")
    mine = {k: v for k, v in ours.state_dict().items()}
    theirs = {k: v for k, v in ref.state_dict().items()}
    same_keys = set(mine) == set(theirs)
    same_shapes = same_keys and all(tuple(mine[k].shape) == tuple(theirs[k].shape) for k in mine)
    missing, unexpected = ref.load_state_dict(mine, strict=False)
    rot = ref.model.rotary_emb
    d = cfg.hidden_size // cfg.num_attention_heads
    theta = (getattr(cfg, "rope_parameters", None) or {}).get("rope_theta", 10000.0)
    with torch.no_grad():
        inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
        rot.inv_freq.copy_(inv)
        if hasattr(rot, "original_inv_freq"):
            rot.original_inv_freq.copy_(inv)
    x = _global_batches(cfg, 1, 2, seed=4)[0]
    with torch.no_grad():
        a = ours(x, labels=x)["loss"].item()
        b = ref(input_ids=x, labels=x)["loss"].item()
    return {"same_keys": same_keys, "same_shapes": same_shapes, "missing": list(missing),
            "unexpected": list(unexpected), "loss_ours": a, "loss_ref": b,
            "only_ours": sorted(set(mine) - set(theirs))[:5], "only_ref": sorted(set(theirs) - set(mine))[:5]}


def _reference_mp(ref_root, cfg, sd, rctx, stage, steps, lr=5e-3, dtype=torch.float32):
    """The reference's model + MixedPrecisionManager (torch AdamW) + LR schedule on CPU."""
    from femtotron_b200.models.model_loader import shard_for_rank
    from femtotron_b200.models.parallel_plan import get_llama_parallel_plan
    _, rbuild = _load_reference(ref_root)
    from femtotron.model.parallel_plan import get_llama_parallel_plan as rplan
    from femtotron.training.train_config import TrainConfig as RTC
    from femtotron.training.optimizer import get_param_groups as rgroups
    from femtotron.training.mixed_precision_manager import MixedPrecisionManager as RMP
    from femtotron.training.lr_schedule import create_lr_schedule as rlr
    from femtotron.sharding.factory import create_sharding_strategy as rstrat
    from femtotron.sharding.zero_config import ZeROConfig as RZ
    from femtotron.scripts.presets import get_wrap_policy
    from femtotron.parallel.data_parallel.gradient_synchronizer import create_grad_synchronizer as rsync
    ref = rbuild(cfg, rctx).to_empty(device="cpu")
    plan = get_llama_parallel_plan()
    with torch.no_grad():
        for name, p in ref.named_parameters():
            p.copy_(shard_for_rank(sd[name], name, plan, rctx.tp_rank, rctx.tp_size))
        rot = ref.model.rotary_emb
        d = cfg.hidden_size // cfg.num_attention_heads
        theta = (getattr(cfg, "rope_parameters", None) or {}).get("rope_theta", 10000.0)
        inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
        rot.inv_freq.copy_(inv)
        if hasattr(rot, "original_inv_freq"):
            rot.original_inv_freq.copy_(inv)
    if dtype != torch.float32:
        ref = ref.to(dtype)   # the reference's train.py casts the model (model.bfloat16())
        rot.inv_freq.data = rot.inv_freq.float()
    tc = RTC(master_dtype=torch.float32, param_dtype=dtype, grad_clip=None,
             train_steps=steps, log_interval=10 ** 6, checkpoint_interval=10 ** 6, warmup_steps=1,
             min_lr_ratio=0.1, lr=lr)
    wrap = get_wrap_policy("llama_decoder_layer") if stage == 3 else None
    strategy = rstrat(rctx, RZ(stage=stage, wrap_policy=wrap))
    mp = RMP(model=ref, sharding_strategy=strategy, parallel_ctx=rctx, parallel_plan=rplan(),
             config=tc, inner_optimizer_cls=torch.optim.AdamW,
             inner_optimizer_kwargs={"lr": lr, "betas": (0.9, 0.95), "eps": 1e-8},
             compute_param_groups=rgroups(ref, weight_decay=0.01))
    sched = rlr(mp.inner, warmup_steps=1, total_steps=steps, min_lr_ratio=0.1)
    gs = rsync(mp.groups, rctx, strategy)
    mp.strategy.prepare_for_backward(mp.groups)
    return ref, mp, sched, gs


def w_reference_checkpoint_resume(rank, world, ref_root, stage):
    """A user switching frameworks mid-run: the reference trains 2 steps and its checkpoint
    pieces (model state dict, MixedPrecisionManager state dict, scheduler state dict) are
    loaded into this package's trainer, which continues 2 steps; the reference continues too.
    The continued loss curves must agree."""
    from collections import OrderedDict
    RCtx, _ = _load_reference(ref_root)
    cfg = tiny_config()
    cfg.use_cache = False
    sd = full_state(cfg)
    steps = 4
    batches = [b[rank * 2:(rank + 1) * 2] for b in _global_batches(cfg, steps, 2 * world, seed=17)]
    rctx = RCtx(OrderedDict([("pp", 1), ("dp", world), ("tp", 1)]))
    ref, mp, sched, gs = _reference_mp(ref_root, cfg, sd, rctx, stage, steps)

    def ref_step(x):
        loss = ref(input_ids=x, labels=x)["loss"]
        loss.backward()
        gs.sync_gradients()
        with torch.no_grad():
            mp.step()
        sched.step()
        return loss.item()
    for x in batches[:2]:
        ref_step(x)
    # a checkpoint is a snapshot: state dicts hold live tensors on CPU, so round-trip them
    # through torch.save as the reference's Trainer does
    import io
    buf = io.BytesIO()
    torch.save({"model": ref.state_dict(), "optimizer": mp.state_dict(),
                "scheduler": sched.state_dict()}, buf)
    buf.seek(0)
    ckpt = torch.load(buf, weights_only=False)
    theirs = [ref_step(x) for x in batches[2:]]

    tr = _build_trainer(cfg, sd, ctx_of(dp=world), stage, steps=steps, mb=2, ga=1, seed_data=1)
    tr.model.load_state_dict(ckpt["model"], strict=False)
    tr.mp_manager.load_state_dict(ckpt["optimizer"])
    tr.scheduler.load_state_dict(ckpt["scheduler"])
    ours = [tr.train_step(iter([{"input_ids": x, "labels": x}]))["loss"] for x in batches[2:]]
    return {"ours": ours, "reference": theirs}


# ----------------------------------------------------------------------------- 3D parallelism
def w_3d(rank, world, stage, steps, gb):
    """TP=2 x PP=2 x DP=2 (1F1B, two micro-batches per step) with ZeRO `stage`: the loss curve
    on fixed global batches must equal a single process training on the same batches."""
    from femtotron_b200.models import build_llama_model, get_llama_parallel_plan, materialize_model
    from femtotron_b200.parallel.data_parallel import create_grad_synchronizer
    from femtotron_b200.parallel.pipeline_parallel import (PipelineComm, PipelineRunner, PipelineStage,
                                                           partition_layers)
    from femtotron_b200.parallel.pipeline_parallel.pipeline_config import PipelineConfig
    from femtotron_b200.sharding import ZeROConfig, create_sharding_strategy, llama_wrap_policy
    from femtotron_b200.training import (FusedAdamW, MixedPrecisionManager, TrainConfig, Trainer,
                                         create_lr_schedule, get_param_groups)
    cfg = tiny_config(num_hidden_layers=4, num_key_value_heads=2)
    sd = full_state(cfg)
    ctx = ctx_of(pp=2, dp=2, tp=2)
    nmb, seq = 2, 32
    per_rank = gb // ctx.dp_size
    rng = partition_layers(cfg.num_hidden_layers, ctx.pp_size)[ctx.pp_rank]
    m = build_llama_model(cfg, ctx, use_pp_aware=True, layer_range=rng)
    materialize_model(m, "cpu", dtype=torch.float32, init_std=None)
    load_sharded(m, sd, ctx)
    tc = TrainConfig(train_steps=steps, grad_accum_steps=1, master_dtype=torch.float32,
                     param_dtype=torch.float32, log_interval=10 ** 6, checkpoint_interval=10 ** 6,
                     warmup_steps=1, min_lr_ratio=0.1, pipeline_config=PipelineConfig(nmb, "1f1b"))
    st = create_sharding_strategy(ctx, ZeROConfig(stage=stage, wrap_policy=llama_wrap_policy))
    mp = MixedPrecisionManager(m, ctx, get_llama_parallel_plan(), tc, FusedAdamW,
                               dict(lr=5e-3, betas=(0.9, 0.95), eps=1e-8), get_param_groups(m, 0.01),
                               sharding_strategy=st)
    sch = create_lr_schedule(mp.inner, 1, steps)
    stage_ = PipelineStage(m, ctx, loss_scale=1.0 / nmb)
    comm = PipelineComm(ctx, seq, cfg.hidden_size, torch.float32, device=torch.device("cpu"))
    runner = PipelineRunner(stage_, comm, schedule_name="1f1b", num_microbatches=nmb,
                            recv_shape=(per_rank // nmb, seq, cfg.hidden_size), recv_dtype=torch.float32)
    tr = Trainer(m, mp, sch, None, create_grad_synchronizer(mp.groups, ctx, st), ctx, tc, pp_runner=runner)
    batches = _global_batches(cfg, steps, gb, seq=seq, seed=29)
    r = ctx.dp_rank
    losses = []
    for b in batches:
        x = b[r * per_rank:(r + 1) * per_rank]
        losses.append(tr.train_step(iter([{"input_ids": x, "labels": x}]))["loss"])
    t = torch.tensor(losses, dtype=torch.float64)
    dist.all_reduce(t)
    return (t / world).tolist()


def w_3d_single(rank, world, steps, gb):
    cfg = tiny_config(num_hidden_layers=4, num_key_value_heads=2)
    sd = full_state(cfg)
    return _run_split(cfg, sd, ctx_of(dp=1), 0, steps=steps, mb=gb, ga=1, seed=29)


# ----------------------------------------------------------------------------- TP comm ops
def w_tp_comm_ops(rank, world):
    """The six TP / SP autograd communication ops against their single-process meaning, on
    `world` ranks: forward values and input gradients of y = op(x) with loss sum(y * w)."""
    from femtotron_b200.parallel.tensor_parallel import comm_ops as C
    ctx = ctx_of(tp=world)
    g = ctx.tp_group
    torch.manual_seed(0)
    full = torch.randn(4 * world, 6 * world)          # the same on every rank
    wfull = torch.randn(4 * world, 6 * world)
    rows, cols = full.shape[0] // world, full.shape[1] // world
    res = {}

    def run(op, x, w):
        x = x.clone().requires_grad_(True)
        y = op(x)
        (y * w).sum().backward()
        return y.detach(), x.grad
    # scatter along the last dim: y = own column block; dx = all-gathered (zero-free) w blocks
    y, dx = run(lambda x: C.scatter_to_tp(x, g, -1), full, wfull[:, rank * cols:(rank + 1) * cols])
    res["scatter_fwd"] = torch.equal(y, full[:, rank * cols:(rank + 1) * cols])
    wblocks = [wfull[:, r * cols:(r + 1) * cols] for r in range(world)]
    res["scatter_bwd"] = torch.allclose(dx, torch.cat(wblocks, 1))
    # gather along the last dim: y = full; dx = own block of w
    y, dx = run(lambda x: C.gather_from_tp(x, g, -1), full[:, rank * cols:(rank + 1) * cols], wfull)
    res["gather_fwd"] = torch.equal(y, full)
    res["gather_bwd"] = torch.allclose(dx, wfull[:, rank * cols:(rank + 1) * cols])
    # copy (identity forward, all-reduce backward) and reduce (all-reduce forward, identity backward)
    y, dx = run(lambda x: C.copy_to_tp(x, g), full, wfull * (rank + 1))
    res["copy"] = torch.equal(y, full) and torch.allclose(dx, wfull * sum(range(1, world + 1)))
    y, dx = run(lambda x: C.reduce_from_tp(x, g), full * (rank + 1), wfull)
    res["reduce"] = torch.allclose(y, full * sum(range(1, world + 1))) and torch.allclose(dx, wfull)
    # sequence parallel: gather rows (backward reduce-scatters), reduce-scatter rows (backward gathers)
    y, dx = run(lambda x: C.gather_from_sp(x, g), full[rank * rows:(rank + 1) * rows], wfull * (rank + 1))
    res["sp_gather"] = torch.equal(y, full) and torch.allclose(
        dx, (wfull * sum(range(1, world + 1)))[rank * rows:(rank + 1) * rows])
    y, dx = run(lambda x: C.reduce_scatter_to_sp(x, g), full * (rank + 1), wfull[rank * rows:(rank + 1) * rows])
    res["sp_reduce_scatter"] = torch.allclose(y, (full * sum(range(1, world + 1)))[rank * rows:(rank + 1) * rows]) \
        and torch.allclose(dx, wfull)
    return res


# ----------------------------------------------------------------------------- ParamGroupCluster
def w_param_group_cluster(rank, world):
    """Reference test_param_group_cluster semantics on gloo ranks: a cluster takes over its
    parameter groups (compute data becomes a placeholder), holds this rank's slice of the
    padded flat buffer, unshard restores every parameter exactly, reshard drops it again, and a
    reduce-scatter of per-rank gradients yields this rank's slice of their mean."""
    from femtotron_b200.models import LlamaForTraining, materialize_model
    from femtotron_b200.models.parallel_plan import get_llama_parallel_plan
    from femtotron_b200.sharding.param_group_cluster import ParamGroupCluster
    from femtotron_b200.training.param_group import ParamGroup
    cfg = tiny_config(num_hidden_layers=1)
    sd = full_state(cfg)
    ctx = ctx_of(dp=world)
    with torch.device("meta"):
        m = LlamaForTraining(cfg)
    materialize_model(m, "cpu", dtype=torch.float32, init_std=None)
    m.load_state_dict(sd)
    layer = m.model.layers["0"] if hasattr(m.model.layers, "keys") else m.model.layers[0]
    names = {p: n for n, p in m.named_parameters()}
    pgs = [ParamGroup(names[p], p, None, {}, ctx, get_llama_parallel_plan()) for p in layer.parameters()]
    originals = {pg.name: pg.compute.detach().clone() for pg in pgs}
    total = sum(t.numel() for t in originals.values())
    c = ParamGroupCluster("layer0", layer, pgs, ctx.dp_group, torch.float32)
    out = {}
    out["claimed"] = all(pg.cluster is c for pg in pgs)
    out["placeholders"] = all(pg.compute.numel() == 0 for pg in pgs)
    out["shard_size"] = c.shard_size == -(-total // world) and c.padded_size == c.shard_size * world
    flat = torch.cat([originals[pg.name].reshape(-1) for pg in pgs])
    flat = torch.cat([flat, flat.new_zeros(c.padded_size - total)])
    out["shard_content"] = torch.equal(c.flat_param_shard, flat[rank * c.shard_size:(rank + 1) * c.shard_size])
    c.unshard()
    out["unshard_restores"] = all(torch.equal(pg.compute.detach(), originals[pg.name]) for pg in pgs)
    c.reshard()
    out["reshard_drops"] = all(pg.compute.numel() == 0 for pg in pgs)
    # reduce-scatter (AVG) of per-rank gradients
    c.unshard()
    c.prepare_grad_buffer()
    for pg in pgs:
        pg.compute.main_grad.copy_(torch.full_like(pg.compute.main_grad, float(rank + 1)))
    c.reduce_scatter_grads()
    c.reshard()
    mean = sum(range(1, world + 1)) / world
    want = torch.full((c.shard_size,), mean)
    lo = rank * c.shard_size
    pad_from = max(0, min(c.shard_size, total - lo))   # padding reduces to zero
    want[pad_from:] = 0.0
    out["reduce_scatter_mean"] = torch.allclose(c.flat_grad_shard, want)
    return out


# ----------------------------------------------------------------------------- PipelineComm
def w_pipeline_comm(rank, world):
    """Reference test_pipeline_comm on two pipeline ranks: forward / backward round trips, the
    combined send+recv operations of 1F1B's steady state (both sides submit at once without
    deadlocking), edge-stage no-ops, buffer validation and dtypes."""
    from femtotron_b200.parallel.pipeline_parallel import PipelineComm
    ctx = ctx_of(pp=world)
    out = {}
    for dtype in (torch.float32, torch.bfloat16):
        comm = PipelineComm(ctx, 8, 16, dtype, device=torch.device("cpu"))
        act = torch.full((8, 16), 1.0 + rank, dtype=dtype)
        if rank == 0:
            comm.send_forward(act)
            g = comm.recv_backward()
            out[f"roundtrip_{dtype}"] = torch.equal(g, torch.full((8, 16), 10.0, dtype=dtype))
            out[f"first_recv_forward_none_{dtype}"] = comm.recv_forward() is None
            # steady state: send activation i+1, receive gradient i, in one submission
            g2 = comm.send_forward_recv_backward(act * 2)
            out[f"sfrb_{dtype}"] = torch.equal(g2, torch.full((8, 16), 20.0, dtype=dtype))
        else:
            x = comm.recv_forward()
            out[f"roundtrip_{dtype}"] = torch.equal(x, torch.full((8, 16), 1.0, dtype=dtype))
            comm.send_backward(torch.full((8, 16), 10.0, dtype=dtype))
            out[f"last_recv_backward_none_{dtype}"] = comm.recv_backward() is None
            x2 = comm.send_backward_recv_forward(torch.full((8, 16), 20.0, dtype=dtype))
            out[f"sbrf_{dtype}"] = torch.equal(x2, torch.full((8, 16), 2.0, dtype=dtype))
    comm = PipelineComm(ctx, 8, 16, torch.float32, device=torch.device("cpu"))
    try:
        comm._buf(torch.empty(8, 16, dtype=torch.bfloat16))
        out["bad_dtype_refused"] = False
    except ValueError:
        out["bad_dtype_refused"] = True
    return out


# ----------------------------------------------------------------------------- memory ordering
def w_state_bytes(rank, world):
    """Reference test_zero1_2_3 memory ordering, as persistent state per rank after one step:
    compute parameters + fp32 masters + AdamW moments (+ ZeRO-3 cluster shards).  ZeRO-1 keeps
    1/dp of ZeRO-0's masters and moments; ZeRO-3 also shards the compute parameters."""
    cfg = tiny_config()
    sd = full_state(cfg)
    x = _global_batches(cfg, 1, 2 * world, seed=3)[0][rank * 2:(rank + 1) * 2]
    out = {}
    for stage in (0, 1, 2, 3):
        tr = _build_trainer(cfg, sd, ctx_of(dp=world), stage, steps=1, mb=2, ga=1, seed_data=1)
        tr.train_step(iter([{"input_ids": x, "labels": x}]))
        mp = tr.mp_manager
        tr.mp_manager.strategy.force_reshard_all() if stage == 3 else None
        seen, total = set(), 0

        def add(t):
            nonlocal total
            if t is not None and t.numel() and t.data_ptr() not in seen:
                seen.add(t.data_ptr())
                total += t.numel() * t.element_size()
        for p in tr.model.parameters():
            add(p.data)
        for g in mp.groups:
            add(g.master)
        for c in mp.clusters:
            add(c.flat_param_shard)
            add(c.master)
        for st in mp.inner.state.values():
            for v in st.values():
                if torch.is_tensor(v) and v.dim() > 0:
                    add(v)
        out[stage] = total
    return out


def w_reference_bf16_parity(rank, world, ref_root, stage, steps):
    """bf16 compute with fp32 master weights through the reference's MixedPrecisionManager and
    through this package's, same weights and per-rank batches: loss curves agree to bf16
    tolerance (the two compute the same math with different bf16 kernels and roundings)."""
    from collections import OrderedDict
    RCtx, _ = _load_reference(ref_root)
    cfg = tiny_config()
    cfg.use_cache = False
    sd = full_state(cfg)
    batches = [b[rank * 2:(rank + 1) * 2] for b in _global_batches(cfg, steps, 2 * world, seed=31)]
    tr = _build_trainer(cfg, sd, ctx_of(dp=world), stage, steps=steps, mb=2, ga=1, seed_data=1,
                        lr=1e-3, dtype=torch.bfloat16)
    ours = [tr.train_step(iter([{"input_ids": x, "labels": x}]))["loss"] for x in batches]
    rctx = RCtx(OrderedDict([("pp", 1), ("dp", world), ("tp", 1)]))
    ref, mp, sched, gs = _reference_mp(ref_root, cfg, sd, rctx, stage, steps, lr=1e-3, dtype=torch.bfloat16)
    theirs = []
    for x in batches:
        loss = ref(input_ids=x, labels=x)["loss"]
        loss.backward()
        gs.sync_gradients()
        with torch.no_grad():
            mp.step()
        sched.step()
        theirs.append(loss.item())
    return {"ours": ours, "reference": theirs}


# ----------------------------------------------------------------------------- export
def w_train_and_checkpoint(rank, world, tmpdir, tp, stage):
    """Train two steps (TP=tp, DP=world/tp, ZeRO `stage`), checkpoint at step 2, and return the
    trained model's loss on a fixed batch."""
    cfg = tiny_config()
    sd = full_state(cfg)
    ctx = ctx_of(dp=world // tp, tp=tp)
    tr = _build_trainer(cfg, sd, ctx, stage, steps=2, mb=2, ga=1, seed_data=5, ckpt=(tmpdir, 2))
    tr.train()
    x = _global_batches(cfg, 1, 2, seed=8)[0]
    with torch.no_grad():
        loss = tr.model(x, labels=x)["loss"].item()
    return {"loss": loss}


def w_share_fd(rank, world, tmpdir):
    """The descriptor hand-off of the NVLS set-up: rank 0's open file reaches every peer as a
    working descriptor of the same file (read with pread at offset 0)."""
    from femtotron_b200.parallel.nvls import share_fd
    payload = b"multicast handle stand-in"
    if rank == 0:
        path = os.path.join(tmpdir, "fd_payload.bin")
        with open(path, "wb") as f:
            f.write(payload)
        fd = os.open(path, os.O_RDONLY)
        try:
            got = share_fd(dist.group.WORLD, fd)
        finally:
            os.close(fd)
        return {"rank0_returns_none": got is None}
    fd = share_fd(dist.group.WORLD, None)
    try:
        data = os.pread(fd, len(payload), 0)
    finally:
        os.close(fd)
    return {"received": data == payload}


def w_zero3_variants(rank, world):
    """ZeRO-3 loss curves with the per-step gather cache forced on and off, and with the free
    parameters (embedding, final norm, LM head) sharded or replicated: the same math, so the
    same losses; plus the memory effect of sharding the free parameters."""
    cfg = tiny_config()
    sd = full_state(cfg)
    ctx = ctx_of(dp=world)
    out = {}
    saved = {k: os.environ.get(k) for k in ("FT_ZERO3_KEEP_IN_STEP", "FT_ZERO3_SHARD_FREE")}
    try:
        for keep in ("0", "1"):
            for shard in ("0", "1"):
                os.environ["FT_ZERO3_KEEP_IN_STEP"] = keep
                os.environ["FT_ZERO3_SHARD_FREE"] = shard
                tr = _build_trainer(cfg, sd, ctx, 3, steps=4, mb=2, ga=2, seed_data=3, ac=True)
                st = tr.mp_manager.strategy
                hist = tr.train()
                t = torch.tensor([h["loss"] for h in hist])
                dist.all_reduce(t)
                state = sum(c.master.numel() for c in tr.mp_manager.clusters) + \
                    sum(g.master.numel() for g in tr.mp_manager.groups if g.master is not None)
                out[f"keep{keep}_shard{shard}"] = {"loss": (t / world).tolist(),
                                                   "keep": st.keep_in_step,
                                                   "free_clusters": len(st.free_clusters),
                                                   "master_elems": state}
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    return out
