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
                   ac=False, delay_seed=None, check_finite=False):
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
    materialize_model(m, "cpu", dtype=torch.float32, init_std=None)
    load_sharded(m, sd, ctx)
    if delay_seed is not None:
        _inject_delays(m, delay_seed)
    tc = TrainConfig(train_steps=steps, grad_accum_steps=ga, master_dtype=torch.float32,
                     param_dtype=torch.float32, log_interval=10 ** 6,
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
        emb = nan_tr.model.model.embed_tokens.weight
        emb.fill_(float("nan"))
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
