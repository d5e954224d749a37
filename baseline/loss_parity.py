"""Loss-curve parity on GPUs: this framework against the unmodified reference, same initial
weights, same token batches, same optimizer settings, bf16 compute with fp32 master weights.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 baseline/loss_parity.py \
        [--layers 4] [--seq 2048] [--steps 100] [--stage 3] [--json out.json]

Model: the Llama-3-8B shape (hidden 4096, 32 heads, 8 KV heads, FFN 14336, vocab 128256,
RoPE theta 5e5) at reduced depth; ZeRO stage `--stage` over all ranks (data parallel), full
activation checkpointing, AdamW (lr 3e-4, betas 0.9/0.95, eps 1e-8, weight decay 0.01, warm-up
10 steps then cosine to 0.1), micro-batch 1, one micro-batch per step.  Weights: norms 1, the
rest N(0, 0.02) from a fixed seed, generated once on the CPU and loaded by both frameworks.
Data: uniform token ids from a fixed seed, a different batch per rank and step.

Both models live in every process; they train one after the other.  Rank 0 prints one JSON
line with both loss curves (mean over ranks) and the largest absolute difference.  The
reference's own tolerance for ZeRO loss curves is 0.02
(femtotron/test/integration/test_zero1_2_3.py:415-426).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from collections import OrderedDict

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, ROOT)

import femtotron_b200  # noqa: E402,F401
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def full_state(cfg, seed: int = 0) -> dict:
    from femtotron_b200.models import LlamaForTraining, materialize_model

    def init(name, p):
        if p.dim() == 1:
            p.fill_(1.0)
        else:
            p.normal_(0.0, 0.02)
    torch.manual_seed(seed)
    with torch.device("meta"):
        m = LlamaForTraining(cfg)
    materialize_model(m, "cpu", dtype=torch.float32, init_fn=init)
    return {k: v.detach().clone() for k, v in m.state_dict().items()}


def ours(cfg, sd, batches, args, device):
    from femtotron_b200.models import build_llama_model, get_llama_parallel_plan, materialize_model
    from femtotron_b200.models.layers import LlamaDecoderLayer
    from femtotron_b200.parallel.data_parallel import create_grad_synchronizer
    from femtotron_b200.parallel_context import ParallelContext
    from femtotron_b200.sharding import ZeROConfig, create_sharding_strategy, llama_wrap_policy
    from femtotron_b200.training import (FusedAdamW, MixedPrecisionManager, TrainConfig, Trainer,
                                         apply_activation_checkpointing, create_lr_schedule,
                                         get_param_groups)
    from femtotron_b200.training.ckpt_policy import by_class
    ctx = ParallelContext(OrderedDict(dp=dist.get_world_size()))
    m = build_llama_model(cfg, ctx)
    materialize_model(m, device, dtype=torch.bfloat16, init_std=None)
    with torch.no_grad():
        for name, p in m.named_parameters():
            p.copy_(sd[name].to(p.dtype))
    tc = TrainConfig(train_steps=args.steps, grad_accum_steps=1, master_dtype=torch.float32,
                     param_dtype=torch.bfloat16, log_interval=10 ** 9, checkpoint_interval=10 ** 9,
                     warmup_steps=10, min_lr_ratio=0.1, grad_clip=None)
    st = create_sharding_strategy(ctx, ZeROConfig(stage=args.stage, wrap_policy=llama_wrap_policy))
    mp = MixedPrecisionManager(m, ctx, get_llama_parallel_plan(), tc, FusedAdamW,
                               dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-8), get_param_groups(m, 0.01),
                               sharding_strategy=st)
    apply_activation_checkpointing(m, by_class(LlamaDecoderLayer), use_reentrant=False,
                                   preserve_rng_state=False)
    sched = create_lr_schedule(mp.inner, 10, args.steps, 0.1)
    tr = Trainer(m, mp, sched, None, create_grad_synchronizer(mp.groups, ctx, st), ctx, tc)
    out = [tr.train_step(iter([{"input_ids": x, "labels": x}]))["loss"] for x in batches]
    if device.type == "cuda":
        from femtotron_b200.ops.ext import check_kernel_errors
        check_kernel_errors(device)      # a bounded wait that gave up fails the comparison
    mp.cleanup()
    return out


def reference(cfg, sd, batches, args, device):
    ref_root = os.path.join(HERE, "_ref")
    if not os.path.isdir(os.path.join(ref_root, "femtotron")):
        sys.path.insert(0, HERE)
        import install_reference
        if dist.get_rank() == 0:
            install_reference.install()
        dist.barrier()
    sys.path.insert(0, ref_root)
    from femtotron.parallel_context import ParallelContext as RCtx
    from femtotron.model.llama import build_llama_model as rbuild
    from femtotron.model.parallel_plan import get_llama_parallel_plan as rplan
    from femtotron.training.train_config import TrainConfig as RTC
    from femtotron.training.optimizer import get_param_groups as rgroups
    from femtotron.training.mixed_precision_manager import MixedPrecisionManager as RMP
    from femtotron.training.lr_schedule import create_lr_schedule as rlr
    from femtotron.training.activation_ckpt import apply_activation_checkpointing as rac
    from femtotron.sharding.factory import create_sharding_strategy as rstrat
    from femtotron.sharding.zero_config import ZeROConfig as RZ
    from femtotron.scripts.presets import get_wrap_policy, get_ac_policy
    from femtotron.parallel.data_parallel.gradient_synchronizer import create_grad_synchronizer as rsync
    rctx = RCtx(OrderedDict([("pp", 1), ("dp", dist.get_world_size()), ("tp", 1)]))
    with torch.device("meta"):
        ref = rbuild(cfg, rctx)
    ref = ref.to_empty(device=device)
    with torch.no_grad():
        for name, p in ref.named_parameters():
            p.copy_(sd[name].to(device))
        # the reference's own tests recompute RoPE inv_freq after to_empty
        rot = ref.model.rotary_emb
        d = cfg.hidden_size // cfg.num_attention_heads
        theta = (getattr(cfg, "rope_parameters", None) or {}).get("rope_theta", 500000.0)
        inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float32, device=device) / d))
        rot.inv_freq.copy_(inv)
        if hasattr(rot, "original_inv_freq"):
            rot.original_inv_freq.copy_(inv)
    ref = ref.bfloat16()
    rot.inv_freq.data = rot.inv_freq.float()
    tc = RTC(master_dtype=torch.float32, param_dtype=torch.bfloat16, grad_clip=None,
             train_steps=args.steps, log_interval=10 ** 9, checkpoint_interval=10 ** 9,
             warmup_steps=10, min_lr_ratio=0.1, lr=3e-4)
    wrap = get_wrap_policy("llama_decoder_layer") if args.stage == 3 else None
    strategy = rstrat(rctx, RZ(stage=args.stage, wrap_policy=wrap))
    mp = RMP(model=ref, sharding_strategy=strategy, parallel_ctx=rctx, parallel_plan=rplan(),
             config=tc, inner_optimizer_cls=torch.optim.AdamW,
             inner_optimizer_kwargs={"lr": 3e-4, "betas": (0.9, 0.95), "eps": 1e-8},
             compute_param_groups=rgroups(ref, weight_decay=0.01))
    rac(ref, get_ac_policy("llama_decoder_layer"), use_reentrant=False, preserve_rng_state=False)
    sched = rlr(mp.inner, warmup_steps=10, total_steps=args.steps, min_lr_ratio=0.1)
    gs = rsync(mp.groups, rctx, strategy)
    mp.strategy.prepare_for_backward(mp.groups)
    out = []
    for x in batches:
        loss = ref(input_ids=x, labels=x)["loss"]
        loss.backward()
        gs.sync_gradients()
        with torch.no_grad():
            mp.step()
        sched.step()
        out.append(loss.item())
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--stage", type=int, default=3)
    ap.add_argument("--json", default=None)
    args = ap.parse_args()
    from transformers import LlamaConfig
    from femtotron_b200.utils.dist import init_distributed
    rank, world, local = init_distributed("nccl", timeout_s=int(os.environ.get("FT_PG_TIMEOUT", "300")))
    device = torch.device("cuda", local)
    cfg = LlamaConfig(hidden_size=4096, intermediate_size=14336, num_attention_heads=32,
                      num_key_value_heads=8, num_hidden_layers=args.layers, vocab_size=128256,
                      max_position_embeddings=max(8192, args.seq), rms_norm_eps=1e-5,
                      rope_theta=500000.0, tie_word_embeddings=False, attn_implementation="sdpa")
    cfg.use_cache = False
    sd = full_state(cfg)
    g = torch.Generator().manual_seed(11)
    data = torch.randint(0, cfg.vocab_size, (args.steps, world, args.seq), generator=g)
    batches = [data[i, rank:rank + 1].to(device) for i in range(args.steps)]
    a = ours(cfg, sd, batches, args, device)
    torch.cuda.empty_cache()
    b = reference(cfg, sd, batches, args, device)
    t = torch.tensor([a, b], dtype=torch.float64, device=device)
    dist.all_reduce(t)
    t /= world
    a, b = t[0].tolist(), t[1].tolist()
    diff = max(abs(x - y) for x, y in zip(a, b))
    if rank == 0:
        res = {"layers": args.layers, "seq": args.seq, "steps": args.steps, "zero_stage": args.stage,
               "dp": world, "max_abs_diff": diff, "first": [a[0], b[0]], "last": [a[-1], b[-1]],
               "ours": a, "reference": b}
        print(json.dumps(res), flush=True)
        if args.json:
            with open(args.json, "w") as f:
                json.dump(res, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
