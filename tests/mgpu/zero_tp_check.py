"""2-GPU NCCL checks launched by tests/test_multigpu.py through torchrun:
ZeRO-0 and ZeRO-3 (DP=2) give the same bf16 loss curve, and a TP=2 model with sequence
parallelism gives the TP=1 loss on the same weights."""
import json
import os
import sys
from collections import OrderedDict

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from femtotron_b200.utils.dist import init_distributed  # noqa: E402


def train(stage, ctx, cfg, sd, steps=4):
    from common_models import load_sharded
    from femtotron_b200.data import DistributedDataLoader, SyntheticTokens, simple_pretrain_collator
    from femtotron_b200.models import build_llama_model, get_llama_parallel_plan, materialize_model
    from femtotron_b200.models.layers import LlamaDecoderLayer
    from femtotron_b200.parallel.data_parallel import create_grad_synchronizer
    from femtotron_b200.sharding import ZeROConfig, create_sharding_strategy, llama_wrap_policy
    from femtotron_b200.training import (FusedAdamW, MixedPrecisionManager, TrainConfig, Trainer,
                                         apply_activation_checkpointing, create_lr_schedule,
                                         get_param_groups)
    from femtotron_b200.training.ckpt_policy import by_class
    m = build_llama_model(cfg, ctx)
    materialize_model(m, "cuda", dtype=torch.bfloat16, init_std=None)
    load_sharded(m, sd, ctx)
    tc = TrainConfig(train_steps=steps, grad_accum_steps=2, master_dtype=torch.float32,
                     log_interval=10 ** 6, warmup_steps=1)
    st = create_sharding_strategy(ctx, ZeROConfig(stage=stage, wrap_policy=llama_wrap_policy))
    mp = MixedPrecisionManager(m, ctx, get_llama_parallel_plan(), tc, FusedAdamW,
                               dict(lr=3e-3, betas=(0.9, 0.95), eps=1e-8), get_param_groups(m, 0.01),
                               sharding_strategy=st)
    apply_activation_checkpointing(m, by_class(LlamaDecoderLayer))
    sch = create_lr_schedule(mp.inner, 1, steps)
    ds = SyntheticTokens(64, 256, cfg.vocab_size, seed=3)
    dl = DistributedDataLoader(ds, ctx, 2, simple_pretrain_collator, num_workers=0)
    tr = Trainer(m, mp, sch, dl, create_grad_synchronizer(mp.groups, ctx, st), ctx, tc)
    losses = torch.tensor([h["loss"] for h in tr.train()], device="cuda")
    dist.all_reduce(losses)
    from femtotron_b200.ops import check_kernel_errors
    check_kernel_errors()
    return (losses / dist.get_world_size()).tolist()


def tp_loss(cfg, sd, tp, sp):
    from common_models import load_sharded
    from femtotron_b200.models import build_llama_model, materialize_model
    from femtotron_b200.parallel_context import ParallelContext
    ctx = ParallelContext(OrderedDict(tp=tp, dp=dist.get_world_size() // tp))
    m = build_llama_model(cfg, ctx, sequence_parallel=sp)
    materialize_model(m, "cuda", dtype=torch.bfloat16, init_std=None)
    load_sharded(m, sd, ctx)
    torch.manual_seed(5)
    ids = torch.randint(0, cfg.vocab_size, (2, 256), device="cuda")
    loss = m(ids, labels=ids)["loss"]
    loss.backward()
    # per-parameter squared gradient norms of the logical (unsharded) tensors
    from femtotron_b200.models.parallel_plan import get_llama_parallel_plan
    plan = get_llama_parallel_plan()
    norms = {}
    for n, p in m.named_parameters():
        g = p.main_grad if getattr(p, "main_grad", None) is not None else p.grad
        sq = g.float().pow(2).sum()
        rule = plan.get_rule(n.rsplit(".", 1)[0]) if tp > 1 else None
        if rule is not None and rule.parallel_type != "replicate":
            dist.all_reduce(sq, group=ctx.tp_group)
        norms[n] = sq.sqrt().item()
    return loss.item(), norms


def main():
    from common_models import full_state, tiny_config
    from femtotron_b200.parallel_context import ParallelContext
    init_distributed("nccl", timeout_s=120)
    cfg = tiny_config(hidden_size=256, intermediate_size=512, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=1024, max_position_embeddings=512)
    sd = full_state(cfg)
    ctx = ParallelContext(OrderedDict(dp=dist.get_world_size()))
    z0 = train(0, ctx, cfg, sd)
    z3 = train(3, ctx, cfg, sd)
    os.environ["FT_ZERO3_SYMM"] = "0"       # NCCL all-gather / reduce-scatter for comparison
    z3_nccl = train(3, ctx, cfg, sd)
    os.environ.pop("FT_ZERO3_SYMM")
    os.environ["FT_FUSED_RS_ADAMW"] = "0"   # reduce-scatter, then the optimizer at step time
    z3_p2p = train(3, ctx, cfg, sd)
    os.environ.pop("FT_FUSED_RS_ADAMW")
    t1, g1 = tp_loss(cfg, sd, 1, False)
    t2, g2 = tp_loss(cfg, sd, 2, True)
    worst = max(abs(g1[k] - g2[k]) / (g1[k] + 1e-12) for k in g1)
    res = {"z0": z0, "z3": z3, "z3_nccl": z3_nccl, "z3_p2p": z3_p2p, "tp1": t1, "tp2_sp": t2, "grad_norm_rel_err": worst}
    if dist.get_rank() == 0:
        print("RESULT " + json.dumps(res), flush=True)
        out = os.environ.get("FT_TEST_RESULT_DIR")
        if out:
            with open(os.path.join(out, "zero_tp_check.json"), "w") as f:
                json.dump(res, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
