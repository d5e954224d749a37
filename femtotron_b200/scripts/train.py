"""Training entry point: YAML config + command-line overrides (reference
femtotron/scripts/train.py:63-425).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m femtotron_b200.scripts.train \\
        --config configs/tiny_llama_debug.yaml --tp 2 --zero_stage 3

Accepted YAML keys (same names as the reference): tp, dp, pp, zero_stage, zero_wrap_policy,
ac_enabled, ac_policy, ac_use_reentrant, ac_preserve_rng_state, model_name, hidden_size,
intermediate_size, num_attention_heads, num_key_value_heads, num_hidden_layers,
max_position_embeddings, vocab_size, tie_word_embeddings, init_std, dataset, num_samples,
seq_len, tokenizer, data_dir, train_steps, micro_batch_size, lr, weight_decay, adam_beta1,
adam_beta2, adam_eps, grad_clip, warmup_steps, min_lr_ratio, log_interval,
checkpoint_interval, checkpoint_dir.  Additionally honoured: grad_accum_steps,
num_microbatches and schedule (pipeline), sequence_parallel, rope_theta, rms_norm_eps,
synthetic_data (uniform random tokens instead of a tokenised dataset), seed, metrics_path.

Unlike the reference script, pipeline parallelism (pp > 1) builds a PipelineRunner, gradient
clipping and gradient accumulation are applied, and the vocabulary comes from the config
when synthetic data is used.
"""
from __future__ import annotations

import argparse
import os
import sys
from collections import OrderedDict

import torch
import torch.distributed as dist
import yaml

from femtotron_b200.utils.dist import init_distributed


def log(msg: str) -> None:
    if not dist.is_initialized() or dist.get_rank() == 0:
        print(f"[femtotron_b200] {msg}", flush=True)


def _bool(x: str) -> bool:
    v = x.lower()
    if v in ("true", "1", "yes", "on"):
        return True
    if v in ("false", "0", "no", "off"):
        return False
    raise argparse.ArgumentTypeError(f"expected true/false, got {x!r}")


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="femtotron_b200 LLaMA pretraining")
    p.add_argument("--config", type=str, default=None)
    for k in ("dp", "tp", "pp", "zero_stage", "num_hidden_layers", "hidden_size", "intermediate_size",
              "num_attention_heads", "num_key_value_heads", "vocab_size", "max_position_embeddings",
              "train_steps", "micro_batch_size",
              "seq_len", "warmup_steps", "num_samples", "log_interval", "checkpoint_interval",
              "grad_accum_steps", "num_microbatches", "seed"):
        p.add_argument(f"--{k}", type=int, default=None)
    for k in ("lr", "grad_clip", "weight_decay", "min_lr_ratio", "init_std", "rope_theta", "rms_norm_eps"):
        p.add_argument(f"--{k}", type=float, default=None)
    for k in ("zero_wrap_policy", "ac_policy", "model_name", "dataset", "checkpoint_dir", "resume",
              "schedule", "metrics_path", "data_dir", "tokenizer"):
        p.add_argument(f"--{k}", type=str, default=None)
    for k in ("ac_enabled", "sequence_parallel", "synthetic_data"):
        # `--ac_enabled true|false` as in the reference's CLI, or the bare flag for true
        p.add_argument(f"--{k}", type=_bool, nargs="?", const=True, default=None)
    return p.parse_args(argv)


DEFAULTS = dict(tp=1, pp=1, zero_stage=0, zero_wrap_policy="llama_decoder_layer", ac_enabled=False,
                ac_policy="llama_decoder_layer", ac_use_reentrant=False, ac_preserve_rng_state=True,
                model_name=None, hidden_size=256, intermediate_size=512, num_attention_heads=8,
                num_key_value_heads=4, num_hidden_layers=4, max_position_embeddings=512,
                vocab_size=32000, tie_word_embeddings=False, init_std=0.02, seq_len=128,
                num_samples=2000, train_steps=100, micro_batch_size=4, lr=3e-4, weight_decay=0.01,
                adam_beta1=0.9, adam_beta2=0.95, adam_eps=1e-8, grad_clip=1.0, warmup_steps=10,
                min_lr_ratio=0.1, log_interval=10, checkpoint_interval=1000,
                checkpoint_dir="./checkpoints", grad_accum_steps=1, num_microbatches=1,
                schedule="1f1b", sequence_parallel=False, rope_theta=10000.0, rms_norm_eps=1e-5,
                synthetic_data=True, seed=1234, metrics_path=None, data_dir="./data", dataset=None,
                tokenizer=None)


def load_config(args) -> dict:
    """DEFAULTS <- YAML <- command line.  ``cfg["_explicit"]`` names the keys the user set
    (YAML or command line), as opposed to defaults."""
    cfg = dict(DEFAULTS)
    explicit: set[str] = set()
    if args.config:
        with open(args.config) as f:
            y = {k: v for k, v in (yaml.safe_load(f) or {}).items()}
        cfg.update(y)
        explicit |= set(y)
    cli = {k: v for k, v in vars(args).items() if v is not None and k != "config"}
    cfg.update(cli)
    explicit |= set(cli)
    cfg["_explicit"] = explicit
    return cfg


def model_config_from(cfg: dict):
    from transformers import AutoConfig, LlamaConfig
    if cfg.get("model_name"):
        mc = AutoConfig.from_pretrained(cfg["model_name"])
        # a pretrained config keeps its own depth unless the user asked for another one
        if "num_hidden_layers" in cfg.get("_explicit", ()):
            mc.num_hidden_layers = cfg["num_hidden_layers"]
        return mc
    return LlamaConfig(hidden_size=cfg["hidden_size"], intermediate_size=cfg["intermediate_size"],
                       num_attention_heads=cfg["num_attention_heads"],
                       num_key_value_heads=cfg["num_key_value_heads"],
                       num_hidden_layers=cfg["num_hidden_layers"],
                       max_position_embeddings=max(cfg["max_position_embeddings"], cfg["seq_len"]),
                       vocab_size=cfg["vocab_size"], rms_norm_eps=cfg["rms_norm_eps"],
                       rope_theta=cfg["rope_theta"], tie_word_embeddings=cfg["tie_word_embeddings"])


def build_all(cfg: dict):
    from femtotron_b200.data import (DistributedDataLoader, PackedDataset, SyntheticTokens,
                                     simple_pretrain_collator)
    from femtotron_b200.models import (build_llama_model, get_llama_parallel_plan,
                                       materialize_model)
    from femtotron_b200.models.model_loader import ModelLoader
    from femtotron_b200.parallel.data_parallel import create_grad_synchronizer
    from femtotron_b200.parallel.pipeline_parallel import (PipelineComm, PipelineRunner,
                                                           PipelineStage, partition_layers)
    from femtotron_b200.parallel_context import ParallelContext
    from femtotron_b200.scripts.presets import get_ac_policy, get_wrap_policy
    from femtotron_b200.sharding import ZeROConfig, create_sharding_strategy
    from femtotron_b200.training import (ClipGradNorm, FusedAdamW, MixedPrecisionManager,
                                         TrainConfig, Trainer, apply_activation_checkpointing,
                                         create_lr_schedule, get_param_groups)
    from femtotron_b200.parallel.pipeline_parallel.pipeline_config import PipelineConfig

    world = dist.get_world_size()
    tp, pp = cfg["tp"], cfg["pp"]
    dp = cfg.get("dp") or world // (tp * pp)
    if dp * tp * pp != world:
        raise ValueError(f"dp({dp}) * tp({tp}) * pp({pp}) != world_size({world})")
    ctx = ParallelContext(OrderedDict([("pp", pp), ("dp", dp), ("tp", tp)]))
    device = ctx.device
    log(f"parallel: dp={dp} tp={tp} pp={pp} sp={cfg['sequence_parallel']} zero={cfg['zero_stage']}")
    mc = model_config_from(cfg)
    torch.manual_seed(cfg["seed"])
    layer_range = partition_layers(mc.num_hidden_layers, pp)[ctx.pp_rank] if pp > 1 else None
    model = build_llama_model(mc, ctx, use_pp_aware=pp > 1, layer_range=layer_range,
                              sequence_parallel=cfg["sequence_parallel"])
    if cfg.get("model_name"):
        materialize_model(model, device, dtype=torch.bfloat16, init_std=None)
        ModelLoader(ctx).load_and_distribute(model, cfg["model_name"], device=device)
    else:
        materialize_model(model, device, dtype=torch.bfloat16, init_std=cfg["init_std"])
    log(f"model: {sum(p.numel() for p in model.parameters()):,} parameters on this rank")
    tc = TrainConfig(train_steps=cfg["train_steps"], grad_accum_steps=cfg["grad_accum_steps"],
                     grad_clip=cfg["grad_clip"], log_interval=cfg["log_interval"],
                     checkpoint_interval=cfg["checkpoint_interval"], checkpoint_dir=cfg["checkpoint_dir"],
                     master_dtype=torch.float32, param_dtype=torch.bfloat16, lr=cfg["lr"],
                     warmup_steps=cfg["warmup_steps"], min_lr_ratio=cfg["min_lr_ratio"],
                     metrics_path=cfg.get("metrics_path"),
                     pipeline_config=PipelineConfig(cfg["num_microbatches"], cfg["schedule"]))
    wrap = get_wrap_policy(cfg["zero_wrap_policy"]) if cfg["zero_stage"] == 3 else None
    strategy = create_sharding_strategy(ctx, ZeROConfig(stage=cfg["zero_stage"], wrap_policy=wrap))
    transforms = [ClipGradNorm(cfg["grad_clip"], ctx, dp_sharded=strategy.grads_are_dp_sharded())] \
        if cfg["grad_clip"] else None
    mp = MixedPrecisionManager(model, ctx, get_llama_parallel_plan(cfg["sequence_parallel"]), tc,
                               FusedAdamW,
                               dict(lr=cfg["lr"], betas=(cfg["adam_beta1"], cfg["adam_beta2"]),
                                    eps=cfg["adam_eps"]),
                               get_param_groups(model, cfg["weight_decay"]),
                               grad_transforms=transforms, sharding_strategy=strategy)
    if cfg["ac_enabled"]:
        n = apply_activation_checkpointing(model, get_ac_policy(cfg["ac_policy"]),
                                           use_reentrant=cfg["ac_use_reentrant"],
                                           preserve_rng_state=cfg["ac_preserve_rng_state"])
        log(f"activation checkpointing: {n} modules")
    sched = create_lr_schedule(mp.inner, tc.warmup_steps, tc.train_steps, tc.min_lr_ratio)
    S, mb = cfg["seq_len"], cfg["micro_batch_size"]
    if cfg["synthetic_data"] or not cfg.get("dataset"):
        data = SyntheticTokens(cfg["num_samples"], S, mc.vocab_size, seed=cfg["seed"])
    else:
        from femtotron_b200.data.preprocess import preprocess
        path = os.path.join(cfg["data_dir"], f"{cfg['dataset'].replace('/', '_')}_seq{S}.pt")
        if dist.get_rank() == 0 and not os.path.exists(path):
            os.makedirs(cfg["data_dir"], exist_ok=True)
            preprocess(cfg["dataset"], cfg.get("tokenizer") or cfg["model_name"], path, S,
                       num_samples=cfg["num_samples"])
        dist.barrier()
        data = PackedDataset(path)
    global_mb = mb * (cfg["num_microbatches"] if pp > 1 else 1)
    dl = DistributedDataLoader(data, ctx, global_mb, simple_pretrain_collator, seed=cfg["seed"],
                               num_workers=2)
    runner = None
    if pp > 1:
        stage = PipelineStage(model, ctx, loss_scale=1.0 / cfg["num_microbatches"])
        shape = (mb, S, mc.hidden_size) if not cfg["sequence_parallel"] else (mb * S // tp, mc.hidden_size)
        comm = PipelineComm(ctx, S, mc.hidden_size, torch.bfloat16)
        runner = PipelineRunner(stage, comm, schedule_name=cfg["schedule"],
                                num_microbatches=cfg["num_microbatches"], recv_shape=shape,
                                recv_dtype=torch.bfloat16)
    gs = create_grad_synchronizer(mp.groups, ctx, strategy)
    return Trainer(model, mp, sched, dl, gs, ctx, tc, pp_runner=runner)


def main(argv=None):
    args = parse_args(argv)
    cfg = load_config(args)
    init_distributed()
    trainer = build_all(cfg)
    if cfg.get("resume"):
        trainer._load_checkpoint(cfg["resume"])
    trainer.train()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1:])
