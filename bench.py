"""Headline benchmark: Llama-3-8B training throughput (tokens/s for the whole job + MFU) with
ZeRO-3 data parallelism over N B200 GPUs of one node, seq 4096, micro-batch 1, gradient
accumulation 8, full activation checkpointing, bf16 compute with fp32 master weights and
AdamW; synthetic uniform token ids and random-init weights.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Per step each GPU processes grad_accum x micro_batch x seq tokens (weak scaling).

Two measurements of our implementation, each over K steps after W warm-up steps:
  * ``value``: device time (CUDA events on the compute stream, barrier + synchronize on both
    sides, max over ranks) of K steps with the micro-batches already on the device;
  * ``e2e``: K steps through the public API (Trainer.train_step over a DistributedDataLoader):
    every step copies its token ids from pinned host memory to the device and reads the
    loss back to the host; host wall clock, max over ranks.
The per-step working set (weights, optimizer state, activations: >100 GB) exceeds the 126 MB
L2 cache, so no explicit L2 flush is needed between steps.

``--config llama2-13b-tp-sp`` measures the secondary BASELINE configuration instead: Llama-2-13B
with tensor parallelism over all N GPUs plus sequence parallelism (DP=1, micro-batch 2,
seq 4096, no activation checkpointing; strong scaling).

``--impl reference`` runs the unmodified reference (installed under baseline/_ref) through
its own public API on the same configuration and prints the same JSON line with
"impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
import traceback

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
METRIC = "tokens/sec/box + MFU, Llama-3-8B ZeRO-3 & TP=8, 1/2/4/8 B200, max over ranks"

LLAMA3_8B = dict(hidden_size=4096, intermediate_size=14336, num_attention_heads=32,
                 num_key_value_heads=8, num_hidden_layers=32, vocab_size=128256,
                 max_position_embeddings=8192, rms_norm_eps=1e-5, rope_theta=500000.0,
                 tie_word_embeddings=False)


LLAMA2_13B = dict(hidden_size=5120, intermediate_size=13824, num_attention_heads=40,
                  num_key_value_heads=40, num_hidden_layers=40, vocab_size=32000,
                  max_position_embeddings=4096, rms_norm_eps=1e-5, rope_theta=10000.0,
                  tie_word_embeddings=False)

# --config: the default is the headline benchmark; the others are secondary BASELINE configs
CONFIGS = {
    "llama3-8b-zero3": dict(model=LLAMA3_8B, name="Llama-3-8B", micro_batch=1, grad_accum=8, seq=4096),
    "llama2-13b-tp-sp": dict(model=LLAMA2_13B, name="Llama-2-13B", micro_batch=2, grad_accum=1, seq=4096),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="llama3-8b-zero3", choices=sorted(CONFIGS),
                    help="llama3-8b-zero3: ZeRO-3 over all GPUs (headline); llama2-13b-tp-sp: "
                         "tensor parallel over all GPUs with sequence parallelism, DP=1")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seq", type=int, default=None)
    ap.add_argument("--micro-batch", type=int, default=None)
    ap.add_argument("--grad-accum", type=int, default=None)
    ap.add_argument("--layers", type=int, default=None,
                    help="override layer count (debug only; results are then not the benchmark)")
    ap.add_argument("--no-e2e", action="store_true")
    args = ap.parse_args()
    c = CONFIGS[args.config]
    args.seq = args.seq or c["seq"]
    args.micro_batch = args.micro_batch or c["micro_batch"]
    args.grad_accum = args.grad_accum or c["grad_accum"]
    args.tp = args.config == "llama2-13b-tp-sp"
    args.model_name = c["name"]
    return args


def model_config(layers=None, config="llama3-8b-zero3"):
    from transformers import LlamaConfig
    kw = dict(CONFIGS[config]["model"])
    if layers:
        kw["num_hidden_layers"] = layers
    cfg = LlamaConfig(**kw)
    cfg.use_cache = False
    return cfg


def flops_per_token(cfg, seq) -> float:
    """Model FLOPs per trained token: 6 x (matmul parameters) + 6 x L x H x S for causal
    attention (score and value products, forward+backward).  Recomputation is not counted."""
    from femtotron_b200.utils.flops import llama_flops_per_token
    return llama_flops_per_token(cfg, seq)


def peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except OSError:
        return {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0}


def progress(msg: str):
    """Rank-tagged, flushed progress line on stderr (every rank), so a stop is localised."""
    print(f"[bench r{os.environ.get('RANK', '0')} {time.strftime('%H:%M:%S')}] {msg}",
          file=sys.stderr, flush=True)


def emit(line: dict):
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- our arm
def build_ours(cfg, args, ctx, device):
    from femtotron_b200.models import build_llama_model, get_llama_parallel_plan, materialize_model
    from femtotron_b200.parallel.data_parallel import create_grad_synchronizer
    from femtotron_b200.sharding import ZeROConfig, create_sharding_strategy, llama_wrap_policy
    from femtotron_b200.training import (FusedAdamW, MixedPrecisionManager, TrainConfig,
                                         apply_activation_checkpointing, create_lr_schedule,
                                         get_param_groups)
    from femtotron_b200.training.ckpt_policy import by_class
    from femtotron_b200.models.layers import LlamaDecoderLayer
    torch.manual_seed(1234)
    model = build_llama_model(cfg, ctx, sequence_parallel=args.tp and ctx.tp_size > 1)
    materialize_model(model, device, dtype=torch.bfloat16, init_std=0.02)
    total_steps = args.warmup + 2 * args.steps + 10
    tc = TrainConfig(train_steps=total_steps, grad_accum_steps=args.grad_accum, grad_clip=None,
                     master_dtype=torch.float32, param_dtype=torch.bfloat16, log_interval=10 ** 9,
                     checkpoint_interval=10 ** 9, warmup_steps=2, lr=3e-4)
    zc = ZeROConfig(stage=0) if args.tp else ZeROConfig(stage=3, wrap_policy=llama_wrap_policy)
    strategy = create_sharding_strategy(ctx, zc)
    mp = MixedPrecisionManager(model, ctx, get_llama_parallel_plan(), tc, FusedAdamW,
                               dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-8),
                               get_param_groups(model, 0.01), sharding_strategy=strategy)
    if not args.tp:   # the ZeRO-3 config trains with full activation checkpointing
        apply_activation_checkpointing(model, by_class(LlamaDecoderLayer), use_reentrant=False,
                                       preserve_rng_state=False)
    sched = create_lr_schedule(mp.inner, tc.warmup_steps, total_steps, 0.1)
    gsync = create_grad_synchronizer(mp.groups, ctx, strategy)
    return model, mp, sched, gsync, tc


def run_ours(args):
    from collections import OrderedDict
    from femtotron_b200.data import DistributedDataLoader, SyntheticTokens, simple_pretrain_collator
    from femtotron_b200.ops import attention, ext
    from femtotron_b200.parallel_context import ParallelContext
    from femtotron_b200.training import Trainer
    from femtotron_b200.utils.clocks import ClockSampler
    from femtotron_b200.utils.dist import init_distributed, max_over_ranks

    rank, world, local = init_distributed("nccl", timeout_s=int(os.environ.get("FT_PG_TIMEOUT", "300")))
    device = torch.device("cuda", local)
    cfg = model_config(args.layers, args.config)
    ctx = ParallelContext(OrderedDict(tp=world) if args.tp else OrderedDict(dp=world))
    model, mp, sched, gsync, tc = build_ours(cfg, args, ctx, device)
    ga, mb, S = args.grad_accum, args.micro_batch, args.seq

    # ---- device-timed phase: micro-batches pre-staged on the device
    g = torch.Generator(device="cpu")
    g.manual_seed(1000 + ctx.dp_rank)   # tensor-parallel peers share their batch
    dev_batches = [torch.randint(0, cfg.vocab_size, (mb, S), generator=g).to(device) for _ in range(ga)]

    class DevIter:
        def __iter__(self):
            return self

        def __next__(self):
            self.i = getattr(self, "i", -1) + 1
            x = dev_batches[self.i % ga]
            return {"input_ids": x, "labels": x}

    class Null:
        micro_batch_size = mb
        dataset = None

        def set_epoch(self, e):
            pass

    trainer = Trainer(model, mp, sched, Null(), gsync, ctx, tc)
    mp.strategy.prepare_for_backward(mp.groups)
    it = DevIter()
    progress("ours: model built, starting warm-up")
    for i in range(args.warmup):
        info = trainer.train_step(it)
        progress(f"ours: warm-up step {i} {info['step_ms']:.0f} ms loss {info['loss']:.4f}")
    ext.check_kernel_errors(device)
    torch.cuda.synchronize()
    dist.barrier()
    progress("ours: timed region")
    l0 = ext.LAUNCHES[0]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    losses = []
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        dist.barrier()
        start.record()
        from femtotron_b200.utils.comm_timing import TIMER
        TIMER.collect()
        comm_tot: dict = {}
        for i in range(args.steps):
            info = trainer._train_one_step_standard(it)
            TIMER.mark("optimizer")
            trainer.grad_sync.sync_gradients()
            mp.step()
            sched.step()
            TIMER.mark(None)
            losses.append(info)
            if TIMER.enabled:  # diagnostic mode: syncs on the step's wait events
                for k, v in TIMER.collect().items():
                    comm_tot[k] = comm_tot.get(k, 0.0) + v
        end.record()
        torch.cuda.synchronize()
        dist.barrier()
    launches = ext.LAUNCHES[0] - l0
    dev_ms = start.elapsed_time(end)
    dev_ms = max_over_ranks(dev_ms)
    loss_last = float(losses[-1].item())
    ext.check_kernel_errors(device)
    ms_per_step = dev_ms / args.steps
    dp = ctx.dp_size
    tokens_per_step = ga * mb * S * dp
    value = tokens_per_step / (ms_per_step / 1e3)

    # ---- end-to-end phase through the public API (pinned host -> device, loss -> host)
    progress(f"ours: timed region done, {dev_ms / args.steps:.1f} ms/step")
    e2e = None
    if not args.no_e2e:
        ds = SyntheticTokens(num_samples=ga * mb * dp * (args.steps + 2), seq_len=S,
                             vocab_size=cfg.vocab_size, seed=7)
        dl = DistributedDataLoader(ds, ctx, mb, simple_pretrain_collator, num_workers=2, pin_memory=True)
        trainer.dataloader = dl
        dl.set_epoch(0)
        it2 = iter(dl)
        trainer.train_step(it2)  # warm the loader workers
        torch.cuda.synchronize()
        dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            trainer.train_step(it2)  # includes H2D of ids/labels and the loss .item()
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        dist.barrier()
        e2e_ms = max_over_ranks((t1 - t0) * 1e3) / args.steps
        progress(f"ours: end-to-end {e2e_ms:.1f} ms/step")
        e2e = {"value": tokens_per_step / (e2e_ms / 1e3), "unit": "tokens/s",
               "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": ga * mb * S * 8 * 2,   # input_ids + labels, int64
               "d2h_bytes_per_step": 4}                     # fp32 loss

    pk = peaks()
    mfu = value * flops_per_token(cfg, S) / (world * pk["bf16_tflops"] * 1e12)
    exposed = None
    if comm_tot:
        # compute-stream time blocked on communication, per step, max over ranks
        exposed = {k: round(max_over_ranks(v) / args.steps, 2) for k, v in sorted(comm_tot.items())}
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 2),
        "higher_is_better": True, "scaling": "strong" if args.tp else "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (uniform random token ids, random-init weights)",
        "config": {"model": args.model_name if not args.layers else f"{args.model_name}-{args.layers}L(debug)",
                   "global_batch": ga * mb * dp, "micro_batch": mb, "grad_accum": ga,
                   "seq_len": S,
                   "parallelism": f"tp{world}-sp" if args.tp else f"zero3-dp{world}",
                   "activation_checkpointing": "none" if args.tp else "full",
                   "optimizer": "AdamW fp32 master", "l2": "per-step working set (weights, optimizer state, activations) >> 126 MB L2 (no flush needed)"},
        "mfu": round(mfu, 4), "mfu_peak_tflops": pk["bf16_tflops"],
        "flops_per_token": flops_per_token(cfg, S),
        "loss_last": loss_last,
        "gpu_launches": launches,
        "sdpa_fallbacks": attention.SDPA_FALLBACKS[0],
        "impl": "ours",
        "clocks": clk.summary(),
    }
    if e2e is not None:
        line["e2e"] = e2e
    if exposed is not None:
        line["exposed_comm_ms_per_step"] = exposed
    emit(line)
    dist.barrier()
    dist.destroy_process_group()


# ----------------------------------------------------------------------------- reference arm
def run_reference(args):
    if args.config != "llama3-8b-zero3":
        emit({"impl": "reference", "unavailable": "the reference arm covers the headline configuration only"})
        return
    ref_root = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "femtotron")):
        # only rank 0 installs; the others wait for the package to appear
        if int(os.environ.get("LOCAL_RANK", "0")) == 0:
            sys.path.insert(0, os.path.join(HERE, "baseline"))
            try:
                import install_reference
                progress("reference: " + install_reference.install())
            except Exception as e:
                emit({"impl": "reference", "unavailable": f"reference install failed: {e!r}"[:300]})
                return
        else:
            t0 = time.time()
            while not os.path.isdir(os.path.join(ref_root, "femtotron", "training")) and time.time() - t0 < 600:
                time.sleep(2)
    sys.path.insert(0, ref_root)
    from collections import OrderedDict
    from femtotron_b200.utils.clocks import ClockSampler
    from femtotron_b200.utils.dist import init_distributed, max_over_ranks
    rank, world, local = init_distributed("nccl")
    device = torch.device("cuda", local)
    try:
        from femtotron.parallel_context import ParallelContext as RCtx
        from femtotron.model.llama import build_llama_model as rbuild
        from femtotron.model.parallel_plan import get_llama_parallel_plan as rplan
        from femtotron.training.train_config import TrainConfig as RTC
        from femtotron.training.optimizer import get_param_groups as rgroups
        from femtotron.training.mixed_precision_manager import MixedPrecisionManager as RMP
        from femtotron.training.lr_schedule import create_lr_schedule as rlr
        from femtotron.training.activation_ckpt import apply_activation_checkpointing as rac
        from femtotron.training.trainer import Trainer as RTrainer
        from femtotron.sharding.factory import create_sharding_strategy as rstrat
        from femtotron.sharding.zero_config import ZeROConfig as RZ
        from femtotron.scripts.presets import get_wrap_policy, get_ac_policy
        from femtotron.parallel.data_parallel.gradient_synchronizer import create_grad_synchronizer as rsync
        from femtotron.data.data_loader import DistributedDataLoader as RDL
        from femtotron.data.collator import simple_pretrain_collator as rcoll
    except Exception as e:  # pragma: no cover
        emit({"impl": "reference", "unavailable": f"reference import failed: {e!r}"[:300]})
        return
    cfg = model_config(args.layers)
    ga, mb, S = args.grad_accum, args.micro_batch, args.seq
    try:
        ctx = RCtx(OrderedDict([("pp", 1), ("dp", world), ("tp", 1)]))
        torch.manual_seed(1234)
        with torch.device("meta"):
            model = rbuild(cfg, ctx)
        model = model.to_empty(device=device)
        for p in model.parameters():
            torch.nn.init.normal_(p, mean=0.0, std=0.02)
        # the reference's own tests re-create rotary inv_freq after to_empty
        rot = model.model.rotary_emb
        dim = cfg.hidden_size // cfg.num_attention_heads
        theta = (getattr(cfg, "rope_parameters", None) or {}).get("rope_theta", 10000.0)
        inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.int64).to(
            device=device, dtype=torch.float) / dim))
        rot.inv_freq.copy_(inv)
        if hasattr(rot, "original_inv_freq"):
            rot.original_inv_freq.copy_(inv)
        model = model.bfloat16()
        total = args.warmup + 2 * args.steps + 10
        tc = RTC(master_dtype=torch.float32, grad_clip=None, train_steps=total, log_interval=10 ** 9,
                 checkpoint_interval=10 ** 9, warmup_steps=2, min_lr_ratio=0.1)
        tc.grad_accum_steps = ga
        strategy = rstrat(ctx, RZ(stage=3, wrap_policy=get_wrap_policy("llama_decoder_layer")))
        mp = RMP(model=model, sharding_strategy=strategy, parallel_ctx=ctx, parallel_plan=rplan(),
                 config=tc, inner_optimizer_cls=torch.optim.AdamW,
                 inner_optimizer_kwargs={"lr": 3e-4, "betas": (0.9, 0.95), "eps": 1e-8},
                 compute_param_groups=rgroups(model, weight_decay=0.01))
        rac(model, get_ac_policy("llama_decoder_layer"), use_reentrant=False, preserve_rng_state=False)
        sched = rlr(mp.inner, warmup_steps=2, total_steps=total, min_lr_ratio=0.1)
        g = torch.Generator()
        g.manual_seed(7)
        data = torch.randint(0, cfg.vocab_size, (ga * mb * world * (args.warmup + args.steps + 2), S), generator=g)
        dl = RDL(dataset=data, parallel_ctx=ctx, micro_batch_size=mb, collator=rcoll, num_workers=2)
        gs = rsync(mp.groups, ctx, strategy)
        trainer = RTrainer(model=model, mp_manager=mp, scheduler=sched, dataloader=dl, grad_sync=gs,
                           parallel_ctx=ctx, train_config=tc)
        mp.strategy.prepare_for_backward(mp.groups)
        dl.set_epoch(0)
        it = iter(dl)
        progress("reference: model built, starting warm-up")
        for i in range(args.warmup):
            t_s = time.perf_counter()
            trainer._train_one_step(it)
            progress(f"reference: warm-up step {i} {time.perf_counter() - t_s:.1f}s")
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            t0 = time.perf_counter()
            s.record()
            info = None
            for _ in range(args.steps):
                info = trainer._train_one_step(it)   # stock step: H2D, fwd/bwd, mp.step, loss.item()
            e.record()
            torch.cuda.synchronize()
            t1 = time.perf_counter()
            dist.barrier()
        ms = max_over_ranks(s.elapsed_time(e)) / args.steps
        wall = max_over_ranks((t1 - t0) * 1e3) / args.steps
    except torch.cuda.OutOfMemoryError as ex:
        emit({"impl": "reference", "unavailable": f"reference ran out of GPU memory on this config: {str(ex)[:160]}"})
        dist.destroy_process_group()
        return
    tokens = ga * mb * S * world
    value = tokens / (ms / 1e3)
    pk = peaks()
    emit({"metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
          "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2),
          "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
          "data": "synthetic (uniform random token ids, random-init weights)",
          "config": {"model": "Llama-3-8B" if not args.layers else f"Llama-3-8B-{args.layers}L(debug)",
                     "global_batch": ga * mb * world, "seq_len": S, "parallelism": f"zero3-dp{world}",
                     "activation_checkpointing": "full"},
          "mfu": round(value * flops_per_token(cfg, S) / (world * pk["bf16_tflops"] * 1e12), 4),
          "loss_last": info["loss"] if info else None,
          "e2e": {"value": tokens / (wall / 1e3), "unit": "tokens/s", "ms_per_step": wall,
                  "h2d_bytes_per_step": ga * mb * S * 8 * 2, "d2h_bytes_per_step": 4},
          "impl": "reference", "clocks": clk.summary()})
    dist.barrier()
    dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
