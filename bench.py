"""Training-throughput benchmark of the BASELINE configurations (tokens/s for the whole job +
MFU), one process per GPU of one node; synthetic uniform token ids, random-init weights.

    python bench.py [--config NAME] [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Configurations (``--config``; the default is the headline):
  llama3-8b-zero3       Llama-3-8B, ZeRO-3 over all N GPUs, seq 4096, micro-batch 1, grad-accum
                        8, full activation checkpointing (weak scaling: fixed work per GPU)
  llama2-13b-tp-sp      Llama-2-13B, tensor parallel over all N GPUs with sequence parallelism,
                        DP=1, seq 4096, micro-batch 2 (strong scaling); the reference has no
                        sequence parallelism, so its arm runs plain tensor parallelism
  llama2-7b-3d          Llama-2-7B, TP=2 x PP=2 x DP=N/4 with ZeRO-1, 1F1B over 8 micro-batches
                        of 1 x seq 2048 (N a multiple of 4; weak scaling over DP)
  llama3-70b-tp4-zero3  Llama-3-70B, TP=4 x ZeRO-3 DP=N/4, seq 4096, micro-batch 1,
                        grad-accum 16, full activation checkpointing (N a multiple of 4)

Every configuration is built through the public training entry point
(``femtotron_b200.scripts.train.build_all`` with the YAML under configs/), bf16 compute with
fp32 master weights and AdamW.  Two measurements, each over K steps after W warm-up steps:
  * ``value``: device time (CUDA events on the compute stream, barrier + synchronize on both
    sides, max over ranks) of K optimizer steps whose micro-batches are already on the device;
  * ``e2e``: K steps through ``Trainer.train_step`` over the DistributedDataLoader: every step
    copies its token ids from pinned host memory to the device and reads the loss back to the
    host; host wall clock, max over ranks.
The per-step working set (weights, optimizer state, activations: tens of GB) exceeds the
126 MB L2 cache, so no explicit flush is needed between steps.

``--impl reference`` runs the unmodified reference (installed under baseline/_ref on first
use) through its own public API and stock training step on the same configuration and prints
the same JSON line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import sys
import time

import femtotron_b200  # noqa: F401  (sets the stream/queue environment before CUDA starts)
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
METRIC = "tokens/sec/box + MFU, Llama-3-8B ZeRO-3 & TP=8, 1/2/4/8 B200, max over ranks"


def _layout_dp(w):
    return 1, w, 1


def _layout_tp(w):
    return 1, 1, w


def _layout_3d(w):
    if w % 4:
        raise ValueError("llama2-7b-3d needs a multiple of 4 GPUs (TP=2 x PP=2 x DP)")
    return 2, w // 4, 2


def _layout_tp4(w):
    if w % 4:
        raise ValueError("llama3-70b-tp4-zero3 needs a multiple of 4 GPUs (TP=4 x DP)")
    return 1, w // 4, 4


# per configuration: YAML, model name, (pp, dp, tp) for N GPUs, and the scaling kind
CONFIGS = {
    "llama3-8b-zero3": dict(yaml="llama3_8b_zero3.yaml", name="Llama-3-8B", layout=_layout_dp,
                            scaling="weak"),
    "llama2-13b-tp-sp": dict(yaml="llama2_13b_tp8_sp.yaml", name="Llama-2-13B", layout=_layout_tp,
                             scaling="strong"),
    "llama2-7b-3d": dict(yaml="llama2_7b_3d.yaml", name="Llama-2-7B", layout=_layout_3d,
                         scaling="weak"),
    "llama3-70b-tp4-zero3": dict(yaml="llama3_70b_tp4_zero3.yaml", name="Llama-3-70B",
                                 layout=_layout_tp4, scaling="weak"),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="llama3-8b-zero3", choices=sorted(CONFIGS))
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
    return ap.parse_args()


def bench_cfg(args, world: int) -> dict:
    """The training configuration of the benchmark: the entry point's defaults <- the YAML of
    the configuration <- the benchmark's settings (layout for N GPUs, no clipping, synthetic
    data large enough for every step)."""
    import yaml
    from femtotron_b200.scripts.train import DEFAULTS
    c = CONFIGS[args.config]
    cfg = dict(DEFAULTS)
    with open(os.path.join(HERE, "configs", c["yaml"])) as f:
        cfg.update(yaml.safe_load(f) or {})
    pp, dp, tp = c["layout"](world)
    cfg.update(pp=pp, dp=dp, tp=tp)
    if args.seq:
        cfg["seq_len"] = args.seq
    if args.micro_batch:
        cfg["micro_batch_size"] = args.micro_batch
    if args.grad_accum:
        cfg["grad_accum_steps"] = args.grad_accum
    if args.layers:
        cfg["num_hidden_layers"] = args.layers
    cfg["max_position_embeddings"] = max(cfg["max_position_embeddings"], cfg["seq_len"])
    total = args.warmup + 2 * args.steps + 10
    rows = cfg["micro_batch_size"] * (cfg["num_microbatches"] if pp > 1 else 1)
    cfg.update(grad_clip=None, train_steps=total, warmup_steps=2, lr=3e-4, min_lr_ratio=0.1,
               log_interval=10 ** 9, checkpoint_interval=10 ** 9, synthetic_data=True,
               num_samples=cfg["grad_accum_steps"] * rows * dp * (args.steps + args.warmup + 4),
               init_std=0.02, seed=1234, metrics_path=None, ac_preserve_rng_state=False,
               _explicit=set())
    cfg["_rows"] = rows
    return cfg


def model_config(cfg):
    from femtotron_b200.scripts.train import model_config_from
    mc = model_config_from(cfg)
    mc.use_cache = False
    return mc


def flops_per_token(mc, seq) -> float:
    """Model FLOPs per trained token: 6 x (matmul parameters) + 6 x L x H x S for causal
    attention (score and value products, forward+backward).  Recomputation is not counted."""
    from femtotron_b200.utils.flops import llama_flops_per_token
    return llama_flops_per_token(mc, seq)


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


def describe(args, cfg) -> dict:
    pp, dp, tp = cfg["pp"], cfg["dp"], cfg["tp"]
    c = CONFIGS[args.config]
    par = f"zero{cfg['zero_stage']}-dp{dp}"
    if tp > 1:
        par = f"tp{tp}" + ("-sp" if cfg.get("sequence_parallel") else "") + (f"-{par}" if dp > 1 else "")
    if pp > 1:
        par = f"pp{pp}-{cfg['schedule']}-{par}"
    model = c["name"] if not args.layers else f"{c['name']}-{args.layers}L(debug)"
    return {"model": model, "global_batch": cfg["grad_accum_steps"] * cfg["_rows"] * dp,
            "micro_batch": cfg["micro_batch_size"], "grad_accum": cfg["grad_accum_steps"],
            "pipeline_microbatches": cfg["num_microbatches"] if pp > 1 else None,
            "seq_len": cfg["seq_len"], "parallelism": par,
            "activation_checkpointing": "full" if cfg["ac_enabled"] else "none",
            "optimizer": "AdamW fp32 master",
            "l2": "per-step working set (weights, optimizer state, activations) >> 126 MB L2 (no flush needed)"}


# ----------------------------------------------------------------------------- our arm
def run_ours(args):
    from femtotron_b200.ops import attention, ext
    from femtotron_b200.scripts.train import build_all
    from femtotron_b200.utils.clocks import ClockSampler
    from femtotron_b200.utils.comm_timing import TIMER
    from femtotron_b200.utils.dist import init_distributed, max_over_ranks

    rank, world, local = init_distributed("nccl", timeout_s=int(os.environ.get("FT_PG_TIMEOUT", "300")))
    device = torch.device("cuda", local)
    cfg = bench_cfg(args, world)
    mc = model_config(cfg)
    progress(f"ours: building {args.config} pp={cfg['pp']} dp={cfg['dp']} tp={cfg['tp']}")
    with contextlib.redirect_stdout(sys.stderr):   # stdout carries only the JSON line
        trainer = build_all(cfg)
    mp, sched = trainer.mp_manager, trainer.scheduler
    ctx = trainer.parallel_ctx
    ga, rows, S, dp = cfg["grad_accum_steps"], cfg["_rows"], cfg["seq_len"], cfg["dp"]

    # ---- device-timed phase: the step's micro-batches pre-staged on the device
    g = torch.Generator(device="cpu")
    g.manual_seed(1000 + ctx.dp_rank)   # tensor- and pipeline-parallel peers share their batch
    dev_batches = [torch.randint(0, mc.vocab_size, (rows, S), generator=g).to(device) for _ in range(ga)]

    class DevIter:
        i = -1

        def __iter__(self):
            return self

        def __next__(self):
            self.i += 1
            x = dev_batches[self.i % ga]
            return {"input_ids": x, "labels": x}

    def device_step(it):
        if trainer.pp_runner is None:
            loss = trainer._train_one_step_standard(it)
        else:
            loss = trainer._train_one_step_pp(it)
        TIMER.mark("optimizer")
        trainer.grad_sync.sync_gradients()
        mp.step()
        sched.step()
        TIMER.mark(None)
        return loss

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
    comm_tot: dict = {}
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        dist.barrier()
        TIMER.collect()
        start.record()
        for i in range(args.steps):
            losses.append(device_step(it))
            if TIMER.enabled:  # diagnostic mode: syncs on the step's wait events
                for k, v in TIMER.collect().items():
                    comm_tot[k] = comm_tot.get(k, 0.0) + v
        end.record()
        torch.cuda.synchronize()
        dist.barrier()
    launches = ext.LAUNCHES[0] - l0
    dev_ms = max_over_ranks(start.elapsed_time(end))
    loss_last = float(losses[-1].item())
    ext.check_kernel_errors(device)
    ms_per_step = dev_ms / args.steps
    tokens_per_step = ga * rows * S * dp
    value = tokens_per_step / (ms_per_step / 1e3)
    progress(f"ours: timed region done, {ms_per_step:.1f} ms/step")

    # ---- end-to-end phase through the public API (pinned host -> device, loss -> host)
    e2e = None
    if not args.no_e2e:
        trainer.dataloader.set_epoch(0)
        it2 = iter(trainer.dataloader)
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
               # input_ids + labels (int64) of this rank's micro-batches; the fp32 loss back
               "h2d_bytes_per_step": ga * rows * S * 8 * 2,
               "d2h_bytes_per_step": 4}

    pk = peaks()
    mfu = value * flops_per_token(mc, S) / (world * pk["bf16_tflops"] * 1e12)
    exposed = None
    if comm_tot:
        # compute-stream time blocked on communication, and per-phase device time, per step,
        # max over ranks
        exposed = {k: round(max_over_ranks(v) / args.steps, 2) for k, v in sorted(comm_tot.items())}
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 2),
        "higher_is_better": True, "scaling": CONFIGS[args.config]["scaling"], "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (uniform random token ids, random-init weights)",
        "config": describe(args, cfg),
        "mfu": round(mfu, 4), "mfu_peak_tflops": pk["bf16_tflops"],
        "flops_per_token": flops_per_token(mc, S),
        "loss_last": loss_last,
        "gpu_launches": launches,
        "sdpa_fallbacks": attention.SDPA_FALLBACKS[0],
        "peak_mem_gb": round(max_over_ranks(torch.cuda.max_memory_allocated(device) / 2 ** 30), 1),
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
def _install_reference(ref_root: str) -> str | None:
    """Returns None when the reference is importable from ref_root, else the reason."""
    if os.path.isdir(os.path.join(ref_root, "femtotron", "training")):
        return None
    # only one process installs; the others wait for the package to appear
    if int(os.environ.get("LOCAL_RANK", "0")) == 0:
        sys.path.insert(0, os.path.join(HERE, "baseline"))
        try:
            import install_reference
            progress("reference: " + install_reference.install())
        except Exception as e:
            return f"reference install failed: {e!r}"[:300]
        finally:
            sys.path.pop(0)
    else:
        t0 = time.time()
        while not os.path.isdir(os.path.join(ref_root, "femtotron", "training")) and time.time() - t0 < 600:
            time.sleep(2)
    return None if os.path.isdir(os.path.join(ref_root, "femtotron", "training")) else \
        "reference not installed under baseline/_ref"


def run_reference(args):
    ref_root = os.path.join(HERE, "baseline", "_ref")
    why = _install_reference(ref_root)
    if why is not None:
        emit({"impl": "reference", "unavailable": why})
        return
    sys.path.insert(0, ref_root)
    from collections import OrderedDict
    from femtotron_b200.utils.clocks import ClockSampler
    from femtotron_b200.utils.dist import init_distributed, max_over_ranks
    rank, world, local = init_distributed("nccl", timeout_s=int(os.environ.get("FT_PG_TIMEOUT", "600")))
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
        from femtotron.parallel.pipeline_parallel.comm_ops import PipelineComm as RComm
        from femtotron.parallel.pipeline_parallel.runner import PipelineRunner as RRunner
        from femtotron.parallel.pipeline_parallel.stage import PipelineStage as RStage
        from femtotron.parallel.pipeline_parallel.partition import partition_layers as rpart
        from femtotron.parallel.pipeline_parallel.pipeline_config import PipelineConfig as RPC
        from femtotron.data.data_loader import DistributedDataLoader as RDL
        from femtotron.data.collator import simple_pretrain_collator as rcoll
    except Exception as e:  # pragma: no cover
        emit({"impl": "reference", "unavailable": f"reference import failed: {e!r}"[:300]})
        return
    cfg = bench_cfg(args, world)
    mc = model_config(cfg)
    pp, dp, tp = cfg["pp"], cfg["dp"], cfg["tp"]
    ga, rows, S, mb = cfg["grad_accum_steps"], cfg["_rows"], cfg["seq_len"], cfg["micro_batch_size"]
    nmb = cfg["num_microbatches"] if pp > 1 else 1
    try:
        ctx = RCtx(OrderedDict([("pp", pp), ("dp", dp), ("tp", tp)]))
        torch.manual_seed(1234)
        layer_range = None
        if pp > 1:
            part = rpart(mc.num_hidden_layers, pp, strategy="uniform")[ctx.pp_rank]
            layer_range = range(part[0], part[-1] + 1)
        with torch.device("meta"):
            model = rbuild(mc, ctx, use_pp_aware=pp > 1, layer_range=layer_range)
        model = model.to_empty(device=device)
        for p in model.parameters():
            torch.nn.init.normal_(p, mean=0.0, std=0.02)
        # the reference's own tests re-create rotary inv_freq after to_empty (its random-init
        # path leaves it uninitialised)
        rot = model.model.rotary_emb
        dim = mc.hidden_size // mc.num_attention_heads
        theta = (getattr(mc, "rope_parameters", None) or {}).get("rope_theta", cfg["rope_theta"])
        inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.int64).to(
            device=device, dtype=torch.float) / dim))
        rot.inv_freq.copy_(inv)
        if hasattr(rot, "original_inv_freq"):
            rot.original_inv_freq.copy_(inv)
        model = model.bfloat16()
        total = cfg["train_steps"]
        tc = RTC(master_dtype=torch.float32, grad_clip=None, train_steps=total, log_interval=10 ** 9,
                 checkpoint_interval=10 ** 9, warmup_steps=2, min_lr_ratio=0.1,
                 pipeline_config=RPC(num_microbatches=nmb, schedule=cfg["schedule"]))
        tc.grad_accum_steps = ga
        wrap = get_wrap_policy("llama_decoder_layer") if cfg["zero_stage"] == 3 else None
        strategy = rstrat(ctx, RZ(stage=cfg["zero_stage"], wrap_policy=wrap))
        mp = RMP(model=model, sharding_strategy=strategy, parallel_ctx=ctx, parallel_plan=rplan(),
                 config=tc, inner_optimizer_cls=torch.optim.AdamW,
                 inner_optimizer_kwargs={"lr": 3e-4, "betas": (0.9, 0.95), "eps": 1e-8},
                 compute_param_groups=rgroups(model, weight_decay=0.01))
        if cfg["ac_enabled"]:
            rac(model, get_ac_policy("llama_decoder_layer"), use_reentrant=False, preserve_rng_state=False)
        sched = rlr(mp.inner, warmup_steps=2, total_steps=total, min_lr_ratio=0.1)
        runner = None
        if pp > 1:
            stage = RStage(model, ctx, loss_scale=1.0 / (ga * nmb))
            comm = RComm(ctx, seqlen=S, hidden_size=mc.hidden_size, dtype=torch.bfloat16)
            runner = RRunner(stage, comm, schedule_name=cfg["schedule"], num_microbatches=nmb,
                             recv_shape=(mb, S, mc.hidden_size), recv_dtype=torch.bfloat16)
        g = torch.Generator()
        g.manual_seed(7)
        data = torch.randint(0, mc.vocab_size, (ga * rows * dp * (args.warmup + args.steps + 2), S), generator=g)
        dl = RDL(dataset=data, parallel_ctx=ctx, micro_batch_size=rows, collator=rcoll, num_workers=2)
        gs = rsync(mp.groups, ctx, strategy)
        trainer = RTrainer(model=model, mp_manager=mp, scheduler=sched, dataloader=dl, grad_sync=gs,
                           parallel_ctx=ctx, train_config=tc, pp_runner=runner)
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
    tokens = ga * rows * S * dp
    value = tokens / (ms / 1e3)
    pk = peaks()
    desc = describe(args, cfg)
    if cfg.get("sequence_parallel"):
        desc["parallelism"] = desc["parallelism"].replace("-sp", "") + " (reference: no sequence parallelism)"
    emit({"metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
          "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2),
          "higher_is_better": True, "scaling": CONFIGS[args.config]["scaling"], "vs_baseline": None,
          "dtype": "bf16", "data": "synthetic (uniform random token ids, random-init weights)",
          "config": desc,
          "mfu": round(value * flops_per_token(mc, S) / (world * pk["bf16_tflops"] * 1e12), 4),
          "loss_last": info["loss"] if info else None,
          "e2e": {"value": tokens / (wall / 1e3), "unit": "tokens/s", "ms_per_step": wall,
                  "h2d_bytes_per_step": ga * rows * S * 8 * 2, "d2h_bytes_per_step": 4},
          "peak_mem_gb": round(max_over_ranks(torch.cuda.max_memory_allocated(device) / 2 ** 30), 1),
          "impl": "reference", "clocks": clk.summary(),
          **({"notes": "the reference's activation checkpointing calls torch checkpoint with "
                       "debug=True (femtotron/training/activation_ckpt.py:84), which records "
                       "every op with its tracebacks; its step is host-bound"}
             if cfg["ac_enabled"] else {})})
    dist.barrier()
    dist.destroy_process_group()


def main():
    args = parse()
    if not torch.cuda.is_available():
        emit({"impl": args.impl, "unavailable": "no CUDA device: the benchmark runs on B200 GPUs"})
        sys.exit(0 if args.impl == "reference" else 1)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
