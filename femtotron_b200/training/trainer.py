"""Training-loop orchestrator (reference femtotron/training/trainer.py:30-415).

One optimizer step = ``grad_accum_steps`` micro-batches (forward + backward, gradient sync
deferred with ``no_sync`` on all but the last) or one pipeline-runner step, then gradient
synchronisation, ``MixedPrecisionManager.step()`` and the LR scheduler.

Additions over the reference:
  * step time measured with CUDA events and reduced as the max over ranks at log steps
    (``step_ms_max``), tokens/s for the whole job (host clock and device clock), MFU, the
    compute stream's time blocked on communication (FT_COMM_TIMING=1), peak memory, and JSONL
    metrics (``TrainConfig.metrics_path``);
  * the loss stays on the device until the end of the step (one device->host read);
  * optional NaN/Inf abort, kernel bounded-wait error check at log intervals;
  * checkpoints keep the reference layout (``step_N/meta.json``, ``shard_tp{t}_dp{d}.pt``,
    ``dataloader_dp{d}.pt``, ``_SUCCESS``) and add ``_pp{p}`` to the shard name when pp>1 so
    stages no longer overwrite each other; every rank restores the data-loader state.
"""
from __future__ import annotations

import json
import os
import random
import time
from contextlib import nullcontext

import numpy as np
import torch
import torch.distributed as dist


def _rank() -> int:
    return dist.get_rank() if dist.is_available() and dist.is_initialized() else 0


def _barrier():
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


class Trainer:
    def __init__(self, model, mp_manager, scheduler, dataloader, grad_sync, parallel_ctx,
                 train_config, pp_runner=None, *, check_finite: bool = False):
        self.model = model
        self.mp_manager = mp_manager
        self.scheduler = scheduler
        self.dataloader = dataloader
        self.parallel_ctx = parallel_ctx
        self.grad_sync = grad_sync
        self.train_config = train_config
        self.pp_runner = pp_runner
        self.check_finite = check_finite
        self.global_step = 0
        self.epoch = 0
        self._resumed_mid_epoch = False
        self.history: list[dict] = []
        self._last_log_time = None
        self._last_log_step = None
        if torch.cuda.is_available():
            self.device = torch.device("cuda", torch.cuda.current_device())
        else:
            self.device = torch.device("cpu")

    # ------------------------------------------------------------------ loop
    def train(self):
        self.mp_manager.strategy.prepare_for_backward(self.mp_manager.groups)
        while self.global_step < self.train_config.train_steps:
            if self._resumed_mid_epoch:
                # keep the sampler offset restored from the checkpoint (set_epoch would
                # rewind to the start of the epoch and replay samples)
                self._resumed_mid_epoch = False
            else:
                self.dataloader.set_epoch(self.epoch)
            it = iter(self.dataloader)
            while self.global_step < self.train_config.train_steps:
                try:
                    info = self.train_step(it)
                except StopIteration:
                    break
                self.global_step += 1
                self.history.append(info)
                if self.global_step % self.train_config.log_interval == 0:
                    self._log_step(info)
                if self.global_step % self.train_config.checkpoint_interval == 0:
                    self._save_checkpoint()
            self.epoch += 1
        return self.history

    def train_step(self, data_iter) -> dict:
        """One optimizer step; returns {loss, lr, successful, step_ms, grad_norm?}."""
        # idempotent: registers the strategy's backward hooks (ZeRO-2) on first use, so a
        # caller driving train_step directly gets the same gradients as train()
        self.mp_manager.strategy.prepare_for_backward(self.mp_manager.groups)
        timed = self.device.type == "cuda"
        if timed:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
        t0 = time.perf_counter()
        if self.pp_runner is None:
            loss = self._train_one_step_standard(data_iter)
        else:
            loss = self._train_one_step_pp(data_iter)
        if self.check_finite and not torch.isfinite(loss).item():
            raise FloatingPointError(f"non-finite loss at step {self.global_step}")
        self.grad_sync.sync_gradients()
        ok = self.mp_manager.step()
        self.scheduler.step()
        loss_val = float(loss.item())
        if timed:
            ev1.record()
            ev1.synchronize()
            ms = ev0.elapsed_time(ev1)
        else:
            ms = (time.perf_counter() - t0) * 1e3
        info = {"step": self.global_step + 1, "loss": loss_val,
                "lr": self.scheduler.get_last_lr()[0], "successful": ok, "step_ms": ms}
        for tr in self.mp_manager.grad_transforms:
            norm = getattr(tr, "last_norm", None)
            if norm is not None:
                info["grad_norm"] = float(norm.item())
        return info

    def _batch_to_device(self, batch):
        return {k: v.to(self.device, non_blocking=True) for k, v in batch.items()}

    def _train_one_step_standard(self, data_iter) -> torch.Tensor:
        from femtotron_b200.utils.comm_timing import TIMER
        n = self.train_config.grad_accum_steps
        total = torch.zeros((), device=self.device)
        for micro in range(n):
            batch = self._batch_to_device(next(data_iter))
            last = micro == n - 1
            ctx = self.mp_manager.final_backward() if last else self.grad_sync.no_sync()
            with ctx:
                TIMER.mark("fwd_last" if last else "fwd")
                out = self.model(input_ids=batch["input_ids"], labels=batch["labels"])
                loss = out["loss"] / n
                TIMER.mark("bwd_last" if last else "bwd")
                loss.backward()
                TIMER.mark(None)
                total += loss.detach().float() * n
            self.mp_manager.accumulate_grads() if self.train_config.grad_acc_dtype is not None else None
        return total / n

    def _train_one_step_pp(self, data_iter) -> torch.Tensor:
        n = self.train_config.grad_accum_steps
        ctx = self.parallel_ctx
        total = torch.zeros((), device=self.device)
        for micro in range(n):
            batch = self._batch_to_device(next(data_iter))
            sctx = nullcontext() if micro == n - 1 else self.grad_sync.no_sync()
            with sctx:
                losses = self.pp_runner.run_step(batch)
                if self.pp_runner.is_last_stage:
                    total += (sum(losses.values()) * n).detach().float()
        if ctx.pp_size > 1:
            last = ctx.get_ranks_in_group("pp")[-1]
            dist.broadcast(total, src=last, group=ctx.pp_group)
        return total / n

    # ------------------------------------------------------------------ logging
    def _reduce_max(self, values: list[float]) -> list[float]:
        """Element-wise max over all ranks (every rank calls this at the same steps)."""
        if not (dist.is_available() and dist.is_initialized()):
            return values
        dev = self.device if dist.get_backend() == "nccl" else torch.device("cpu")
        t = torch.tensor(values, dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    def _log_step(self, info: dict):
        """Called on every rank at log intervals: reduces the step time (and, with
        FT_COMM_TIMING=1, the compute stream's time blocked on communication) as the max over
        ranks, checks the native kernels' status words, then rank 0 prints and appends the
        JSONL record."""
        from femtotron_b200.utils.comm_timing import TIMER
        from femtotron_b200.utils.flops import B200_BF16_DENSE_TFLOPS, llama_flops_per_token
        blocked = None
        if TIMER.enabled and self.device.type == "cuda":
            waits = {k: v for k, v in TIMER.collect().items() if not k.startswith("phase:")}
            blocked = sum(waits.values())
        step_ms, blocked_max = self._reduce_max([info["step_ms"], blocked or 0.0])
        if self.device.type == "cuda":
            from femtotron_b200.ops.ext import check_kernel_errors
            check_kernel_errors(self.device)
        if _rank() != 0:
            return
        now = time.perf_counter()
        tok = self.tokens_per_step()
        if self._last_log_time is not None:
            tps = tok * (self.global_step - self._last_log_step) / (now - self._last_log_time)
        else:       # first record: no earlier wall-clock mark, use the step's own time
            tps = tok / (step_ms / 1e3) if step_ms > 0 else 0.0
        self._last_log_time, self._last_log_step = now, self.global_step
        mem = torch.cuda.max_memory_allocated() / 2 ** 30 if self.device.type == "cuda" else 0.0
        rec = dict(info, step_ms_max=step_ms, tokens_per_s=tps, peak_mem_gb=mem, time=time.time())
        if tok and step_ms > 0:
            rec["tokens_per_s_device"] = tok / (step_ms / 1e3)
            cfg = getattr(self.model, "config", None)
            seq = self._seq_len()
            if cfg is not None and seq:
                peak = self.train_config.peak_tflops or B200_BF16_DENSE_TFLOPS
                world = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
                rec["mfu"] = rec["tokens_per_s_device"] * llama_flops_per_token(cfg, seq) / (world * peak * 1e12)
                rec["mfu_peak_tflops"] = peak
        if blocked is not None:
            rec["comm_blocked_ms_max"] = blocked_max
            rec["comm_blocked_frac"] = blocked_max / step_ms if step_ms > 0 else float("nan")
        msg = (f"step {self.global_step:>6}/{self.train_config.train_steps} | loss {info['loss']:7.4f} | "
               f"lr {info['lr']:.2e} | tok/s {tps:>9.0f} | step {step_ms:.1f} ms | mem {mem:.1f}GB")
        if "mfu" in rec:
            msg += f" | mfu {rec['mfu']:.3f}"
        if "grad_norm" in info:
            msg += f" | gnorm {info['grad_norm']:.3f}"
        print(msg, flush=True)
        path = getattr(self.train_config, "metrics_path", None)
        if path:
            with open(path, "a") as f:
                f.write(json.dumps(rec) + "\n")

    def _seq_len(self) -> int:
        ds = getattr(self.dataloader, "dataset", None)
        return int(ds.shape[1]) if ds is not None and hasattr(ds, "shape") else 0

    def tokens_per_step(self) -> int:
        return (self.dataloader.micro_batch_size * self._seq_len() * self.train_config.grad_accum_steps
                * self.parallel_ctx.dp_size)

    # ------------------------------------------------------------------ checkpoints
    def _shard_name(self) -> str:
        c = self.parallel_ctx
        base = f"shard_tp{c.tp_rank}_dp{c.dp_rank}"
        return base + (f"_pp{c.pp_rank}" if c.pp_size > 1 else "") + ".pt"

    def _save_checkpoint(self):
        d = os.path.join(self.train_config.checkpoint_dir, f"step_{self.global_step}")
        c = self.parallel_ctx
        _barrier()
        if _rank() == 0:
            os.makedirs(d, exist_ok=True)
            meta = {"step": self.global_step, "epoch": self.epoch, "tp_size": c.tp_size,
                    "dp_size": c.dp_size, "pp_size": c.pp_size,
                    "config": {k: str(v) for k, v in self.train_config.__dict__.items()}}
            with open(os.path.join(d, "meta.json"), "w") as f:
                json.dump(meta, f, indent=2, default=str)
        _barrier()
        torch.save({"model": self.model.state_dict(), "optimizer": self.mp_manager.state_dict(),
                    "scheduler": self.scheduler.state_dict(), "rng": self._rng_state_dict()},
                   os.path.join(d, self._shard_name()))
        if c.tp_rank == 0 and (c.pp_size == 1 or c.pp_rank == 0):
            torch.save(self.dataloader.state_dict(), os.path.join(d, f"dataloader_dp{c.dp_rank}.pt"))
        _barrier()
        if _rank() == 0:
            with open(os.path.join(d, "_SUCCESS"), "w") as f:
                f.write("ok")
            print(f"Saved checkpoint to {d}", flush=True)
        return d

    def _load_checkpoint(self, ckpt_dir: str):
        c = self.parallel_ctx
        if not os.path.isfile(os.path.join(ckpt_dir, "_SUCCESS")):
            raise RuntimeError(f"checkpoint at {ckpt_dir} is incomplete (missing _SUCCESS marker)")
        with open(os.path.join(ckpt_dir, "meta.json")) as f:
            meta = json.load(f)
        if meta["tp_size"] != c.tp_size:
            raise RuntimeError(f"tp_size mismatch: ckpt={meta['tp_size']}, current={c.tp_size}")
        if meta["dp_size"] != c.dp_size:
            raise RuntimeError(f"dp_size mismatch: ckpt={meta['dp_size']}, current={c.dp_size}")
        if meta.get("pp_size", 1) != c.pp_size:
            raise RuntimeError(f"pp_size mismatch: ckpt={meta.get('pp_size', 1)}, current={c.pp_size}")
        shard = torch.load(os.path.join(ckpt_dir, self._shard_name()), map_location=self.device,
                           weights_only=False)
        self.model.load_state_dict(shard["model"], strict=False)
        self.mp_manager.load_state_dict(shard["optimizer"])
        self.scheduler.load_state_dict(shard["scheduler"])
        self._load_rng_state(shard["rng"])
        dl = os.path.join(ckpt_dir, f"dataloader_dp{c.dp_rank}.pt")
        if os.path.isfile(dl):
            self.dataloader.load_state_dict(torch.load(dl, weights_only=False))
            self._resumed_mid_epoch = True
        self.global_step = meta["step"]
        self.epoch = meta["epoch"]
        if _rank() == 0:
            print(f"Resumed from {ckpt_dir} at step {self.global_step}", flush=True)

    def _rng_state_dict(self) -> dict:
        st = {"torch": torch.get_rng_state(), "numpy": np.random.get_state(), "python": random.getstate()}
        if torch.cuda.is_available():
            st["cuda"] = torch.cuda.get_rng_state()
        return st

    def _load_rng_state(self, st: dict):
        torch.set_rng_state(st["torch"].cpu() if hasattr(st["torch"], "cpu") else st["torch"])
        if "cuda" in st and torch.cuda.is_available():
            torch.cuda.set_rng_state(st["cuda"].cpu())
        np.random.set_state(st["numpy"])
        random.setstate(st["python"])
