"""Load HF-format safetensors checkpoints straight into a (TP-sharded, possibly PP-partial)
model (reference femtotron/model/model_loader.py:28-148).

Each rank opens the checkpoint files itself and reads only its slice of every tensor through
``safe_open(...).get_slice`` directly onto its device; the slicing rule comes from the
parallel plan (column / row / vocab / replicate).  Non-persistent buffers need no
re-initialisation here: the rotary tables of this package's model are computed from the
config on demand.
"""
from __future__ import annotations

import json
import os

import torch
import torch.distributed as dist
from torch import nn

from .parallel_plan import get_llama_parallel_plan
from .shard_loader import resolve_loader


def _module_name(param_name: str) -> str:
    return param_name.rsplit(".", 1)[0] if "." in param_name else param_name


def shard_for_rank(full: torch.Tensor, name: str, plan, rank: int, world: int) -> torch.Tensor:
    """This rank's TP slice of a full tensor named `name` (in-memory counterpart of the
    safetensors path)."""
    rule = plan.get_rule(_module_name(name)) if world > 1 else None
    return resolve_loader(rule, name).load(full, rank, world)


def load_one_param(f, name: str, rule, rank: int, world_size: int) -> torch.Tensor:
    """This rank's slice of tensor `name` from an open safetensors handle `f` (``safe_open``),
    sliced by `rule` (column / row / vocab / replicate; None = replicate)."""
    return resolve_loader(rule, name).load(f.get_slice(name), rank, world_size)


class ModelLoader:
    def __init__(self, parallel_ctx):
        self.parallel_ctx = parallel_ctx

    def _files(self, path: str) -> dict[str, str]:
        """Map tensor name -> file for a directory (index json or single file) or a file."""
        if os.path.isfile(path):
            from safetensors import safe_open
            with safe_open(path, framework="pt") as f:
                return {k: path for k in f.keys()}
        idx = os.path.join(path, "model.safetensors.index.json")
        if os.path.isfile(idx):
            with open(idx) as f:
                wm = json.load(f)["weight_map"]
            return {k: os.path.join(path, v) for k, v in wm.items()}
        single = os.path.join(path, "model.safetensors")
        if os.path.isfile(single):
            return self._files(single)
        raise FileNotFoundError(f"no safetensors checkpoint under {path}")

    @torch.no_grad()
    def load_and_distribute(self, model: nn.Module, model_name_or_path: str, parallel_plan=None,
                            device=None, strict: bool = True) -> nn.Module:
        from safetensors import safe_open
        plan = parallel_plan or get_llama_parallel_plan()
        ctx = self.parallel_ctx
        rank, world = ctx.tp_rank, ctx.tp_size
        device = torch.device(device) if device is not None else ctx.device
        files = self._files(model_name_or_path)
        by_file: dict[str, list[tuple[str, torch.Tensor]]] = {}
        missing = []
        for name, p in model.named_parameters():
            key = name.replace("._checkpoint_wrapped_module", "")
            if key not in files:
                missing.append(key)
                continue
            by_file.setdefault(files[key], []).append((key, p))
        if missing and strict:
            raise KeyError(f"{len(missing)} parameters missing from the checkpoint, e.g. {missing[:3]}")
        for fname, items in by_file.items():
            with safe_open(fname, framework="pt", device=str(device)) as f:
                for key, p in items:
                    rule = plan.get_rule(_module_name(key)) if world > 1 else None
                    t = load_one_param(f, key, rule, rank, world)
                    if tuple(t.shape) != tuple(p.shape):
                        raise ValueError(f"{key}: checkpoint slice {tuple(t.shape)} != parameter {tuple(p.shape)}")
                    if p.device.type == "meta":
                        raise ValueError("materialize the model before loading weights")
                    p.copy_(t.to(p.dtype))
        if dist.is_available() and dist.is_initialized():
            dist.barrier()
        return model
