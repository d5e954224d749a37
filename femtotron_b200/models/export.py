"""Consolidate a Trainer checkpoint into one unsharded Hugging Face model.

A checkpoint directory ``step_N/`` holds one ``shard_tp{t}_dp{d}[_pp{p}].pt`` per rank.  The
fp32 master weights inside them are reassembled per parameter:

* replicated masters (ZeRO-0, and ZeRO-3's free parameters) are taken as they are;
* ZeRO-1/2 masters are flat DP shards of the padded parameter: concatenated over the DP ranks
  and cut back to the parameter's size;
* ZeRO-3 cluster masters are flat DP shards of a whole decoder layer: concatenated over the
  DP ranks and split in the layer's parameter order;

then TP slices are concatenated along the dimension the parallel plan split (column and
vocabulary: rows; row-parallel: columns).  Checkpoints without masters fall back to the
compute parameters of the model state dict.  Shapes come from the model configuration,
which the checkpoint does not store, so the caller passes it.

``export_hf`` writes ``config.json`` + ``model.safetensors`` that
``transformers.LlamaForCausalLM.from_pretrained`` and this package's ``ModelLoader`` read.
The reference has no exporter (it only loads Hugging Face weights,
femtotron/model/model_loader.py:28-104).
"""
from __future__ import annotations

import glob
import json
import os
import re

import torch

from .parallel_plan import get_llama_parallel_plan


def _full_shapes(model_config) -> dict[str, torch.Size]:
    from .llama import LlamaForTraining
    with torch.device("meta"):
        m = LlamaForTraining(model_config)
    return {n: p.shape for n, p in m.named_parameters()}


def _split_dim(plan, name: str):
    """Dimension the TP plan splits parameter `name` along (None: replicated)."""
    rule = plan.get_rule(name.rsplit(".", 1)[0])
    if rule is None or rule.parallel_type == "replicate":
        return None
    if rule.parallel_type in ("column", "vocab_embed"):
        return 0
    if rule.parallel_type == "row":
        return None if name.endswith(".bias") else 1
    raise ValueError(f"unknown parallel type {rule.parallel_type!r} for {name}")


def _local_shape(full: torch.Size, dim, tp: int) -> torch.Size:
    if dim is None:
        return full
    s = list(full)
    if s[dim] % tp:
        raise ValueError(f"dim {dim} of {tuple(full)} not divisible by tp={tp}")
    s[dim] //= tp
    return torch.Size(s)


def consolidate_checkpoint(ckpt_dir: str, model_config) -> dict[str, torch.Tensor]:
    """Full fp32 state dict (Hugging Face parameter names) of the model in `ckpt_dir`."""
    with open(os.path.join(ckpt_dir, "meta.json")) as f:
        meta = json.load(f)
    tp, dp, pp = meta["tp_size"], meta["dp_size"], meta.get("pp_size", 1)
    pat = re.compile(r"shard_tp(\d+)_dp(\d+)(?:_pp(\d+))?\.pt$")
    files = {}
    for fn in glob.glob(os.path.join(ckpt_dir, "shard_tp*_dp*.pt")):
        m = pat.search(os.path.basename(fn))
        if m:
            files[(int(m.group(1)), int(m.group(2)), int(m.group(3) or 0))] = fn
    need = {(t, d, p) for t in range(tp) for d in range(dp) for p in range(pp)}
    if set(files) != need:
        raise FileNotFoundError(f"{ckpt_dir}: expected {len(need)} shard files, found {len(files)}")
    plan = get_llama_parallel_plan()
    shapes = _full_shapes(model_config)
    dims = {n: _split_dim(plan, n) for n in shapes}
    local_shapes = {n: _local_shape(s, dims[n], tp) for n, s in shapes.items()}
    per_tp: list[dict[str, torch.Tensor]] = [{} for _ in range(tp)]
    for t in range(tp):
        for p in range(pp):
            sds = [torch.load(files[(t, d, p)], map_location="cpu", weights_only=False) for d in range(dp)]
            opt = [s["optimizer"] for s in sds]
            got = per_tp[t]
            mw0 = opt[0].get("master_weights", {})
            specs = opt[0].get("master_specs", {})
            for name in mw0:
                ls = local_shapes[name]
                if name in specs:   # DP-sharded flat master (ZeRO-1/2)
                    flat = torch.cat([o["master_weights"][name].reshape(-1) for o in opt])
                    got[name] = flat[:ls.numel()].reshape(ls).float()
                else:
                    got[name] = mw0[name].reshape(ls).float()
            for cname, c0 in opt[0].get("cluster_masters", {}).items():
                parts = sorted((o["cluster_masters"][cname] for o in opt), key=lambda c: c["dp_rank"])
                flat = torch.cat([c["master"].reshape(-1) for c in parts])
                off = 0
                for name in c0["names"]:
                    n = local_shapes[name].numel()
                    got[name] = flat[off:off + n].reshape(local_shapes[name]).float()
                    off += n
            for name, v in sds[0]["model"].items():   # no masters: compute parameters
                key = name.replace("._checkpoint_wrapped_module", "")
                if key in local_shapes and key not in got and v.numel() == local_shapes[key].numel():
                    got[key] = v.reshape(local_shapes[key]).float()
    out = {}
    for name, full in shapes.items():
        parts = [per_tp[t].get(name) for t in range(tp)]
        if any(x is None for x in parts):
            raise KeyError(f"{name}: not found in every TP rank's shards")
        out[name] = parts[0] if dims[name] is None else torch.cat(parts, dim=dims[name])
        if out[name].shape != full:
            raise ValueError(f"{name}: consolidated {tuple(out[name].shape)} != {tuple(full)}")
    return out


def export_hf(ckpt_dir: str, model_config, out_dir: str, dtype: torch.dtype = torch.bfloat16) -> str:
    """Write `ckpt_dir`'s model as a Hugging Face directory (config.json + model.safetensors)."""
    from safetensors.torch import save_file
    sd = consolidate_checkpoint(ckpt_dir, model_config)
    os.makedirs(out_dir, exist_ok=True)
    save_file({k: v.to(dtype).contiguous() for k, v in sd.items()},
              os.path.join(out_dir, "model.safetensors"), metadata={"format": "pt"})
    model_config.save_pretrained(out_dir)
    return out_dir
