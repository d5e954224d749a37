"""Export a Trainer checkpoint as a Hugging Face model directory.

    python -m femtotron_b200.scripts.export_hf --checkpoint checkpoints/step_1000 \\
        --config configs/llama3_8b_zero3.yaml --out exported/ [--dtype bf16|fp32]

The model shape comes from the same YAML / command-line keys as ``train.py`` (or
``--model_name``); the checkpoint's TP / PP / ZeRO shards are consolidated from their fp32
master weights (``femtotron_b200.models.export``).  Runs in one process, without GPUs.
"""
from __future__ import annotations

import argparse
import sys

import torch


def main(argv=None) -> str:
    from femtotron_b200.models.export import export_hf
    from femtotron_b200.scripts.train import load_config, model_config_from, parse_args
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--checkpoint", required=True, help="a step_N directory written by the Trainer")
    ap.add_argument("--out", required=True)
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "fp32"])
    args, rest = ap.parse_known_args(argv)
    cfg = load_config(parse_args(rest))
    mc = model_config_from(cfg)
    out = export_hf(args.checkpoint, mc, args.out,
                    dtype=torch.bfloat16 if args.dtype == "bf16" else torch.float32)
    print(f"[femtotron_b200] exported {args.checkpoint} -> {out}", flush=True)
    return out


if __name__ == "__main__":
    main(sys.argv[1:])
