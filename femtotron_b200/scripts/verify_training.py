"""Check a trained checkpoint: greedy / temperature sampling and validation loss (reference
femtotron/scripts/verify_training.py:49-107).  Every TP rank computes the same logits; the
sampled token is taken from rank 0 and broadcast so all ranks stay in lock-step.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m femtotron_b200.scripts.verify_training \\
        --config configs/tiny_llama_debug.yaml --resume checkpoints/tiny_debug/step_10
"""
from __future__ import annotations

import sys

import torch
import torch.distributed as dist

from femtotron_b200.scripts.train import build_all, load_config, log, parse_args
from femtotron_b200.utils.dist import init_distributed


@torch.no_grad()
def generate(model, prompt_ids: torch.Tensor, max_new_tokens: int = 32, temperature: float = 0.0):
    ids = prompt_ids.clone()
    for _ in range(max_new_tokens):
        logits = model(ids)["logits"][:, -1, :].float()
        if temperature > 0:
            nxt = torch.multinomial(torch.softmax(logits / temperature, -1), 1)
        else:
            nxt = logits.argmax(-1, keepdim=True)
        if dist.is_initialized():
            dist.broadcast(nxt, src=0)
        ids = torch.cat([ids, nxt], 1)
    return ids


@torch.no_grad()
def compute_val_loss(model, data: torch.Tensor, device, num_batches: int = 8, batch_size: int = 4) -> float:
    tot, n = 0.0, 0
    for i in range(min(num_batches, data.shape[0] // batch_size)):
        x = data[i * batch_size:(i + 1) * batch_size].to(device)
        tot += model(x, labels=x)["loss"].item()
        n += 1
    return tot / max(n, 1)


def main(argv=None):
    args = parse_args(argv)
    cfg = load_config(args)
    init_distributed()
    trainer = build_all(cfg)
    if cfg.get("resume"):
        trainer._load_checkpoint(cfg["resume"])
    model = trainer.model
    model.eval()
    data = trainer.dataloader.dataset.data
    loss = compute_val_loss(model, data, trainer.device)
    log(f"validation loss: {loss:.4f}")
    out = generate(model, data[:1, :8].to(trainer.device), max_new_tokens=16)
    log(f"greedy continuation ids: {out[0].tolist()}")
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1:])
