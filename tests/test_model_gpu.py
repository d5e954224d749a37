"""End-to-end numerics of the LLaMA model on the GPU kernels against the same model in fp32
PyTorch math on the CPU (same weights), and a short ZeRO-3 training run on one GPU."""
import pytest
import torch
from transformers import LlamaConfig

from femtotron_b200.models import LlamaForTraining, materialize_model
from femtotron_b200.ops.ext import check_kernel_errors

pytestmark = pytest.mark.gpu


def _cfg(layers=2):
    return LlamaConfig(hidden_size=256, intermediate_size=768, num_attention_heads=4,
                       num_key_value_heads=2, num_hidden_layers=layers, vocab_size=2048,
                       max_position_embeddings=512, rms_norm_eps=1e-5, rope_theta=10000.0)


def rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def test_model_fwd_bwd_matches_fp32_cpu():
    torch.manual_seed(0)
    cfg = _cfg()
    with torch.device("meta"):
        ref = LlamaForTraining(cfg)
    # HF-style init (norm weights 1, matrices N(0, 0.02)): well-conditioned gradients
    init = lambda n, p: p.fill_(1.0) if p.dim() == 1 else p.normal_(0, 0.02)
    materialize_model(ref, "cpu", dtype=torch.float32, init_fn=init)
    with torch.device("meta"):
        gpu = LlamaForTraining(cfg)
    materialize_model(gpu, "cuda", dtype=torch.bfloat16, init_std=None)
    with torch.no_grad():
        for pg, pr in zip(gpu.parameters(), ref.parameters()):
            pg.copy_(pr.to(torch.bfloat16))
            pr.copy_(pg.float().cpu())   # both see the same bf16-representable weights
    ids = torch.randint(0, cfg.vocab_size, (2, 128))
    lr_ = ref(ids, labels=ids)["loss"]
    lr_.backward()
    lg = gpu(ids.cuda(), labels=ids.cuda())["loss"]
    lg.backward()
    torch.cuda.synchronize()
    check_kernel_errors()
    assert abs(lg.item() - lr_.item()) < 2e-2 * abs(lr_.item())
    for (n, pg), pr in zip(gpu.named_parameters(), ref.parameters()):
        assert rel(pg.grad.cpu(), pr.grad) < 5e-2, n


def test_zero3_training_runs_on_gpu():
    import os
    from collections import OrderedDict
    import torch.distributed as dist
    from femtotron_b200.utils.dist import init_distributed
    from femtotron_b200.parallel_context import ParallelContext
    from femtotron_b200.models import build_llama_model, get_llama_parallel_plan
    from femtotron_b200.training import (FusedAdamW, MixedPrecisionManager, TrainConfig, Trainer,
                                         apply_activation_checkpointing, create_lr_schedule,
                                         get_param_groups)
    from femtotron_b200.training.ckpt_policy import by_class
    from femtotron_b200.models.layers import LlamaDecoderLayer
    from femtotron_b200.sharding import ZeROConfig, create_sharding_strategy, llama_wrap_policy
    from femtotron_b200.parallel.data_parallel import create_grad_synchronizer
    from femtotron_b200.data import DistributedDataLoader, SyntheticTokens, simple_pretrain_collator
    init_distributed("nccl")
    ctx = ParallelContext(OrderedDict(dp=1))
    cfg = _cfg(layers=3)
    torch.manual_seed(0)
    m = build_llama_model(cfg, ctx)
    materialize_model(m, "cuda", dtype=torch.bfloat16)
    tc = TrainConfig(train_steps=6, grad_accum_steps=2, master_dtype=torch.float32, log_interval=3)
    st = create_sharding_strategy(ctx, ZeROConfig(stage=3, wrap_policy=llama_wrap_policy))
    mp = MixedPrecisionManager(m, ctx, get_llama_parallel_plan(), tc, FusedAdamW,
                               dict(lr=2e-3, betas=(0.9, 0.95), eps=1e-8), get_param_groups(m, 0.01),
                               sharding_strategy=st)
    apply_activation_checkpointing(m, by_class(LlamaDecoderLayer))
    sch = create_lr_schedule(mp.inner, 1, 6)
    ds = SyntheticTokens(64, 128, cfg.vocab_size, seed=1)
    # a learnable signal: repeat each sample's first half so the loss can drop
    ds.data[:, 64:] = ds.data[:, :64]
    dl = DistributedDataLoader(ds, ctx, 4, simple_pretrain_collator, num_workers=0)
    tr = Trainer(m, mp, sch, dl, create_grad_synchronizer(mp.groups, ctx, st), ctx, tc)
    hist = tr.train()
    check_kernel_errors()
    losses = [h["loss"] for h in hist]
    assert all(l == l for l in losses)
    assert losses[-1] < losses[0]
