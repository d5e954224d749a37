"""Training configuration (field names of the reference femtotron/training/train_config.py:8-48)."""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from femtotron_b200.parallel.pipeline_parallel.pipeline_config import PipelineConfig
from femtotron_b200.sharding.zero_config import ZeROConfig


@dataclass
class TrainConfig:
    train_steps: int = 0
    grad_accum_steps: int = 1
    grad_clip: float | None = 1.0
    log_interval: int = 10
    checkpoint_interval: int = 1000
    checkpoint_dir: str = "checkpoints"
    eval_interval: int | None = None

    param_dtype: torch.dtype = torch.bfloat16
    master_dtype: torch.dtype | None = None
    grad_acc_dtype: torch.dtype | None = None
    reduce_dtype: torch.dtype | None = None

    ZeRO_config: ZeROConfig = field(default_factory=ZeROConfig)
    pipeline_config: PipelineConfig = field(default_factory=PipelineConfig)

    use_loss_scaler: bool = False
    initial_scale: float = 2.0 ** 16

    optimizer: str = "adamw"
    lr: float = 1e-4
    warmup_steps: int = 50
    min_lr_ratio: float = 0.1
    metrics_path: str | None = None      # JSONL metrics per logged step (rank 0)
    peak_tflops: float | None = None     # per-GPU bf16 peak for MFU (None: B200 dense 2250)
