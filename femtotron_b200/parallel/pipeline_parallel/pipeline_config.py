"""Pipeline settings (reference: femtotron/parallel/pipeline_parallel/pipeline_config.py:8)."""
from __future__ import annotations

from dataclasses import dataclass


@dataclass
class PipelineConfig:
    num_microbatches: int = 1
    schedule: str = "1f1b"   # "gpipe" | "1f1b"
