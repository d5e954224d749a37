from .layers import (LlamaAttention, LlamaDecoderLayer, LlamaMLP, LlamaRMSNorm,
                     LlamaRotaryEmbedding)
from .llama import LlamaForTraining, build_llama_model
from .llama_causal import LlamaForCausalLM
from .llama_partial_model import LlamaPartialModel
from .materialize import materialize_model
from .parallel_plan import ParallelPlan, ParallelRule, get_llama_parallel_plan
from .parallelize_model import parallelize_model

__all__ = [
    "LlamaAttention", "LlamaDecoderLayer", "LlamaMLP", "LlamaRMSNorm", "LlamaRotaryEmbedding",
    "LlamaForTraining", "LlamaForCausalLM", "LlamaPartialModel", "build_llama_model",
    "materialize_model", "ParallelPlan", "ParallelRule", "get_llama_parallel_plan",
    "parallelize_model",
]
