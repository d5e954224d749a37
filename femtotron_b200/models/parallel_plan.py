"""Tensor-parallel plans: suffix-matched module names -> parallel rule.

Same matching semantics as the reference (femtotron/model/parallel_plan.py:3-118): rules
are tried in order and the first suffix match wins; unmatched modules are replicated.
``get_llama_parallel_plan(sequence_parallel=True)`` adds Megatron sequence parallelism to
the column/row/embedding rules, and ``lm_head`` stays vocab-sharded (its loss is computed
with the vocab-parallel cross-entropy, so full-vocab logits are never gathered).
"""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class ParallelRule:
    parallel_type: str                      # "column" | "row" | "vocab_embed" | "replicate"
    kwargs: dict = field(default_factory=dict)


class ParallelPlan:
    def __init__(self, rules: dict[str, ParallelRule]):
        self.rules = rules

    def get_rule(self, param_name: str) -> ParallelRule | None:
        for pattern, rule in self.rules.items():
            if param_name.endswith(pattern):
                return rule
        return None


def get_llama_parallel_plan(sequence_parallel: bool = False) -> ParallelPlan:
    sp = {"sequence_parallel": True} if sequence_parallel else {}
    rules = [
        ("model.embed_tokens", ParallelRule("vocab_embed", dict(sp))),
        ("self_attn.q_proj", ParallelRule("column", {"gather_output": False, **sp})),
        ("self_attn.k_proj", ParallelRule("column", {"gather_output": False, **sp})),
        ("self_attn.v_proj", ParallelRule("column", {"gather_output": False, **sp})),
        ("self_attn.o_proj", ParallelRule("row", {"scatter_input": False, **sp})),
        ("mlp.gate_proj", ParallelRule("column", {"gather_output": False, **sp})),
        ("mlp.up_proj", ParallelRule("column", {"gather_output": False, **sp})),
        ("mlp.down_proj", ParallelRule("row", {"scatter_input": False, **sp})),
        ("lm_head", ParallelRule("column", {"gather_output": True})),
    ]
    return ParallelPlan(dict(rules))
