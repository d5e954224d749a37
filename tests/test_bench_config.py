"""CPU checks of the benchmark's configurations: every ``bench.py --config`` builds the model
shape, parallel layout and training settings that the benchmark names (Llama-3-8B ZeRO-3,
Llama-2-13B TP+SP, Llama-2-7B TP2 x PP2 x DP, Llama-3-70B TP4 x ZeRO-3), and its FLOPs per
token, used for MFU, equal a count written out from the layer shapes."""
from __future__ import annotations

import argparse
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("ft_bench", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def args_for(config, **kw):
    a = dict(config=config, gpus=1, steps=5, warmup=3, impl="ours", seq=None, micro_batch=None,
             grad_accum=None, layers=None, no_e2e=False)
    a.update(kw)
    return argparse.Namespace(**a)


SHAPES = {
    # hidden, ffn, heads, kv heads, layers, vocab, rope theta
    "llama3-8b-zero3": (4096, 14336, 32, 8, 32, 128256, 500000.0),
    "llama2-13b-tp-sp": (5120, 13824, 40, 40, 40, 32000, 10000.0),
    "llama2-7b-3d": (4096, 11008, 32, 32, 32, 32000, 10000.0),
    "llama3-70b-tp4-zero3": (8192, 28672, 64, 8, 80, 128256, 500000.0),
}


@pytest.mark.parametrize("config", sorted(SHAPES))
def test_model_shape(bench, config):
    cfg = bench.bench_cfg(args_for(config), 8)
    mc = bench.model_config(cfg)
    h, f, nh, nkv, L, V, theta = SHAPES[config]
    assert (mc.hidden_size, mc.intermediate_size, mc.num_attention_heads,
            mc.num_key_value_heads, mc.num_hidden_layers, mc.vocab_size) == (h, f, nh, nkv, L, V)
    rope = getattr(mc, "rope_parameters", None) or {}
    assert rope.get("rope_theta", getattr(mc, "rope_theta", None)) == theta
    assert not mc.tie_word_embeddings
    assert mc.rms_norm_eps == 1e-5


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_headline_zero3_layout(bench, world):
    cfg = bench.bench_cfg(args_for("llama3-8b-zero3"), world)
    assert (cfg["pp"], cfg["dp"], cfg["tp"]) == (1, world, 1)
    assert cfg["zero_stage"] == 3 and cfg["ac_enabled"]
    assert (cfg["seq_len"], cfg["micro_batch_size"], cfg["grad_accum_steps"]) == (4096, 1, 8)
    d = bench.describe(args_for("llama3-8b-zero3"), cfg)
    assert d["model"] == "Llama-3-8B" and d["global_batch"] == 8 * world
    assert d["parallelism"] == f"zero3-dp{world}" and d["activation_checkpointing"] == "full"
    # every timed and warm-up step has its own samples
    assert cfg["num_samples"] >= 8 * world * (5 + 3)


def test_tp_sp_layout(bench):
    cfg = bench.bench_cfg(args_for("llama2-13b-tp-sp"), 8)
    assert (cfg["pp"], cfg["dp"], cfg["tp"]) == (1, 1, 8)
    assert cfg["sequence_parallel"] and cfg["zero_stage"] == 0
    assert (cfg["seq_len"], cfg["micro_batch_size"]) == (4096, 2)
    assert bench.describe(args_for("llama2-13b-tp-sp"), cfg)["parallelism"] == "tp8-sp"
    assert bench.CONFIGS["llama2-13b-tp-sp"]["scaling"] == "strong"


def test_3d_layout(bench):
    cfg = bench.bench_cfg(args_for("llama2-7b-3d"), 8)
    assert (cfg["pp"], cfg["dp"], cfg["tp"]) == (2, 2, 2)
    assert cfg["zero_stage"] == 1 and cfg["schedule"] == "1f1b"
    assert (cfg["num_microbatches"], cfg["micro_batch_size"], cfg["seq_len"]) == (8, 1, 2048)
    d = bench.describe(args_for("llama2-7b-3d"), cfg)
    assert d["parallelism"] == "pp2-1f1b-tp2-zero1-dp2"
    assert d["pipeline_microbatches"] == 8 and d["global_batch"] == 8 * 2
    with pytest.raises(ValueError):
        bench.bench_cfg(args_for("llama2-7b-3d"), 2)


def test_70b_layout(bench):
    cfg = bench.bench_cfg(args_for("llama3-70b-tp4-zero3"), 8)
    assert (cfg["pp"], cfg["dp"], cfg["tp"]) == (1, 2, 4)
    assert cfg["zero_stage"] == 3 and cfg["ac_enabled"] and cfg["sequence_parallel"]
    assert (cfg["seq_len"], cfg["micro_batch_size"], cfg["grad_accum_steps"]) == (4096, 1, 16)
    with pytest.raises(ValueError):
        bench.bench_cfg(args_for("llama3-70b-tp4-zero3"), 6)


def test_benchmark_settings_are_not_reduced(bench):
    """Only explicit debug flags change the shape; the defaults are the named configuration."""
    cfg = bench.bench_cfg(args_for("llama3-8b-zero3"), 1)
    assert cfg["grad_clip"] is None and cfg["synthetic_data"]
    d = bench.describe(args_for("llama3-8b-zero3", layers=2), bench.bench_cfg(
        args_for("llama3-8b-zero3", layers=2), 1))
    assert "debug" in d["model"]


def test_flops_per_token_llama3_8b(bench):
    cfg = bench.bench_cfg(args_for("llama3-8b-zero3"), 1)
    mc = bench.model_config(cfg)
    h, f, kv = 4096, 14336, 1024
    per_layer = (h * h) + 2 * (h * kv) + (h * h) + 3 * (h * f)      # q, k, v, o, gate, up, down
    n = 32 * per_layer + 128256 * h                                     # + LM head
    attn = 6 * 32 * h * 4096                                            # causal S and PV, fwd+bwd
    assert bench.flops_per_token(mc, 4096) == pytest.approx(6 * n + attn, rel=1e-12)
    assert 6 * n + attn == pytest.approx(48.2e9, rel=5e-3)
