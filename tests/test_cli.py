"""The YAML + command-line training entry point on CPU gloo ranks (TP=2, ZeRO-3 and a 1F1B
pipeline), plus the checkpoint it writes and the verification script reading it back."""
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(args, tmp_path, nproc=2, module="femtotron_b200.scripts.train"):
    from dist_helpers import free_port
    env = dict(os.environ, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", str(nproc),
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()), "-m", module] + args
    return subprocess.run(cmd, cwd=str(tmp_path), env=env, capture_output=True, text=True, timeout=600)


def test_cli_tp2_then_verify(tmp_path):
    cfg = os.path.join(ROOT, "configs", "tiny_llama_debug.yaml")
    common = ["--config", cfg, "--num_hidden_layers", "2", "--seq_len", "64", "--micro_batch_size", "2",
              "--checkpoint_dir", str(tmp_path / "ck")]
    metrics = tmp_path / "metrics.jsonl"
    out = _run(common + ["--train_steps", "4", "--checkpoint_interval", "4", "--zero_stage", "3",
                         "--log_interval", "2", "--metrics_path", str(metrics)], tmp_path)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-3000:]
    assert "step      4/4" in out.stdout
    import json
    recs = [json.loads(l) for l in metrics.read_text().splitlines()]
    assert [r["step"] for r in recs] == [2, 4]
    for key in ("loss", "lr", "step_ms_max", "tokens_per_s_device", "mfu", "peak_mem_gb"):
        assert key in recs[-1], (key, recs[-1])
    assert recs[-1]["step_ms_max"] >= recs[-1]["step_ms"] > 0
    assert os.path.isfile(tmp_path / "ck" / "step_4" / "_SUCCESS")
    out = _run(common + ["--zero_stage", "3", "--resume", str(tmp_path / "ck" / "step_4")], tmp_path,
               module="femtotron_b200.scripts.verify_training")
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-3000:]
    assert "validation loss" in out.stdout


def test_cli_pipeline_1f1b(tmp_path):
    cfg = os.path.join(ROOT, "configs", "tiny_llama_debug.yaml")
    out = _run(["--config", cfg, "--tp", "1", "--pp", "2", "--num_microbatches", "2", "--num_hidden_layers", "2",
                "--seq_len", "32", "--micro_batch_size", "2", "--train_steps", "3", "--zero_stage", "1"], tmp_path)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-3000:]
    assert "step      3/3" in out.stdout


def test_cli_trains_on_a_local_corpus(tmp_path):
    """The non-synthetic data path end to end without network: a local .jsonl corpus, the
    byte tokenizer, rank-0 preprocessing into data_dir, then TP=2 training on the packed rows."""
    import json
    corpus = tmp_path / "corpus.jsonl"
    corpus.write_text("\n".join(json.dumps({"text": f"document {i}: the quick brown fox jumps over the lazy dog"})
                                for i in range(60)) + "\n")
    cfg = os.path.join(ROOT, "configs", "tiny_llama_debug.yaml")
    out = _run(["--config", cfg, "--num_hidden_layers", "2", "--seq_len", "64", "--micro_batch_size", "2",
                "--train_steps", "3", "--synthetic_data", "false", "--dataset", str(corpus),
                "--tokenizer", "bytes", "--data_dir", str(tmp_path / "data"), "--num_samples", "60"], tmp_path)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-3000:]
    assert "step      3/3" in out.stdout
    assert any(f.endswith("_seq64.pt") for f in os.listdir(tmp_path / "data"))


def test_cli_starts_from_a_local_hf_checkpoint(tmp_path):
    """--model_name pointing at a local Hugging Face directory (config.json + safetensors):
    the config comes from it and every TP rank loads its weight slices with ModelLoader."""
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM
    hf_dir = tmp_path / "hf"
    cfg = LlamaConfig(hidden_size=64, intermediate_size=160, num_attention_heads=4, num_key_value_heads=2,
                      num_hidden_layers=2, vocab_size=512, max_position_embeddings=256)
    torch.manual_seed(0)
    LlamaForCausalLM(cfg).save_pretrained(str(hf_dir), safe_serialization=True)
    out = _run(["--model_name", str(hf_dir), "--tp", "2", "--seq_len", "32", "--micro_batch_size", "2",
                "--train_steps", "2", "--warmup_steps", "1", "--log_interval", "1", "--synthetic_data", "true"],
               tmp_path)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-3000:]
    assert "step      2/2" in out.stdout


def test_cli_sequence_parallel_with_clipping_and_accumulation(tmp_path):
    """TP=2 with sequence parallelism, gradient clipping and gradient accumulation through the
    command line (the reference's script ignores grad_accum_steps and never clips)."""
    cfg = os.path.join(ROOT, "configs", "tiny_llama_debug.yaml")
    out = _run(["--config", cfg, "--tp", "2", "--sequence_parallel", "true", "--num_hidden_layers", "2",
                "--seq_len", "64", "--micro_batch_size", "2", "--grad_accum_steps", "2", "--grad_clip", "1.0",
                "--train_steps", "3", "--zero_stage", "1"], tmp_path)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-3000:]
    assert "step      3/3" in out.stdout and "gnorm" in out.stdout


def _losses(stdout: str) -> dict:
    out = {}
    for line in stdout.splitlines():
        if line.startswith("step") and "| loss" in line:
            step = int(line.split("/")[0].split()[-1])
            out[step] = float(line.split("| loss")[1].split("|")[0])
    return out


def test_cli_pipeline_checkpoint_resume(tmp_path):
    """PP=2 (1F1B) checkpoints carry a _pp<p> suffix per stage; resuming from step 2 reproduces
    the uninterrupted run's losses for steps 3-4."""
    cfg = os.path.join(ROOT, "configs", "tiny_llama_debug.yaml")
    common = ["--config", cfg, "--tp", "1", "--pp", "2", "--num_microbatches", "2", "--num_hidden_layers", "2",
              "--seq_len", "32", "--micro_batch_size", "2", "--train_steps", "4", "--zero_stage", "1",
              "--warmup_steps", "1", "--log_interval", "1", "--checkpoint_dir", str(tmp_path / "ck")]
    full = _run(common + ["--checkpoint_interval", "2"], tmp_path)
    assert full.returncode == 0, full.stdout[-2000:] + full.stderr[-3000:]
    names = sorted(os.listdir(tmp_path / "ck" / "step_2"))
    assert "shard_tp0_dp0_pp0.pt" in names and "shard_tp0_dp0_pp1.pt" in names, names
    resumed = _run(common + ["--checkpoint_interval", "1000", "--resume", str(tmp_path / "ck" / "step_2")],
                   tmp_path)
    assert resumed.returncode == 0, resumed.stdout[-2000:] + resumed.stderr[-3000:]
    a, b = _losses(full.stdout), _losses(resumed.stdout)
    assert set(b) >= {3, 4}, resumed.stdout[-1500:]
    for s in (3, 4):
        assert abs(a[s] - b[s]) < 1e-4, (s, a, b)
    # the per-stage shards also consolidate into one Hugging Face model
    from transformers import LlamaForCausalLM
    from femtotron_b200.scripts import export_hf
    out = export_hf.main(["--checkpoint", str(tmp_path / "ck" / "step_2"), "--out", str(tmp_path / "hf"),
                          "--config", cfg, "--num_hidden_layers", "2"])
    hf = LlamaForCausalLM.from_pretrained(out)
    assert hf.config.num_hidden_layers == 2 and len(hf.model.layers) == 2


def test_cli_runs_the_references_own_yaml(tmp_path):
    """A reference user's config file works unchanged (its dataset and tokenizer need the
    network, so synthetic tokens are switched on from the command line, as a bare flag)."""
    import pytest
    sys.path.insert(0, os.path.join(ROOT, "baseline"))
    import install_reference
    ref_yaml = os.path.join(install_reference.DEFAULT_SOURCE, "tiny_llama_debug.yaml")
    if not os.path.isfile(ref_yaml):
        pytest.skip("the reference's YAML is not on this machine")
    out = _run(["--config", ref_yaml, "--train_steps", "2", "--warmup_steps", "1", "--log_interval", "1",
                "--num_hidden_layers", "2", "--synthetic_data", "--checkpoint_dir", str(tmp_path / "ck")],
               tmp_path)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-3000:]
    assert "tp=2" in out.stdout and "step      2/2" in out.stdout
