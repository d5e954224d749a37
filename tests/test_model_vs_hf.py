"""The LLaMA model of this package against transformers' LlamaForCausalLM (the layer the
reference wraps) in fp32 on CPU: identical parameter names, loss and gradients."""
import torch
from transformers import LlamaConfig
from transformers import LlamaForCausalLM as HFLlama

from femtotron_b200.models import LlamaForCausalLM, LlamaForTraining, materialize_model


def _cfg(**kw):
    base = dict(hidden_size=256, intermediate_size=688, num_attention_heads=8, num_key_value_heads=4,
                num_hidden_layers=2, vocab_size=2048, max_position_embeddings=512, rms_norm_eps=1e-5,
                attn_implementation="sdpa")
    base.update(kw)
    return LlamaConfig(**base)


def _compare(cfg, ours_cls):
    torch.manual_seed(0)
    hf = HFLlama(cfg).float()
    with torch.device("meta"):
        m = ours_cls(cfg)
    materialize_model(m, "cpu", dtype=torch.float32, init_std=None)
    m.load_state_dict(hf.state_dict(), strict=True)
    ids = torch.randint(0, cfg.vocab_size, (2, 64))
    lh = hf(ids, labels=ids).loss
    lm = m(ids, labels=ids)["loss"]
    assert abs(lh.item() - lm.item()) < 1e-5
    lh.backward()
    lm.backward()
    hp = dict(hf.named_parameters())
    for n, p in m.named_parameters():
        g1, g2 = p.grad, hp[n].grad
        assert ((g1 - g2).norm() / g2.norm()).item() < 1e-4, n


def test_llama_for_training_matches_hf():
    _compare(_cfg(), LlamaForTraining)


def test_llama_causal_matches_hf_mha_theta():
    _compare(_cfg(num_key_value_heads=8, rope_theta=500000.0), LlamaForCausalLM)


def test_logits_materialized_without_labels():
    torch.manual_seed(0)
    cfg = _cfg()
    hf = HFLlama(cfg).float()
    with torch.device("meta"):
        m = LlamaForTraining(cfg)
    materialize_model(m, "cpu", dtype=torch.float32, init_std=None)
    m.load_state_dict(hf.state_dict())
    ids = torch.randint(0, cfg.vocab_size, (2, 32))
    with torch.no_grad():
        a = hf(ids).logits
        b = m(ids)["logits"]
    assert torch.allclose(a, b, atol=1e-4, rtol=1e-4)
