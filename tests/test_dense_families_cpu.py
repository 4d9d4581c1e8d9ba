"""Dense decoder families beyond Qwen / Llama on CPU: Granite (embedding /
residual / attention / logits multipliers) and Phi-3 (fused qkv_proj and
gate_up_proj, LongRoPE short factors with the attention factor, partial
RoPE); the decoder oracle against transformers."""
import math

import pytest
import torch

from rlx_models_b200.config import DecoderConfig
from rlx_models_b200.models.oracle import DecoderOracle


def _rand(m):
    torch.manual_seed(0)
    with torch.no_grad():
        for _, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
    return m.eval()


def _check(m, cfg, n=41):
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    ids = torch.randint(0, cfg.vocab_size, (n,), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = m(ids[None]).logits[0].float()
    got, _ = DecoderOracle(cfg, sd).forward(ids)
    err = (got - ref).abs().max() / ref.abs().max()
    assert err < 1e-4, err


def test_granite_matches_transformers():
    from transformers import GraniteConfig, GraniteForCausalLM
    hc = GraniteConfig(vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                       num_attention_heads=4, num_key_value_heads=2, embedding_multiplier=12.0,
                       residual_multiplier=0.22, attention_multiplier=0.0078125, logits_scaling=8.0,
                       tie_word_embeddings=True, rms_norm_eps=1e-5)
    m = _rand(GraniteForCausalLM(hc))
    cfg = DecoderConfig.from_hf_dict(hc.to_dict())
    assert cfg.model_type == "granite" and cfg.residual_multiplier == 0.22 and cfg.logits_scaling == 8.0
    _check(m, cfg)


@pytest.mark.parametrize("partial", [1.0, 0.75])
def test_phi3_longrope_matches_transformers(partial):
    from transformers import Phi3Config, Phi3ForCausalLM
    D = 32
    rot = int(D * partial)
    g = torch.Generator().manual_seed(3)
    short = (1.0 + torch.rand(rot // 2, generator=g) * 2).tolist()
    long = (2.0 + torch.rand(rot // 2, generator=g) * 8).tolist()
    rp = {"rope_type": "longrope", "short_factor": short, "long_factor": long,
          "original_max_position_embeddings": 64, "rope_theta": 10000.0, "partial_rotary_factor": partial}
    hc = Phi3Config(vocab_size=128, hidden_size=128, intermediate_size=128, num_hidden_layers=2,
                    num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256,
                    original_max_position_embeddings=64, rope_parameters=rp, partial_rotary_factor=partial,
                    rms_norm_eps=1e-5, pad_token_id=0, tie_word_embeddings=False)
    m = _rand(Phi3ForCausalLM(hc))
    sd = m.state_dict()
    assert any(k.endswith("qkv_proj.weight") for k in sd) and any(k.endswith("gate_up_proj.weight") for k in sd)
    cfg = DecoderConfig.from_hf_dict(hc.to_dict())
    assert cfg.model_type == "phi3" and cfg.rotary_dim == rot
    assert cfg.rope_scaling["rope_type"] == "longrope"
    _check(m, cfg, n=50)  # below original_max_position_embeddings: the short factors


def _gemma_rand(m):
    torch.manual_seed(0)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
            else:  # (1 + w) norms: perturb around zero
                p.normal_(0, 0.2)
    return m.eval()


@pytest.mark.parametrize("family", ["gemma", "gemma2", "gemma3_text"])
def test_gemma_family_matches_transformers(family):
    """GeGLU, (1 + w) norms, sqrt(H) embedding scale, and for Gemma-2 / 3 the
    sandwich norms, query_pre_attn_scalar, sliding-window layers (window 8 <
    sequence), Gemma-2 attention / final logit softcapping, Gemma-3 QK-norm and
    the local RoPE base of sliding layers."""
    import transformers as tf
    common = dict(vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=4, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=32, rms_norm_eps=1e-6)
    if family == "gemma":
        hc = tf.GemmaConfig(**common, hidden_act="gelu_pytorch_tanh")
        m = tf.GemmaForCausalLM(hc)
    elif family == "gemma2":
        hc = tf.Gemma2Config(**common, sliding_window=8, query_pre_attn_scalar=24, attn_logit_softcapping=5.0,
                             final_logit_softcapping=3.0)
        m = tf.Gemma2ForCausalLM(hc)
    else:
        hc = tf.Gemma3TextConfig(**common, sliding_window=8, query_pre_attn_scalar=24,
                                 layer_types=["sliding_attention", "sliding_attention", "sliding_attention",
                                              "full_attention"],
                                 rope_parameters={"sliding_attention": {"rope_type": "default", "rope_theta": 1e4},
                                                  "full_attention": {"rope_type": "linear", "factor": 4.0,
                                                                     "rope_theta": 1e6}})
        m = tf.Gemma3ForCausalLM(hc)
    m = _gemma_rand(m)
    if hasattr(m.config, "_attn_implementation"):
        m.config._attn_implementation = "eager"
    cfg = DecoderConfig.from_hf_dict(hc.to_dict())
    assert cfg.norm_unit_offset and cfg.mlp_act == "gelu_tanh"
    if family != "gemma":
        assert cfg.sandwich_norm and cfg.layer_window(0) == 8
    if family == "gemma3_text":
        assert cfg.qk_norm and cfg.rope_local_theta == 1e4 and cfg.rope_scaling["rope_type"] == "linear"
    _check(m, cfg, n=29)
