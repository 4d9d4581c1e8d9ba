"""GLM-4.5 family (glm4_moe) on CPU: partial RoPE (half the head), optional
qkv bias and QK-norm, DeepSeek-style sigmoid group-limited routing with the
correction bias, shared experts and dense first layers; the decoder oracle
against transformers' Glm4MoeForCausalLM."""
import math

import pytest
import torch

from rlx_models_b200.config import DecoderConfig
from rlx_models_b200.models.oracle import DecoderOracle
from rlx_models_b200.weights.aliases import split_fused_experts


def tiny_glm(**kw):
    d = dict(model_type="glm4_moe", vocab_size=128, hidden_size=64, intermediate_size=96, moe_intermediate_size=32,
             num_hidden_layers=3, num_attention_heads=4, num_key_value_heads=2, head_dim=32,
             partial_rotary_factor=0.5, n_shared_experts=1, n_routed_experts=16, num_experts_per_tok=4, n_group=4,
             topk_group=2, routed_scaling_factor=2.0, first_k_dense_replace=1, norm_topk_prob=True,
             attention_bias=True, use_qk_norm=False, rms_norm_eps=1e-5, max_position_embeddings=256)
    d.update(kw)
    return d


def _hf(d):
    from transformers import Glm4MoeConfig, Glm4MoeForCausalLM
    torch.manual_seed(0)
    m = Glm4MoeForCausalLM(Glm4MoeConfig(**{k: v for k, v in d.items() if k != "model_type"})).eval()
    with torch.no_grad():
        for _, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
            elif p.dim() == 1 and "bias" in _:
                p.normal_(0, 0.1)
        for mod in m.modules():
            if hasattr(mod, "e_score_correction_bias"):
                mod.e_score_correction_bias.normal_(0, 0.1)
    return m


@pytest.mark.parametrize("qk_norm,bias", [(False, True), (True, False)])
def test_glm4_moe_oracle_matches_transformers(qk_norm, bias):
    d = tiny_glm(use_qk_norm=qk_norm, attention_bias=bias)
    m = _hf(d)
    sd = split_fused_experts({k: v.detach() for k, v in m.state_dict().items()})
    cfg = DecoderConfig.from_hf_dict(m.config.to_dict())
    assert cfg.model_type == "glm4_moe" and cfg.rotary_dim == 16 and cfg.router_scoring == "sigmoid"
    assert cfg.qk_norm == qk_norm and cfg.is_moe_layer(1) and not cfg.is_moe_layer(0)
    ids = torch.randint(0, 128, (37,), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = m(ids[None]).logits[0].float()
    got, _ = DecoderOracle(cfg, sd).forward(ids)
    err = (got - ref).abs().max() / ref.abs().max()
    assert err < 1e-4, err


def test_partial_rope_reference():
    from rlx_models_b200.ops import reference as R
    x = torch.randn(5, 2, 32)
    inv = 1.0 / (10000 ** (torch.arange(0, 16, 2).float() / 16))
    y = R.rope(x, torch.arange(5), inv)
    assert torch.equal(y[..., 16:], x[..., 16:])
    assert torch.allclose(y[..., :16], R.rope(x[..., :16], torch.arange(5), inv))
    assert not torch.allclose(y[1:, :, :16], x[1:, :, :16])
