"""GLM-4.7-Flash (glm4_moe_lite) and GLM-5 (glm_moe_dsa) on CPU: the MLA +
DeepSeekMoE oracle against transformers, GLM-5's DSA indexer (top-k keys per
query) included."""
import math

import pytest
import torch

from rlx_models_b200.models.deepseek import DeepseekConfig, DeepseekOracle, random_weights


def _tiny(**kw):
    d = dict(vocab_size=128, hidden_size=64, intermediate_size=96, moe_intermediate_size=32, num_hidden_layers=3,
             num_attention_heads=4, num_key_value_heads=4, n_shared_experts=1, n_routed_experts=8,
             routed_scaling_factor=1.8, kv_lora_rank=32, q_lora_rank=48, qk_rope_head_dim=16, v_head_dim=32,
             qk_nope_head_dim=24, n_group=1, topk_group=1, num_experts_per_tok=2, norm_topk_prob=True,
             max_position_embeddings=256, mlp_layer_types=["dense", "sparse", "sparse"])
    d.update(kw)
    return d


def _randomise(m):
    torch.manual_seed(0)
    with torch.no_grad():
        for _, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
        for mod in m.modules():
            if hasattr(mod, "e_score_correction_bias"):
                mod.e_score_correction_bias.normal_(0, 0.1)
    return m.eval()


def _compare(m, d, mt, S, seed):
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    cfg = DeepseekConfig.from_dict(dict(d, model_type=mt))
    ids = torch.randint(0, 128, (1, S), generator=torch.Generator().manual_seed(seed))
    with torch.no_grad():
        ref = m(ids).logits[0].float()
    orc = DeepseekOracle(cfg, sd)
    got = orc.logits(ids[0])
    err = (got - ref).abs().max() / ref.abs().max()
    assert err < 1e-4, err
    return cfg, orc, ids


def test_glm4_moe_lite_matches_transformers():
    from transformers import Glm4MoeLiteConfig, Glm4MoeLiteForCausalLM
    d = _tiny()
    m = _randomise(Glm4MoeLiteForCausalLM(Glm4MoeLiteConfig(**d)))
    cfg, _, _ = _compare(m, d, "glm4_moe_lite", 37, 1)
    assert cfg.rope_interleave and not cfg.is_moe(0) and cfg.is_moe(1) and cfg.index_topk == 0


@pytest.mark.parametrize("topk", [8, 64])
def test_glm5_dsa_matches_transformers(topk):
    """With index_topk below the sequence length the indexer drops keys (the
    output differs from dense MLA); at or above it attention is dense."""
    from transformers import GlmMoeDsaConfig, GlmMoeDsaForCausalLM
    d = _tiny(index_topk=topk, index_n_heads=4, index_head_dim=32)
    hc = GlmMoeDsaConfig(**d)
    # eager attention: transformers' SDPA path hands the DSA mask no causal part
    # when it has no padding mask, so only the eager path is the causal model
    hc._attn_implementation = "eager"
    m = _randomise(GlmMoeDsaForCausalLM(hc))
    cfg, orc, ids = _compare(m, d, "glm_moe_dsa", 40, 2)
    assert not cfg.rope_interleave and cfg.index_topk == topk
    dense = DeepseekOracle(DeepseekConfig.from_dict(dict(d, model_type="glm_moe_dsa", index_topk=0)), orc.w)
    diff = (dense.logits(ids[0]) - orc.logits(ids[0])).abs().max()
    assert (diff > 1e-3) if topk < 40 else (diff < 1e-5), diff


def test_dsa_selection_bounds():
    """Each query keeps min(index_topk, S) positions; rows before index_topk keep
    every causal position, later rows exactly index_topk of them."""
    cfg = DeepseekConfig.from_dict(_tiny(model_type="glm_moe_dsa", index_topk=6, index_n_heads=2, index_head_dim=32,
                                         num_hidden_layers=1, mlp_layer_types=["dense"]))
    w = random_weights(cfg, seed=3, dtype=torch.float32)
    orc = DeepseekOracle(cfg, w)
    S = 20
    x = torch.randn(S, cfg.hidden_size, generator=torch.Generator().manual_seed(5))
    a = "model.layers.0.self_attn."
    q_res = orc._rms(x @ orc._t(a + "q_a_proj.weight").t(), orc._t(a + "q_a_layernorm.weight"), 1e-6)
    sel = orc.dsa_select(0, x, q_res, torch.arange(S))
    assert sel.shape == (S, 6)
    for s in range(S):
        causal = [t for t in sel[s].tolist() if t <= s]
        assert len(set(causal)) == min(s + 1, 6)
