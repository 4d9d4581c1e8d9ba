"""DeepSeek-V3 / V2 family on CPU: the fp32 oracle against transformers, the
group-limited router, and the absorbed latent decode attention against the
expanded attention."""
import math

import pytest
import torch

from rlx_models_b200.models.deepseek import (DeepseekConfig, DeepseekOracle, apply_rope, latent_decode_attention,
                                             random_weights, route)


def tiny_v3(**kw):
    d = dict(vocab_size=128, hidden_size=64, intermediate_size=96, moe_intermediate_size=32, num_hidden_layers=3,
             num_attention_heads=4, n_shared_experts=1, n_routed_experts=16, routed_scaling_factor=2.5,
             kv_lora_rank=32, q_lora_rank=48, qk_rope_head_dim=16, v_head_dim=24, qk_nope_head_dim=24, n_group=4,
             topk_group=2, num_experts_per_tok=4, first_k_dense_replace=1, norm_topk_prob=True,
             max_position_embeddings=256, rope_interleave=True)
    d.update(kw)
    return d


def _hf_v3(d, rope=None):
    from transformers import DeepseekV3Config, DeepseekV3ForCausalLM
    hd = dict(d)
    if rope:
        hd["rope_parameters"] = rope
    cfg = DeepseekV3Config(**hd)
    torch.manual_seed(0)
    m = DeepseekV3ForCausalLM(cfg).eval()
    with torch.no_grad():
        for name, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
        for mod in m.modules():
            if hasattr(mod, "e_score_correction_bias"):
                mod.e_score_correction_bias.normal_(0, 0.1)
    return m


@pytest.mark.parametrize("rope", [None, {"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 64,
                                         "beta_fast": 32.0, "beta_slow": 1.0, "mscale": 1.0, "mscale_all_dim": 1.0,
                                         "rope_theta": 10000.0}])
@pytest.mark.parametrize("q_lora", [48, None])
def test_v3_oracle_matches_transformers(rope, q_lora):
    d = tiny_v3(q_lora_rank=q_lora)
    m = _hf_v3(d, rope)
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    hd = dict(d, model_type="deepseek_v3")
    if rope:
        hd["rope_parameters"] = rope
    cfg = DeepseekConfig.from_dict(hd)
    ids = torch.randint(0, 128, (1, 40), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = m(ids).logits[0].float()
    got = DeepseekOracle(cfg, sd).logits(ids[0])
    err = (got - ref).abs().max() / ref.abs().max()
    assert err < 1e-4, err


def test_v2_oracle_matches_transformers():
    from transformers import DeepseekV2Config, DeepseekV2ForCausalLM
    d = tiny_v3(q_lora_rank=None, n_group=4, topk_group=2, norm_topk_prob=False, routed_scaling_factor=1.0)
    d.pop("rope_interleave")
    hd = dict(d, topk_method="greedy")  # transformers' group_limited_greedy branch does not run
    torch.manual_seed(0)
    m = DeepseekV2ForCausalLM(DeepseekV2Config(**hd)).eval()
    with torch.no_grad():
        for _, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    cfg = DeepseekConfig.from_dict(dict(hd, model_type="deepseek_v2"))
    assert cfg.scoring_func == "softmax" and cfg.topk_method == "greedy"
    ids = torch.randint(0, 128, (1, 33), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        ref = m(ids).logits[0].float()
    got = DeepseekOracle(cfg, sd).logits(ids[0])
    err = (got - ref).abs().max() / ref.abs().max()
    assert err < 1e-4, err


def test_router_group_limit():
    cfg = DeepseekConfig(n_routed_experts=8, n_group=4, topk_group=1, num_experts_per_tok=2, norm_topk_prob=True,
                         routed_scaling_factor=2.0)
    logits = torch.full((1, 8), -4.0)
    logits[0, 0] = 3.0  # group 0 holds the best single expert...
    logits[0, 6] = 2.5
    logits[0, 7] = 2.5  # ...but group 3 has the best top-2 sum
    idx, w = route(cfg, logits, None)
    assert sorted(idx[0].tolist()) == [6, 7]
    assert torch.allclose(w.sum(), torch.tensor(2.0))
    bias = torch.zeros(8)
    bias[0] = bias[1] = 5.0  # the correction bias steers the choice, not the weights
    idx, w = route(cfg, logits, bias)
    assert sorted(idx[0].tolist()) == [0, 1]
    s = logits.sigmoid()[0]
    assert torch.allclose(w[0].sort().values, (torch.stack([s[1], s[0]]) / (s[0] + s[1]) * 2).sort().values)


def test_router_v2_group_limited_greedy():
    cfg = DeepseekConfig(n_routed_experts=8, n_group=4, topk_group=2, num_experts_per_tok=2, norm_topk_prob=False,
                         routed_scaling_factor=1.0, scoring_func="softmax", topk_method="group_limited_greedy")
    logits = torch.tensor([[3.0, -9, 2.9, -9, -9, 2.8, 0.0, 0.1]])
    idx, w = route(cfg, logits, None)  # groups by max: g0 (3.0), g1 (2.9) survive; g2's 2.8 is dropped
    assert sorted(idx[0].tolist()) == [0, 2]
    p = logits.softmax(-1)[0]
    assert torch.allclose(w[0].sort().values, torch.stack([p[2], p[0]]))


def test_latent_decode_matches_expanded():
    """Absorbed decode over a paged latent cache == the oracle's expanded
    attention at the last position of each sequence."""
    cfg = DeepseekConfig.from_dict(tiny_v3())
    w = random_weights(cfg, seed=3, dtype=torch.float32)
    orc = DeepseekOracle(cfg, w)
    nh, dn, dr, dv, r = cfg.num_attention_heads, cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim, \
        cfg.kv_lora_rank
    a = "model.layers.0.self_attn."
    g = torch.Generator().manual_seed(4)
    lens = [5, 21, 37]
    nb = 12
    cache = torch.zeros(nb, 16, cfg.latent_dim)
    tables = torch.tensor([[0, 11, 11], [1, 2, 11], [3, 4, 5]])
    outs, qn, qr = [], [], []
    for b, n in enumerate(lens):
        x = torch.randn(n, cfg.hidden_size, generator=g)
        pos = torch.arange(n)
        outs.append(orc.attention_heads(0, x, pos)[-1])
        ckv = x @ orc._t(a + "kv_a_proj_with_mqa.weight").t()
        lat = torch.cat([orc._rms(ckv[:, :r], orc._t(a + "kv_a_layernorm.weight"), 1e-6),
                         apply_rope(ckv[:, r:], pos, orc.inv, orc.mult, True)], -1)
        for t in range(n):
            cache[tables[b, t // 16], t % 16] = lat[t]
        q = orc._rms(x[-1:] @ orc._t(a + "q_a_proj.weight").t(), orc._t(a + "q_a_layernorm.weight"), 1e-6)
        q = (q @ orc._t(a + "q_b_proj.weight").t()).view(1, nh, dn + dr)
        qn.append(q[0, :, :dn])
        qr.append(apply_rope(q[:, :, dn:], pos[-1:], orc.inv, orc.mult, True)[0])
    kvb = orc._t(a + "kv_b_proj.weight").view(nh, dn + dv, r)
    got = latent_decode_attention(torch.stack(qn), torch.stack(qr), kvb[:, :dn], kvb[:, dn:].transpose(1, 2),
                                  cache, tables, torch.tensor(lens), cfg.softmax_scale)
    ref = torch.stack(outs)
    assert (got - ref).abs().max() < 1e-3 * ref.abs().max() + 1e-4


def test_config_roundtrip_and_scale():
    rope = {"rope_type": "yarn", "factor": 40.0, "mscale": 1.0, "mscale_all_dim": 1.0,
            "original_max_position_embeddings": 4096, "beta_fast": 32, "beta_slow": 1}
    cfg = DeepseekConfig.from_dict({"model_type": "deepseek_v3", "rope_scaling": rope, "rope_theta": 10000.0})
    m = 0.1 * math.log(40.0) + 1.0
    assert abs(cfg.softmax_scale - 192 ** -0.5 * m * m) < 1e-9
    assert cfg.latent_dim == 576 and cfg.is_moe(3) and not cfg.is_moe(2)
    cfg2 = DeepseekConfig.from_dict(cfg.to_hf_dict())
    assert cfg2.rope_scaling["factor"] == 40.0 and cfg2.softmax_scale == cfg.softmax_scale
