"""Qwen3.5 hybrid (Gated DeltaNet + gated attention) on CPU: the chunked
delta rule against the token-by-token recurrence, the fp32 oracle against
transformers' Qwen3_5ForCausalLM."""
import math

import pytest
import torch

from rlx_models_b200.models.qwen35 import (Qwen35Config, Qwen35Oracle, causal_conv1d, gated_delta_chunked,
                                           gated_delta_recurrent, l2norm)


def test_chunked_matches_recurrent_and_carries_state():
    g = torch.Generator().manual_seed(0)
    H, L, dk, dv = 3, 150, 16, 24
    q = l2norm(torch.randn(H, L, dk, generator=g)) * dk ** -0.5
    k = l2norm(torch.randn(H, L, dk, generator=g))
    v = torch.randn(H, L, dv, generator=g)
    gl = -torch.rand(H, L, generator=g) * 0.5
    beta = torch.rand(H, L, generator=g)
    s0 = torch.randn(H, dk, dv, generator=g) * 0.1
    o_r, s_r = gated_delta_recurrent(q, k, v, gl, beta, s0)
    for C in (16, 64):
        o_c, s_c = gated_delta_chunked(q, k, v, gl, beta, s0, chunk=C)
        assert torch.allclose(o_c, o_r, atol=1e-4, rtol=1e-4)
        assert torch.allclose(s_c, s_r, atol=1e-4, rtol=1e-4)
    # splitting the sequence and carrying the state gives the same outputs
    o1, s1 = gated_delta_chunked(q[:, :70], k[:, :70], v[:, :70], gl[:, :70], beta[:, :70], s0)
    o2, s2 = gated_delta_chunked(q[:, 70:], k[:, 70:], v[:, 70:], gl[:, 70:], beta[:, 70:], s1)
    assert torch.allclose(torch.cat([o1, o2], 1), o_r, atol=1e-4) and torch.allclose(s2, s_r, atol=1e-4)


def test_conv_window_carries():
    g = torch.Generator().manual_seed(1)
    C, L, K = 5, 11, 4
    x, w = torch.randn(C, L, generator=g), torch.randn(C, K, generator=g)
    y, _ = causal_conv1d(x, w)
    y1, win = causal_conv1d(x[:, :6], w)
    y2, _ = causal_conv1d(x[:, 6:], w, win)
    assert torch.allclose(torch.cat([y1, y2], 1), y, atol=1e-6)


def _hf(layers=4, **kw):
    from transformers import Qwen3_5ForCausalLM, Qwen3_5TextConfig
    d = dict(vocab_size=128, hidden_size=64, intermediate_size=96, num_hidden_layers=layers, num_attention_heads=4,
             num_key_value_heads=2, head_dim=32, linear_key_head_dim=16, linear_value_head_dim=16,
             linear_num_key_heads=2, linear_num_value_heads=4, linear_conv_kernel_dim=4, rms_norm_eps=1e-6,
             tie_word_embeddings=False)
    d.update(kw)
    hc = Qwen3_5TextConfig(**d)
    torch.manual_seed(0)
    m = Qwen3_5ForCausalLM(hc).eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2 and "conv1d" not in n:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
            elif n.endswith("norm.weight") and "linear_attn" not in n:
                p.normal_(0, 0.1)
    return m, hc


@pytest.mark.parametrize("recurrent", [False, True])
def test_oracle_matches_transformers(recurrent):
    m, hc = _hf()
    cfg = Qwen35Config.from_dict(hc.to_dict())
    assert cfg.layer_types == ["linear_attention"] * 3 + ["full_attention"] and cfg.rotary_dim == 8
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    ids = torch.randint(0, 128, (1, 77), generator=torch.Generator().manual_seed(3))
    with torch.no_grad():
        ref = m(ids).logits[0].float()
    got = Qwen35Oracle(cfg, sd, chunk=32).logits(ids[0], recurrent=recurrent)
    err = (got - ref).abs().max() / ref.abs().max()
    assert err < 1e-4, err


def test_moe_oracle_matches_transformers():
    from transformers import Qwen3_5MoeForCausalLM, Qwen3_5MoeTextConfig
    hc = Qwen3_5MoeTextConfig(vocab_size=128, hidden_size=64, num_hidden_layers=4, num_attention_heads=4,
                              num_key_value_heads=2, head_dim=32, linear_key_head_dim=16, linear_value_head_dim=16,
                              linear_num_key_heads=2, linear_num_value_heads=4, num_experts=8, num_experts_per_tok=2,
                              moe_intermediate_size=32, shared_expert_intermediate_size=48, tie_word_embeddings=False)
    torch.manual_seed(0)
    m = Qwen3_5MoeForCausalLM(hc).eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2 and "conv1d" not in n:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
            elif n.endswith("norm.weight") and "linear_attn" not in n:
                p.normal_(0, 0.1)
    cfg = Qwen35Config.from_dict(hc.to_dict())
    assert cfg.is_moe and cfg.num_experts == 8
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    assert "model.layers.0.mlp.experts.gate_up_proj" in sd  # transformers' fused expert layout
    ids = torch.randint(0, 128, (1, 41), generator=torch.Generator().manual_seed(3))
    with torch.no_grad():
        ref = m(ids).logits[0].float()
    got = Qwen35Oracle(cfg, sd, chunk=16).logits(ids[0])
    err = (got - ref).abs().max() / ref.abs().max()
    assert err < 1e-4, err


def test_qwen3_next_matches_transformers():
    """Qwen3-Next: the per-group fused in_proj_qkvz / in_proj_ba regrouped into
    the Qwen3.5 layout, MoE on all but the mlp_only_layers."""
    from transformers import Qwen3NextConfig, Qwen3NextForCausalLM
    hc = Qwen3NextConfig(vocab_size=128, hidden_size=64, intermediate_size=96, num_hidden_layers=4,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=32, linear_key_head_dim=16,
                         linear_value_head_dim=16, linear_num_key_heads=2, linear_num_value_heads=4, num_experts=8,
                         num_experts_per_tok=2, moe_intermediate_size=32, shared_expert_intermediate_size=48,
                         mlp_only_layers=[1], norm_topk_prob=False, tie_word_embeddings=False)
    torch.manual_seed(0)
    m = Qwen3NextForCausalLM(hc).eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2 and "conv1d" not in n:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
            elif n.endswith("norm.weight") and "linear_attn" not in n:
                p.normal_(0, 0.1)
    cfg = Qwen35Config.from_dict(hc.to_dict())
    assert cfg.is_moe_layer(0) and not cfg.is_moe_layer(1) and not cfg.norm_topk_prob
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    assert "model.layers.0.linear_attn.in_proj_qkvz.weight" in sd
    ids = torch.randint(0, 128, (1, 37), generator=torch.Generator().manual_seed(3))
    with torch.no_grad():
        ref = m(ids).logits[0].float()
    got = Qwen35Oracle(cfg, sd, chunk=16).logits(ids[0])
    err = (got - ref).abs().max() / ref.abs().max()
    assert err < 1e-4, err
