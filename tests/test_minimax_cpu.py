"""MiniMax-Text-01 (lightning attention hybrid + MoE) on CPU: the fp32 oracle
== transformers' MiniMaxForCausalLM, continuation from a carried state ==
the full-sequence forward, and the GPU model's lightning-decode mapping onto
the SSD decode kernel (restated here in torch) == the oracle's recurrence."""
import math

import pytest
import torch
import torch.nn.functional as F

from rlx_models_b200.models.minimax import (DT_ONE, LIGHTNING_NORM_EPS, MiniMaxConfig, MiniMaxOracle,
                                            pack_lightning, random_weights)

transformers = pytest.importorskip("transformers")


def _hf(seed=0, **over):
    from transformers import MiniMaxConfig as HFConfig, MiniMaxForCausalLM
    kw = dict(vocab_size=96, hidden_size=64, intermediate_size=64, num_hidden_layers=4, num_attention_heads=4,
              num_key_value_heads=2, head_dim=16, num_local_experts=4, num_experts_per_tok=2, block_size=8,
              layer_types=["linear_attention", "full_attention", "linear_attention", "linear_attention"],
              full_attn_alpha_factor=1.7, full_attn_beta_factor=0.8, linear_attn_alpha_factor=1.3,
              linear_attn_beta_factor=1.1, mlp_alpha_factor=1.5, mlp_beta_factor=0.9, max_position_embeddings=256,
              rope_parameters={"rope_type": "default", "rope_theta": 10000.0}, rms_norm_eps=1e-5)
    kw.update(over)
    hcfg = HFConfig(**kw)
    torch.manual_seed(seed)
    model = MiniMaxForCausalLM(hcfg).float().eval()
    with torch.no_grad():  # norms away from 1 so that a missing weight shows
        for n, p in model.named_parameters():
            if n.endswith("norm.weight") or "layernorm" in n:
                p.add_(0.1 * torch.randn_like(p))
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    return model, MiniMaxConfig.from_dict(hcfg.to_dict()), sd


def test_oracle_matches_transformers():
    model, cfg, sd = _hf()
    ids = torch.randint(0, cfg.vocab_size, (1, 21), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = model(ids).logits[0].float()
    got = MiniMaxOracle(cfg, sd).logits(ids[0])
    assert torch.allclose(got, ref, atol=1e-4, rtol=1e-4), (got - ref).abs().max()


def test_oracle_matches_transformers_cached_decode():
    model, cfg, sd = _hf(seed=3)
    ids = torch.randint(0, cfg.vocab_size, (1, 14), generator=torch.Generator().manual_seed(2))
    orc = MiniMaxOracle(cfg, sd)
    with torch.no_grad():
        out = model(ids[:, :10], use_cache=True)
        past = out.past_key_values
        lg, st = orc.step(ids[0, :10])
        assert torch.allclose(lg, out.logits[0], atol=1e-4, rtol=1e-4)
        for t in range(10, 14):
            out = model(ids[:, t:t + 1], past_key_values=past, use_cache=True)
            past = out.past_key_values
            lg, st = orc.step(ids[0, t:t + 1], st)
            assert torch.allclose(lg, out.logits[0], atol=1e-4, rtol=1e-4), (t, (lg - out.logits[0]).abs().max())


def test_state_continuation_equals_full_sequence():
    cfg = MiniMaxConfig(vocab_size=80, hidden_size=48, num_hidden_layers=3, num_attention_heads=3,
                        num_key_value_heads=1, head_dim=16, intermediate_size=32, num_local_experts=3,
                        num_experts_per_tok=2, block_size=4, sliding_window=9,
                        layer_types=["linear_attention", "full_attention", "linear_attention"])
    w = random_weights(cfg, seed=5, dtype=torch.float32)
    orc = MiniMaxOracle(cfg, w)
    ids = torch.randint(0, 80, (19,), generator=torch.Generator().manual_seed(4))
    full = orc.logits(ids)
    lg, st = orc.step(ids[:7])
    parts = [lg]
    for a, b in ((7, 12), (12, 13), (13, 19)):
        lg, st = orc.step(ids[a:b], st)
        parts.append(lg)
    assert torch.allclose(torch.cat(parts), full, atol=1e-4, rtol=1e-4)


def _ssd_decode_restated(proj, xbc_off, dt_off, conv_w, A_log, dt_bias, Dp, G, S):
    """The SSD decode kernel's arithmetic for one token of one sequence (fp32):
    x / B / C = silu(conv(window, new)) over the projection row, dt =
    softplus(dt_raw + dt_bias), S[h] = exp(-exp(A_log) dt) S[h] + dt B x^T,
    y[h] = S[h]^T C + D x."""
    H, N, P = S.shape
    conv = proj[xbc_off: xbc_off + conv_w.shape[0]] * conv_w[:, -1]  # window holds zeros; taps [.., 1] on the new input
    v = F.silu(conv).to(torch.bfloat16).float()
    x = v[: H * P].view(H, P)
    Bm = v[H * P: H * P + G * N].view(G, N)
    Cm = v[H * P + G * N:].view(G, N)
    dt = F.softplus(proj[dt_off: dt_off + H] + dt_bias)
    dA = torch.exp(-torch.exp(A_log) * dt)
    g = torch.arange(H) // (H // G)
    S = dA[:, None, None] * S + dt[:, None, None] * Bm[g][:, :, None] * x[:, None, :]
    y = torch.einsum("hnp,hn->hp", S, Cm[g]) + Dp[:, None] * x
    return y.reshape(-1), S


def test_lightning_decode_maps_onto_ssd_kernel():
    cfg = MiniMaxConfig(vocab_size=64, hidden_size=32, num_hidden_layers=2, num_attention_heads=2,
                        num_key_value_heads=1, head_dim=8, intermediate_size=16, num_local_experts=2,
                        layer_types=["linear_attention", "full_attention"])
    w = random_weights(cfg, seed=2, dtype=torch.float32)
    a = "model.layers.0.self_attn."
    w_in, Z = pack_lightning(cfg, w[a + "qkv_proj.weight"], w[a + "output_gate.weight"])
    nh, D = cfg.num_attention_heads, cfg.head_dim
    HD = nh * D
    assert w_in.shape[0] == 4 * HD + Z and torch.all(w_in[3 * HD: 3 * HD + Z] == 0)
    conv_w = torch.zeros(3 * HD, 2)
    conv_w[:, 1] = 1
    s = cfg.slopes(0)
    assert math.isclose(F.softplus(torch.tensor(DT_ONE, dtype=torch.float64)).item(), 1.0, rel_tol=1e-12)
    gen = torch.Generator().manual_seed(3)
    S_ref = torch.randn(nh, D, D, generator=gen)
    S_k = S_ref.clone()
    for _ in range(3):
        x = torch.randn(cfg.hidden_size, generator=gen)
        proj = w_in @ x
        y, S_k = _ssd_decode_restated(proj, 0, 3 * HD, conv_w, s.log(), torch.full((nh,), DT_ONE), torch.zeros(nh),
                                      nh, S_k)
        # oracle: silu(qkv) per head, S = exp(-s) S + k^T v, o = q S
        qkv = F.silu(w[a + "qkv_proj.weight"] @ x).to(torch.bfloat16).float().view(nh, 3, D)
        q, k, v = qkv[:, 0], qkv[:, 1], qkv[:, 2]
        S_ref = torch.exp(-s)[:, None, None] * S_ref + k[:, :, None] * v[:, None, :]
        o = torch.einsum("hn,hnp->hp", q, S_ref).reshape(-1)
        assert torch.allclose(y, o, atol=1e-4, rtol=1e-4)
        assert torch.allclose(S_k, S_ref, atol=1e-4, rtol=1e-4)
        gate = proj[3 * HD + Z:]
        assert torch.allclose(gate, w[a + "output_gate.weight"] @ x, atol=1e-5)


def test_release_config_keys():
    d = {"model_type": "minimax", "hidden_size": 64, "num_attention_heads": 4, "num_hidden_layers": 4,
         "attn_type_list": [0, 1, 0, 1], "layernorm_full_attention_alpha": 3.5, "layernorm_mlp_alpha": 2.0,
         "layernorm_linear_attention_beta": 1.0, "rope_theta": 1e6}
    cfg = MiniMaxConfig.from_dict(d)
    assert cfg.layer_types == ["linear_attention", "full_attention"] * 2
    assert cfg.full_attn_alpha_factor == 3.5 and cfg.mlp_alpha_factor == 2.0 and cfg.head_dim == 16
    assert cfg.rope_theta == 1e6 and LIGHTNING_NORM_EPS == 1e-6
