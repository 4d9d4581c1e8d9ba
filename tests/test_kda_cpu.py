"""Kimi Delta Attention on CPU: the chunked prefill form == the token
recurrence (carried state, strong decays, ragged last chunk), the KDA block ==
a literal per-token restatement of the reference block (state [Hv, Dv, Dk],
rms-normed q / k scaled by scale^2 / scale), block continuation == one pass,
the Kimi-Linear oracle (KDA + NoPE MLA + DeepSeek MoE) is causal, and the
config reader takes Kimi-Linear's keys."""
import pytest
import torch
import torch.nn.functional as F

from rlx_models_b200.models.kda import (KimiLinearConfig, KimiLinearOracle, kda_chunked, kda_gate, kda_layer,
                                        kda_recurrent, random_weights)


def _rand(T, H, Dk, Dv, seed, strong=False):
    g = torch.Generator().manual_seed(seed)
    q = F.normalize(torch.randn(T, H, Dk, generator=g), dim=-1) * Dk ** -0.5
    k = F.normalize(torch.randn(T, H, Dk, generator=g), dim=-1)
    v = torch.randn(T, H, Dv, generator=g)
    a = torch.randn(T, H * Dk, generator=g) * (3.0 if strong else 1.0)
    gate = kda_gate(a, torch.rand(H, generator=g) * (8.0 if strong else 1.0) + 0.1, torch.randn(H * Dk, generator=g))
    beta = torch.sigmoid(torch.randn(T, H, generator=g))
    return q, k, v, gate, beta


@pytest.mark.parametrize("T,chunk,strong", [(37, 8, False), (64, 16, False), (50, 64, True), (5, 4, True)])
def test_chunked_equals_recurrent(T, chunk, strong):
    q, k, v, g, beta = _rand(T, 3, 16, 12, seed=T, strong=strong)
    S0 = torch.randn(3, 16, 12, generator=torch.Generator().manual_seed(9)) * 0.3
    o_r, S_r = kda_recurrent(q, k, v, g, beta, S0)
    o_c, S_c = kda_chunked(q, k, v, g, beta, S0, chunk=chunk)
    assert torch.isfinite(o_c).all()
    assert torch.allclose(o_c, o_r, atol=1e-4, rtol=1e-4), (o_c - o_r).abs().max()
    assert torch.allclose(S_c, S_r, atol=1e-4, rtol=1e-4)


def _cfg(**over):
    d = {"model_type": "kimi_linear", "vocab_size": 64, "hidden_size": 48, "intermediate_size": 64,
         "moe_intermediate_size": 32, "num_hidden_layers": 4, "num_attention_heads": 2, "num_key_value_heads": 2,
         "q_lora_rank": None, "kv_lora_rank": 16, "qk_nope_head_dim": 16, "qk_rope_head_dim": 8, "v_head_dim": 16,
         "mla_use_nope": True, "num_experts": 4, "num_experts_per_token": 2, "num_shared_experts": 1,
         "first_k_dense_replace": 1, "moe_router_activation_func": "sigmoid", "moe_renormalize": True,
         "routed_scaling_factor": 2.0, "use_grouped_topk": True, "num_expert_group": 1, "topk_group": 1,
         "rms_norm_eps": 1e-5, "tie_word_embeddings": False,
         "linear_attn_config": {"kda_layers": [1, 2, 4], "full_attn_layers": [3], "num_heads": 2, "head_dim": 8,
                                "short_conv_kernel_size": 4}}
    d.update(over)
    return KimiLinearConfig.from_dict(d)


def test_config_keys():
    c = _cfg()
    assert [c.is_kda(i) for i in range(4)] == [True, True, False, True]
    assert c.n_routed_experts == 4 and c.num_experts_per_tok == 2 and c.n_shared_experts == 1
    assert c.scoring_func == "sigmoid" and c.norm_topk_prob and c.kda_head_dim == 8 and c.kda_conv_kernel == 4
    assert c.is_moe(1) and not c.is_moe(0)


def _reference_block(w, p, x, H, D, eps):
    """The reference block written out per token: short conv + silu, rms-norm
    (eps 1e-6, no gain) with q *= scale^2 and k *= scale, per-channel decay,
    state [H, Dv, Dk], per-head o-norm with gain, sigmoid output gate."""
    T = x.shape[0]
    P = H * D
    sc = D ** -0.5

    def conv(name):
        y = x @ w[p + f"{name}_proj.weight"].t()  # [T, P]
        cw = w[p + f"{name}_conv1d.weight"].reshape(P, -1)
        K = cw.shape[1]
        yp = F.pad(y.t(), (K - 1, 0))
        return F.silu(torch.stack([(yp[:, t:t + K] * cw).sum(-1) for t in range(T)]))  # [T, P]

    def rms(z):
        z = z.view(T, H, D)
        return z * torch.rsqrt(z.pow(2).mean(-1, keepdim=True) + 1e-6)

    q, k, v = rms(conv("q")) * sc * sc, rms(conv("k")) * sc, conv("v").view(T, H, D)
    a = (x @ w[p + "f_a_proj.weight"].t()) @ w[p + "f_b_proj.weight"].t()
    dec = torch.exp(-w[p + "A_log"].exp()[None, :, None] * F.softplus(a.view(T, H, D) + w[p + "dt_bias"].view(H, D)))
    beta = torch.sigmoid(x @ w[p + "b_proj.weight"].t())
    S = torch.zeros(H, D, D)  # [Hv, Dv, Dk]
    ys = []
    for t in range(T):
        Sd = S * dec[t][:, None, :]
        delta = (v[t] - (Sd * k[t][:, None, :]).sum(-1)) * beta[t][:, None]
        S = Sd + k[t][:, None, :] * delta[:, :, None]
        ys.append((S * q[t][:, None, :]).sum(-1))
    y = torch.stack(ys)  # [T, H, D]
    y = y * torch.rsqrt(y.pow(2).mean(-1, keepdim=True) + eps) * w[p + "o_norm.weight"]
    gate = torch.sigmoid((x @ w[p + "g_a_proj.weight"].t()) @ w[p + "g_b_proj.weight"].t()).view(T, H, D)
    return (y * gate).reshape(T, P) @ w[p + "o_proj.weight"].t()


def test_block_matches_reference_restatement_and_continues():
    c = _cfg()
    w = random_weights(c, seed=3)
    p = "model.layers.0.self_attn."
    x = torch.randn(23, c.hidden_size, generator=torch.Generator().manual_seed(5))
    get = w.__getitem__
    ref = _reference_block(w, p, x, c.kda_num_heads, c.kda_head_dim, c.rms_norm_eps)
    out, S, win = kda_layer(get, p, x, c.kda_num_heads, c.kda_head_dim, c.rms_norm_eps, chunk=8)
    assert torch.allclose(out, ref, atol=2e-4, rtol=2e-4), (out - ref).abs().max()
    o1, S1, w1 = kda_layer(get, p, x[:10], c.kda_num_heads, c.kda_head_dim, c.rms_norm_eps, chunk=8)
    o2, S2, w2 = kda_layer(get, p, x[10:11], c.kda_num_heads, c.kda_head_dim, c.rms_norm_eps, S1, w1, chunk=8)
    o3, S3, _ = kda_layer(get, p, x[11:], c.kda_num_heads, c.kda_head_dim, c.rms_norm_eps, S2, w2, chunk=8)
    assert torch.allclose(torch.cat([o1, o2, o3]), out, atol=1e-4, rtol=1e-4)
    assert torch.allclose(S3, S, atol=1e-4, rtol=1e-4)


def test_kimi_linear_oracle_is_causal():
    c = _cfg()
    orc = KimiLinearOracle(c, random_weights(c, seed=1), chunk=4)
    ids = torch.randint(0, c.vocab_size, (13,), generator=torch.Generator().manual_seed(2))
    full = orc.logits(ids)
    assert full.shape == (13, c.vocab_size) and torch.isfinite(full).all()
    part = orc.logits(ids[:6])
    assert torch.allclose(part, full[:6], atol=1e-4, rtol=1e-4)
    # NoPE MLA: the MLA layer's output does not depend on absolute positions
    x = torch.randn(5, c.hidden_size, generator=torch.Generator().manual_seed(3))
    a0 = orc.attention(2, x, torch.arange(5))
    a1 = orc.attention(2, x, torch.arange(5) + 100)
    assert torch.allclose(a0, a1, atol=1e-5)
