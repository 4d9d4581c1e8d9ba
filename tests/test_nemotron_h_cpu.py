"""Nemotron-H (hybrid Mamba-2 / NoPE attention / squared-ReLU MoE) on CPU: the
SSM oracle against transformers' NemotronHForCausalLM, with and without the
MoE latent projection."""
import math

import pytest
import torch

from rlx_models_b200.models.mamba2 import SSMConfig, SSMOracle, gated_norm


@pytest.mark.parametrize("latent", [None, 24])
def test_nemotron_h_oracle_matches_transformers(latent):
    from transformers import NemotronHConfig, NemotronHForCausalLM
    d = dict(vocab_size=128, hidden_size=64, layers_block_type=["mamba", "moe", "attention", "moe", "mamba"],
             num_attention_heads=4, num_key_value_heads=2, head_dim=16, mamba_num_heads=8, mamba_head_dim=16,
             ssm_state_size=16, n_groups=2, conv_kernel=4, expand=2, n_routed_experts=8, num_experts_per_tok=2,
             moe_intermediate_size=32, moe_shared_expert_intermediate_size=48, moe_latent_size=latent, n_group=2,
             topk_group=1, routed_scaling_factor=2.0, norm_topk_prob=True, chunk_size=16, tie_word_embeddings=False)
    torch.manual_seed(0)
    m = NemotronHForCausalLM(NemotronHConfig(**d)).eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2 and "conv1d" not in n:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
            elif n.endswith("norm.weight"):
                p.normal_(1.0, 0.2)
        for mod in m.modules():
            if hasattr(mod, "e_score_correction_bias"):
                mod.e_score_correction_bias.normal_(0, 0.2)
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    cfg = SSMConfig.from_dict(m.config.to_dict())
    assert cfg.layer_types[1] == "moe" and cfg.is_attention(2) and cfg.norm_groups == 2 and cfg.rotary_dim == 0
    ids = torch.randint(0, 128, (45,), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = m(ids[None]).logits[0].float()
    got = SSMOracle(cfg, sd, chunk=16).logits(ids)
    err = (got - ref).abs().max() / ref.abs().max()
    # attention and MoE blocks alone agree to ~5e-7; each Mamba-2 block adds
    # ~2e-4 against transformers' naive (non-kernel) scan
    assert err < 1e-3, err


def test_grouped_gated_norm():
    y, z, w = torch.randn(3, 8), torch.randn(3, 8), torch.rand(8)
    t = y * torch.nn.functional.silu(z)
    a, b = t[:, :4], t[:, 4:]
    ref = torch.cat([a * torch.rsqrt(a.pow(2).mean(-1, keepdim=True) + 1e-5),
                     b * torch.rsqrt(b.pow(2).mean(-1, keepdim=True) + 1e-5)], -1) * w
    assert torch.allclose(gated_norm(y, z, w, 1e-5, groups=2), ref, atol=1e-6)
    assert SSMConfig.from_dict({"model_type": "nemotron_h", "hidden_size": 64, "num_attention_heads": 4,
                                "hybrid_override_pattern": "M*ME"}).layer_types == ["mamba", "attention", "mamba",
                                                                                     "moe"]


def test_nemotron_h_mlp_block():
    """Squared-ReLU MLP blocks ("-" in the hybrid pattern of the dense Nemotron-H
    releases): h += relu(rmsnorm(h) W_up)^2 W_down, the formula of transformers'
    NemotronHMLP with mlp_hidden_act relu2."""
    from transformers import NemotronHConfig
    from transformers.models.nemotron_h.modeling_nemotron_h import NemotronHMLP
    cfg = SSMConfig.from_dict(dict(model_type="nemotron_h", vocab_size=64, hidden_size=32,
                                   hybrid_override_pattern="-", num_attention_heads=4, num_key_value_heads=2,
                                   head_dim=8, mamba_num_heads=4, mamba_head_dim=8, ssm_state_size=8,
                                   tie_word_embeddings=False))
    assert cfg.is_mlp(0) and not cfg.is_mamba(0)
    mlp = NemotronHMLP(NemotronHConfig(hidden_size=32, intermediate_size=48, mlp_hidden_act="relu2")).eval()
    g = torch.Generator().manual_seed(0)
    w = {"backbone.embeddings.weight": torch.randn(64, 32, generator=g),
         "backbone.norm_f.weight": torch.rand(32, generator=g) + 0.5,
         "backbone.layers.0.norm.weight": torch.rand(32, generator=g) + 0.5,
         "backbone.layers.0.mixer.up_proj.weight": mlp.up_proj.weight.detach(),
         "backbone.layers.0.mixer.down_proj.weight": mlp.down_proj.weight.detach(),
         "lm_head.weight": torch.randn(64, 32, generator=g)}
    ids = torch.randint(0, 64, (9,), generator=g)
    got = SSMOracle(cfg, w).logits(ids)

    def rms(x, wt):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.rms_norm_eps) * wt
    h = w["backbone.embeddings.weight"][ids]
    with torch.no_grad():
        h = h + mlp(rms(h, w["backbone.layers.0.norm.weight"]))
    ref = rms(h, w["backbone.norm_f.weight"]) @ w["lm_head.weight"].t()
    assert (got - ref).abs().max() < 1e-4
