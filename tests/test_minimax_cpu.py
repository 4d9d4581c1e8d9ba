"""MiniMax-M2 on CPU: full-width QK-norm (one RMSNorm over all heads of a
token), partial RoPE, sigmoid routing with the correction bias on the MoE
block, Mixtral-style experts; the decoder oracle against transformers'
MiniMaxM2ForCausalLM, with the release's ``block_sparse_moe`` names mapped."""
import math

import torch

from rlx_models_b200.config import DecoderConfig
from rlx_models_b200.models.oracle import DecoderOracle
from rlx_models_b200.weights.aliases import canonical_name, split_fused_experts


def test_minimax_m2_oracle_matches_transformers():
    from transformers import MiniMaxM2Config, MiniMaxM2ForCausalLM
    d = dict(vocab_size=128, hidden_size=64, intermediate_size=32, num_hidden_layers=2, num_attention_heads=4,
             num_key_value_heads=2, head_dim=32, num_local_experts=8, num_experts_per_tok=2,
             partial_rotary_factor=0.5, rms_norm_eps=1e-6, max_position_embeddings=256)
    torch.manual_seed(0)
    m = MiniMaxM2ForCausalLM(MiniMaxM2Config(**d)).eval()
    with torch.no_grad():
        for _, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
            elif "norm" in _:
                p.normal_(1.0, 0.2)
        for mod in m.modules():
            if hasattr(mod, "e_score_correction_bias"):
                mod.e_score_correction_bias.normal_(0, 0.5)
    sd = split_fused_experts({k: v.detach() for k, v in m.state_dict().items()})
    assert "model.layers.0.mlp.e_score_correction_bias" in sd
    sd = {canonical_name("minimax_m2", k): v for k, v in sd.items()}
    cfg = DecoderConfig.from_hf_dict(m.config.to_dict())
    assert cfg.qk_norm_full and cfg.rotary_dim == 16 and cfg.router_scoring == "sigmoid" and cfg.num_experts == 8
    ids = torch.randint(0, 128, (29,), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = m(ids[None]).logits[0].float()
    got, _ = DecoderOracle(cfg, sd).forward(ids)
    err = (got - ref).abs().max() / ref.abs().max()
    assert err < 1e-4, err


def test_release_names():
    assert canonical_name("minimax_m2", "model.layers.3.block_sparse_moe.e_score_correction_bias") == \
        "model.layers.3.mlp.gate.e_score_correction_bias"
    assert canonical_name("minimax_m2", "model.layers.3.block_sparse_moe.experts.5.w3.weight") == \
        "model.layers.3.mlp.experts.5.up_proj.weight"
    assert DecoderConfig.from_hf_dict({"model_type": "minimax_m2", "hidden_size": 3072, "num_attention_heads": 48,
                                      "num_key_value_heads": 8, "head_dim": 128, "rotary_dim": 64}).rotary_dim == 64
