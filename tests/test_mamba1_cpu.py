"""Mamba-1 families on CPU: the fp32 oracle (selective scan) against
transformers' Mamba / FalconMamba / Jamba (Mamba-1 + NoPE attention + top-2 MoE)."""
import math

import pytest
import torch

from rlx_models_b200.models.mamba1 import Mamba1Config, Mamba1Oracle


def _rand(m):
    torch.manual_seed(0)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2 and "conv1d" not in n and "A_log" not in n:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
            elif "norm" in n:
                p.normal_(1.0, 0.1)
    return m.eval()


@pytest.mark.parametrize("family", ["mamba", "falcon_mamba", "jamba"])
def test_oracle_matches_transformers(family):
    import transformers as tf
    if family == "mamba":
        hc = tf.MambaConfig(vocab_size=128, hidden_size=64, num_hidden_layers=2, state_size=16)
        m = tf.MambaForCausalLM(hc)
    elif family == "falcon_mamba":
        hc = tf.FalconMambaConfig(vocab_size=128, hidden_size=64, num_hidden_layers=2, state_size=16)
        m = tf.FalconMambaForCausalLM(hc)
    else:
        hc = tf.JambaConfig(vocab_size=128, hidden_size=64, num_hidden_layers=4, num_attention_heads=4,
                            num_key_value_heads=2, intermediate_size=96, num_experts=4, num_experts_per_tok=2,
                            expert_layer_period=2, expert_layer_offset=1, attn_layer_period=4, attn_layer_offset=2,
                            mamba_d_state=16, mamba_d_conv=4, mamba_expand=2, mamba_dt_rank=8)
        m = tf.JambaForCausalLM(hc)
    m = _rand(m)
    cfg = Mamba1Config.from_dict(hc.to_dict())
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    ids = torch.randint(0, 128, (1, 29), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        ref = m(ids).logits[0].float()
    got = Mamba1Oracle(cfg, sd).logits(ids[0])
    err = (got - ref).abs().max() / ref.abs().max()
    assert err < 1e-4, err
