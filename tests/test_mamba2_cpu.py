"""Mamba-2 (SSD) families on CPU: the chunked decayed linear attention
against the token recurrence, and the fp32 oracle against transformers'
Mamba2ForCausalLM and BambaForCausalLM (Mamba-2 + attention hybrid)."""
import math

import pytest
import torch

from rlx_models_b200.models.mamba2 import SSMConfig, SSMOracle, decay_attention_chunked


def test_chunked_matches_recurrence():
    g = torch.Generator().manual_seed(0)
    H, L, dk, dv = 3, 90, 8, 12
    q, k, v = torch.randn(H, L, dk, generator=g), torch.randn(H, L, dk, generator=g), torch.randn(H, L, dv, generator=g)
    gl = -torch.rand(H, L, generator=g)
    s0 = torch.randn(H, dk, dv, generator=g)
    S = s0.clone()
    ref = []
    for t in range(L):
        S = gl[:, t].exp()[:, None, None] * S + k[:, t, :, None] * v[:, t, None, :]
        ref.append(torch.einsum("hkv,hk->hv", S, q[:, t]))
    o, s1 = decay_attention_chunked(q, k, v, gl, s0, chunk=16)
    assert torch.allclose(o, torch.stack(ref, 1), atol=1e-4, rtol=1e-4) and torch.allclose(s1, S, atol=1e-4)


def _rand(m):
    torch.manual_seed(0)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2 and "conv1d" not in n:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
            elif n.endswith("norm.weight") or "layernorm" in n or n.endswith("norm_f.weight"):
                p.normal_(1.0, 0.1)
    return m.eval()


@pytest.mark.parametrize("family", ["mamba2", "bamba"])
def test_oracle_matches_transformers(family):
    import transformers as tf
    if family == "mamba2":
        hc = tf.Mamba2Config(vocab_size=128, hidden_size=64, num_hidden_layers=2, state_size=16, num_heads=8,
                             head_dim=16, n_groups=2, conv_kernel=4, chunk_size=16, expand=2)
        m = _rand(tf.Mamba2ForCausalLM(hc))
    else:
        hc = tf.BambaConfig(vocab_size=128, hidden_size=64, num_hidden_layers=3, num_attention_heads=4,
                            num_key_value_heads=2, intermediate_size=96, mamba_n_heads=8, mamba_d_head=16,
                            mamba_n_groups=2, mamba_d_state=16, mamba_chunk_size=16, attn_layer_indices=[1])
        m = _rand(tf.BambaForCausalLM(hc))
    cfg = SSMConfig.from_dict(hc.to_dict())
    assert cfg.intermediate == 128 and cfg.conv_dim == 192
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    ids = torch.randint(0, 128, (1, 45), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        ref = m(ids).logits[0].float()
    got = SSMOracle(cfg, sd, chunk=16).logits(ids[0])
    err = (got - ref).abs().max() / ref.abs().max()
    assert err < 1e-4, err
