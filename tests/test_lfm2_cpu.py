"""LFM2 (short-conv + attention hybrid) on CPU: the fp32 oracle against
transformers' Lfm2ForCausalLM; the conv window carries across chunks."""
import math

import torch

from rlx_models_b200.models.lfm2 import Lfm2Config, Lfm2Oracle, short_conv


def test_short_conv_window_carries():
    g = torch.Generator().manual_seed(0)
    x, w, b = torch.randn(6, 13, generator=g), torch.randn(6, 3, generator=g), torch.randn(6, generator=g)
    y, _ = short_conv(x, w, b, None)
    y1, win = short_conv(x[:, :1], w, b, None)
    y2, _ = short_conv(x[:, 1:], w, b, win)
    assert torch.allclose(torch.cat([y1, y2], 1), y, atol=1e-6)


def test_lfm2_oracle_matches_transformers():
    from transformers import Lfm2Config as HFC, Lfm2ForCausalLM
    hc = HFC(vocab_size=128, hidden_size=64, intermediate_size=192, num_hidden_layers=4, num_attention_heads=4,
             num_key_value_heads=2, full_attn_idxs=[1, 3], block_multiple_of=32, conv_bias=True)
    torch.manual_seed(0)
    m = Lfm2ForCausalLM(hc).eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
            else:
                p.normal_(1.0 if "norm" in n else 0.0, 0.1)
    cfg = Lfm2Config.from_dict(hc.to_dict())
    assert [cfg.is_attention(i) for i in range(4)] == [False, True, False, True]
    assert cfg.ff_dim == m.model.layers[0].feed_forward.w1.out_features
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    ids = torch.randint(0, 128, (1, 39), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = m(ids).logits[0].float()
    got = Lfm2Oracle(cfg, sd).logits(ids[0])
    err = (got - ref).abs().max() / ref.abs().max()
    assert err < 1e-4, err
