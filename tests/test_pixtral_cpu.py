"""Mistral-3 VLM (Pixtral tower at native image sizes + patch-merger projector
+ Mistral LM) on CPU against transformers Mistral3ForConditionalGeneration:
logits of a prompt carrying two images of different sizes, whose image tokens
come in one run per merged grid row (break tokens between rows)."""
import math

import pytest
import torch

IMG, BRK, END = 90, 91, 92


def _rand(m):
    torch.manual_seed(0)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p[0].numel()))
            else:
                p.normal_(1.0 if ("norm" in n and n.endswith("weight")) else 0.0, 0.1)
    return m.eval()


def _model():
    import transformers as T
    vc = dict(model_type="pixtral", hidden_size=32, intermediate_size=48, num_hidden_layers=2,
              num_attention_heads=4, image_size=64, patch_size=4, hidden_act="silu",
              rope_parameters={"rope_type": "default", "rope_theta": 10000.0})
    tc = dict(model_type="mistral", vocab_size=96, hidden_size=64, intermediate_size=96, num_hidden_layers=2,
              num_attention_heads=4, num_key_value_heads=2, rms_norm_eps=1e-5, head_dim=16)
    cfg = T.Mistral3Config(vision_config=vc, text_config=tc, image_token_index=IMG, spatial_merge_size=2,
                           vision_feature_layer=-1, tie_word_embeddings=False)
    return cfg, _rand(T.Mistral3ForConditionalGeneration(cfg))


def _image_ids(rows, cols):
    ids = []
    for r in range(rows):
        ids += [IMG] * cols + ([BRK] if r + 1 < rows else [END])
    return ids


def test_mistral3_matches_transformers():
    from rlx_models_b200.models.pixtral import Mistral3Config, Mistral3VLM
    hcfg, m = _model()
    g = torch.Generator().manual_seed(2)
    a = torch.randn(3, 16, 24, generator=g)  # 4 x 6 patches -> 2 x 3 merged
    b = torch.randn(3, 24, 16, generator=g)  # 6 x 4 patches -> 3 x 2 merged
    px = torch.zeros(2, 3, 24, 24)
    px[0, :, :16, :24], px[1, :, :24, :16] = a, b
    text = torch.randint(0, 85, (11,), generator=g).tolist()
    ids = text[:3] + _image_ids(2, 3) + text[3:7] + _image_ids(3, 2) + text[7:]
    with torch.no_grad():
        ref = m(input_ids=torch.tensor([ids]), pixel_values=px, image_sizes=torch.tensor([[16, 24], [24, 16]])
                ).logits[0]
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    vlm = Mistral3VLM(Mistral3Config.from_dict(hcfg.to_dict()), sd)
    segs = vlm.mm_segments(ids, [a, b])
    assert [e.shape[0] for _, e in segs] == [3, 3, 2, 2, 2]
    lg = vlm.oracle_logits(ids, [a, b])
    assert lg.shape == ref.shape
    assert (lg - ref).abs().max() < 2e-4, (lg - ref).abs().max()
    with pytest.raises(ValueError):
        vlm.mm_segments(ids, [a])  # image-token count does not match
