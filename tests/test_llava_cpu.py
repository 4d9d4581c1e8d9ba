"""LLaVA-form VLM on CPU against transformers LlavaForConditionalGeneration:
projected image features and the logits of a prompt whose image placeholder
runs carry them; both checkpoint name layouts."""
import math

import pytest
import torch


def _rand(m):
    torch.manual_seed(0)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p[0].numel()))
            else:
                p.normal_(1.0 if ("norm" in n and n.endswith("weight")) else 0.0, 0.1)
    return m.eval()


def _model(strategy="default", layer=-2):
    import transformers as T
    vc = dict(model_type="clip_vision_model", hidden_size=32, intermediate_size=64, num_hidden_layers=3,
              num_attention_heads=4, image_size=28, patch_size=14)
    tc = dict(model_type="llama", vocab_size=120, hidden_size=64, intermediate_size=96, num_hidden_layers=2,
              num_attention_heads=4, num_key_value_heads=2, rms_norm_eps=1e-6)
    cfg = T.LlavaConfig(vision_config=vc, text_config=tc, image_token_index=119,
                        vision_feature_select_strategy=strategy, vision_feature_layer=layer)
    return cfg, _rand(T.LlavaForConditionalGeneration(cfg))


@pytest.mark.parametrize("strategy,layer,legacy", [("default", -2, False), ("full", -1, True)])
def test_llava_matches_transformers(strategy, layer, legacy):
    from rlx_models_b200.models.llava import LlavaConfig, LlavaVLM
    hcfg, m = _model(strategy, layer)
    n_tok = 4 if strategy == "default" else 5
    g = torch.Generator().manual_seed(2)
    px = torch.randn(2, 3, 28, 28, generator=g)
    text = torch.randint(0, 110, (13,), generator=g).tolist()
    ids = text[:3] + [119] * n_tok + text[3:8] + [119] * n_tok + text[8:]
    with torch.no_grad():
        ref = m(input_ids=torch.tensor([ids]), pixel_values=px).logits[0]
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    if legacy:  # the earlier release layout
        ren = {}
        for k, v in sd.items():
            k2 = k.replace("model.vision_tower.", "vision_tower.").replace(
                "model.multi_modal_projector.", "multi_modal_projector.").replace(
                "model.language_model.", "language_model.model.")
            ren["language_model.lm_head.weight" if k == "lm_head.weight" else k2] = v
        sd = ren
    vlm = LlavaVLM(LlavaConfig.from_dict(hcfg.to_dict()), sd)
    lg = vlm.oracle_logits(ids, px)
    assert lg.shape == ref.shape
    assert (lg - ref).abs().max() < 2e-4
    with pytest.raises(ValueError):
        vlm.mm_segments(ids[:-8], px)  # placeholder count does not match
