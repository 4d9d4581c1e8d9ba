"""LFM2-VL on CPU against transformers' Lfm2VlForConditionalGeneration (the
fp32 oracle): per-image tokens (SigLIP 2 NaFlex tower + pixel-unshuffle
projector) and prompt logits through the LFM2 hybrid LM with two images of
different aspect ratios; the placeholder count rule."""
import numpy as np
import pytest
import torch

from rlx_models_b200.models.lfm2_vl import Lfm2VlConfig, Lfm2VlModel

transformers = pytest.importorskip("transformers")

VC = dict(model_type="siglip2_vision_model", hidden_size=32, intermediate_size=64, num_hidden_layers=2,
          num_attention_heads=2, patch_size=4, num_patches=16)
TC = dict(model_type="lfm2", vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=3,
          num_attention_heads=4, num_key_value_heads=2, layer_types=["conv", "full_attention", "conv"],
          block_auto_adjust_ff_dim=False)
IMGS = [np.random.default_rng(i).integers(0, 256, s, dtype=np.uint8) for i, s in enumerate([(32, 48, 3), (40, 24, 3)])]


@pytest.fixture(scope="module")
def pair():
    torch.manual_seed(0)
    hc = transformers.Lfm2VlConfig(vision_config=VC, text_config=TC, image_token_id=120, projector_hidden_size=48)
    hm = transformers.Lfm2VlForConditionalGeneration(hc).eval()
    sd = {k: v + 0.05 * torch.randn_like(v) for k, v in hm.state_dict().items()}
    sd["lm_head.weight"] = sd["model.language_model.embed_tokens.weight"]    # tied in the checkpoints
    hm.load_state_dict(sd)
    return hm, Lfm2VlModel(Lfm2VlConfig.from_dict(hc.to_dict()), sd)


def test_prompt_logits_match_transformers(pair):
    hm, m = pair
    o = transformers.Siglip2ImageProcessor(max_num_patches=24, patch_size=4)(IMGS, return_tensors="pt")
    shapes = o["spatial_shapes"]
    n = [(h // 2) * (w // 2) for h, w in shapes.tolist()]
    ids = [1, 5] + [120] * n[0] + [7, 8] + [120] * n[1] + [9]
    with torch.no_grad():
        feats = hm.model.get_image_features(pixel_values=o["pixel_values"], spatial_shapes=shapes,
                                            pixel_attention_mask=o["pixel_attention_mask"]).pooler_output
        ref = hm(input_ids=torch.tensor([ids]), pixel_values=o["pixel_values"], spatial_shapes=shapes,
                 pixel_attention_mask=o["pixel_attention_mask"]).logits[0]
    got = m.image_features(o["pixel_values"], shapes, o["pixel_attention_mask"])
    for a, b in zip(got, feats):
        torch.testing.assert_close(a, b, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(m.oracle_logits(ids, o["pixel_values"], shapes, o["pixel_attention_mask"]), ref,
                               atol=1e-4, rtol=1e-4)


def test_image_token_count(pair):
    _, m = pair
    assert m.image_tokens(32, 48, 24) == 6 and m.image_tokens(40, 24, 24) == 6
    segs = m.segments_for_images([3] + [120] * 6 + [4], [IMGS[0]], max_patches=24)
    assert len(segs) == 1 and segs[0][0] == 1 and segs[0][1].shape[0] == 6
    with pytest.raises(ValueError):
        m.segments_for_images([3] + [120] * 5 + [4], [IMGS[0]], max_patches=24)
