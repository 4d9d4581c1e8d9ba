"""SigLIP 2 (NaFlex) on CPU against transformers' Siglip2VisionModel (the fp32
oracle): last hidden states of valid patches and the attention-pooled output
for a batch of images at different aspect ratios (padded patch sequences);
the NaFlex sizing rule and patchification against the SigLIP 2 processor;
``load_image_embedder``."""
import json

import numpy as np
import pytest
import torch

from rlx_models_b200.models.vit import Siglip2Encoder, VisionConfig, naflex_size

transformers = pytest.importorskip("transformers")

VC = dict(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4, patch_size=4,
          num_patches=16)


@pytest.fixture(scope="module")
def pair():
    torch.manual_seed(0)
    hm = transformers.Siglip2VisionModel(transformers.Siglip2VisionConfig(**VC)).eval()
    sd = {k: v + 0.05 * torch.randn_like(v) for k, v in hm.state_dict().items()}
    hm.load_state_dict(sd)
    cfg = VisionConfig.from_dict({**hm.config.to_dict(), "image_size": 16})
    return hm, sd, Siglip2Encoder(cfg, sd)


IMGS = [np.random.default_rng(i).integers(0, 256, s, dtype=np.uint8) for i, s in enumerate([(30, 50, 3), (40, 20, 3)])]


def test_naflex_forward_matches_transformers(pair):
    hm, _, m = pair
    o = transformers.Siglip2ImageProcessor(max_num_patches=24, patch_size=4)(IMGS, return_tensors="pt")
    with torch.no_grad():
        ref = hm(pixel_values=o["pixel_values"], pixel_attention_mask=o["pixel_attention_mask"],
                 spatial_shapes=o["spatial_shapes"])
    x, pooled = m.forward_patches(o["pixel_values"], o["spatial_shapes"], o["pixel_attention_mask"])
    v = o["pixel_attention_mask"].bool()
    torch.testing.assert_close(x[v], ref.last_hidden_state[v], atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(pooled, ref.pooler_output, atol=1e-4, rtol=1e-4)


def test_naflex_preprocessing_matches_processor(pair):
    _, _, m = pair
    o = transformers.Siglip2ImageProcessor(max_num_patches=24, patch_size=4)(IMGS, return_tensors="pt")
    patches, shapes, valid = m.patchify(IMGS, 24)
    assert torch.equal(shapes, o["spatial_shapes"]) and torch.equal(valid, o["pixel_attention_mask"].bool())
    torch.testing.assert_close(patches, o["pixel_values"], atol=2e-2, rtol=0)     # resampler rounding
    for h, w in ((30, 50), (40, 20), (7, 300), (256, 256)):
        th, tw = naflex_size(h, w, 16, 256)
        assert th % 16 == 0 and tw % 16 == 0 and (th // 16) * (tw // 16) <= 256


def test_load_image_embedder_siglip2(pair, tmp_path):
    from rlx_models_b200.api import load_image_embedder
    from rlx_models_b200.weights.safetensors_io import save_file
    hm, sd, m = pair
    d = tmp_path / "siglip2"
    d.mkdir()
    (d / "config.json").write_text(json.dumps({**hm.config.to_dict(), "image_size": 16}))
    save_file({k: v.contiguous() for k, v in sd.items()}, str(d / "model.safetensors"))
    e = load_image_embedder(str(d), device="cpu").embed(IMGS)
    assert e.shape == (2, 64)
    torch.testing.assert_close(e, m.embed_images(IMGS, 256))
