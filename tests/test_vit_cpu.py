"""CLIP and SigLIP vision towers on CPU against transformers (last hidden
state, pooled output, CLIP's projected image embedding), fed by the
package's own image preprocessing."""
import math

import numpy as np
import pytest
import torch


def _rand(m):
    torch.manual_seed(0)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.numel() == 0:
                continue
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p[0].numel()))
            else:
                p.normal_(1.0 if ("norm" in n and n.endswith("weight")) else 0.0, 0.1)
    return m.eval()


def _pixels():
    from PIL import Image
    from rlx_models_b200.utils.preprocess import preprocess_image
    rng = np.random.default_rng(0)
    imgs = [Image.fromarray(rng.integers(0, 256, (50 + 7 * i, 61, 3), dtype=np.uint8)) for i in range(2)]
    return torch.stack([preprocess_image(im, size=32, crop=32) for im in imgs])


def test_clip_vision_matches_transformers():
    from transformers import CLIPVisionConfig, CLIPVisionModelWithProjection
    from rlx_models_b200.models.vit import VisionConfig, VisionEncoder
    hc = CLIPVisionConfig(hidden_size=64, intermediate_size=96, num_hidden_layers=2, num_attention_heads=4,
                          image_size=32, patch_size=8, projection_dim=48)
    m = _rand(CLIPVisionModelWithProjection(hc))
    px = _pixels()
    with torch.no_grad():
        ref = m(pixel_values=px)
    enc = VisionEncoder(VisionConfig.from_dict(hc.to_dict()), {k: v.detach() for k, v in m.state_dict().items()})
    last, _ = enc(px)
    assert (last - ref.last_hidden_state).abs().max() < 1e-4
    e = enc.embed(px, normalize=False)
    assert (e - ref.image_embeds).abs().max() < 1e-4


def test_siglip_vision_matches_transformers():
    from transformers import SiglipVisionConfig, SiglipVisionModel
    from rlx_models_b200.models.vit import VisionConfig, VisionEncoder
    hc = SiglipVisionConfig(hidden_size=64, intermediate_size=96, num_hidden_layers=2, num_attention_heads=4,
                            image_size=32, patch_size=8)
    m = _rand(SiglipVisionModel(hc))
    px = _pixels()
    with torch.no_grad():
        ref = m(pixel_values=px)
    enc = VisionEncoder(VisionConfig.from_dict(hc.to_dict()), {k: v.detach() for k, v in m.state_dict().items()})
    last, pooled = enc(px)
    assert (last - ref.last_hidden_state).abs().max() < 1e-4
    assert (pooled - ref.pooler_output).abs().max() < 1e-4


def test_load_image_embedder(tmp_path):
    import json
    from PIL import Image
    from transformers import CLIPVisionConfig, CLIPVisionModelWithProjection, CLIPImageProcessor
    from rlx_models_b200.api import load_image_embedder
    from rlx_models_b200.weights.safetensors_io import save_file
    hc = CLIPVisionConfig(hidden_size=64, intermediate_size=96, num_hidden_layers=1, num_attention_heads=4,
                          image_size=32, patch_size=8, projection_dim=48)
    m = _rand(CLIPVisionModelWithProjection(hc))
    d = tmp_path / "clipv"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(hc.to_dict()))
    save_file({k: v.detach().contiguous() for k, v in m.state_dict().items()}, str(d / "model.safetensors"))
    img = Image.fromarray(np.random.default_rng(3).integers(0, 256, (40, 48, 3), dtype=np.uint8))
    e = load_image_embedder(str(d), device="cpu").embed(img)
    px = CLIPImageProcessor(size={"shortest_edge": 32}, crop_size={"height": 32, "width": 32})(
        img, return_tensors="pt")["pixel_values"]
    with torch.no_grad():
        r = torch.nn.functional.normalize(m(pixel_values=px).image_embeds, dim=-1)
    assert (e - r).abs().max() < 2e-2  # the resampler's 8-bit rounding on a few pixels


def test_clip_dual_encoder_matches_transformers(tmp_path):
    import json
    from transformers import CLIPConfig, CLIPModel
    from rlx_models_b200.api import load_clip
    from rlx_models_b200.weights.safetensors_io import save_file
    cfg = CLIPConfig(text_config=dict(vocab_size=99, hidden_size=64, intermediate_size=96, num_hidden_layers=2,
                                      num_attention_heads=4, max_position_embeddings=16, eos_token_id=98),
                     vision_config=dict(hidden_size=64, intermediate_size=96, num_hidden_layers=2,
                                        num_attention_heads=4, image_size=32, patch_size=8),
                     projection_dim=40)
    m = _rand(CLIPModel(cfg))
    with torch.no_grad():
        m.logit_scale.fill_(2.0)
    d = tmp_path / "clip"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(cfg.to_dict()))
    save_file({k: v.detach().contiguous() for k, v in m.state_dict().items()}, str(d / "model.safetensors"))
    clip = load_clip(str(d), device="cpu")
    ids = torch.randint(1, 98, (3, 16), generator=torch.Generator().manual_seed(4))
    ids[:, 10] = 98  # end-of-text
    px = _pixels()
    with torch.no_grad():
        ref = m(input_ids=ids, pixel_values=px).logits_per_image
    got = clip.model.logits_per_image(px, ids)
    assert (got - ref).abs().max() < 1e-3


def _dinov2_case(registers: bool, swiglu: bool, size: int):
    import transformers as T
    from rlx_models_b200.models.vit import Dinov2Config, Dinov2Encoder
    kw = dict(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, image_size=28, patch_size=7,
              use_swiglu_ffn=swiglu, layerscale_value=0.5)
    if registers:
        hc = T.Dinov2WithRegistersConfig(num_register_tokens=3, **kw)
        m = _rand(T.Dinov2WithRegistersModel(hc))
    else:
        hc = T.Dinov2Config(**kw)
        m = _rand(T.Dinov2Model(hc))
    torch.manual_seed(1)
    px = torch.randn(2, 3, size, size)
    with torch.no_grad():
        ref = m(pixel_values=px)
    enc = Dinov2Encoder(Dinov2Config.from_dict(hc.to_dict()), {k: v.detach() for k, v in m.state_dict().items()})
    last, pooled = enc(px)
    assert last.shape == ref.last_hidden_state.shape
    assert (last - ref.last_hidden_state).abs().max() < 2e-4
    assert (pooled - ref.pooler_output).abs().max() < 2e-4


def test_dinov2_matches_transformers():
    _dinov2_case(registers=False, swiglu=False, size=28)


def test_dinov2_interpolated_positions_and_swiglu():
    _dinov2_case(registers=False, swiglu=True, size=42)


def test_dinov2_with_registers_matches_transformers():
    _dinov2_case(registers=True, swiglu=False, size=35)


def test_load_image_embedder_dinov2(tmp_path):
    import json
    from PIL import Image
    import transformers as T
    from rlx_models_b200.api import load_image_embedder
    from rlx_models_b200.weights.safetensors_io import save_file
    hc = T.Dinov2Config(hidden_size=64, num_hidden_layers=1, num_attention_heads=4, image_size=56, patch_size=14)
    m = _rand(T.Dinov2Model(hc))
    d = tmp_path / "dino"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(hc.to_dict()))
    save_file({k: v.detach().contiguous() for k, v in m.state_dict().items()}, str(d / "model.safetensors"))
    img = Image.fromarray(np.random.default_rng(4).integers(0, 256, (300, 260, 3), dtype=np.uint8))
    e = load_image_embedder(str(d), device="cpu").embed(img)
    px = T.BitImageProcessor(size={"shortest_edge": 256}, crop_size={"height": 224, "width": 224},
                             image_mean=[0.485, 0.456, 0.406], image_std=[0.229, 0.224, 0.225])(
        img, return_tensors="pt")["pixel_values"]
    with torch.no_grad():
        r = torch.nn.functional.normalize(m(pixel_values=px).pooler_output, dim=-1)
    assert (e - r).abs().max() < 2e-2


@pytest.mark.parametrize("gated,regs,size", [(False, 0, 28), (True, 2, 42)])
def test_dinov3_matches_transformers(gated, regs, size):
    import transformers as T
    from rlx_models_b200.models.vit import Dinov3Config, Dinov3Encoder
    hc = T.DINOv3ViTConfig(hidden_size=64, intermediate_size=96, num_hidden_layers=2, num_attention_heads=4,
                           image_size=28, patch_size=7, num_register_tokens=regs, use_gated_mlp=gated,
                           hidden_act="silu" if gated else "gelu", layerscale_value=0.5)
    m = _rand(T.DINOv3ViTModel(hc))
    px = torch.randn(2, 3, size, size, generator=torch.Generator().manual_seed(3))
    with torch.no_grad():
        ref = m(pixel_values=px)
    enc = Dinov3Encoder(Dinov3Config.from_dict(hc.to_dict()), {k: v.detach() for k, v in m.state_dict().items()})
    last, pooled = enc(px)
    assert last.shape == ref.last_hidden_state.shape
    assert (last - ref.last_hidden_state).abs().max() < 2e-4
    assert (pooled - ref.pooler_output).abs().max() < 2e-4
