"""SAM v1 on CPU against transformers' SamModel (the fp32 oracle): image
embeddings, prompt embeddings of points / boxes / masks, masks and IoU scores
with single- and multi-mask output; mask upscaling against the processor's;
``load_segmenter`` end to end."""
import json

import pytest
import torch

from rlx_models_b200.models.sam import SamConfig, SamModel, upscale_masks

transformers = pytest.importorskip("transformers")

VC = dict(hidden_size=64, num_hidden_layers=3, num_attention_heads=4, mlp_dim=128, image_size=128, patch_size=16,
          window_size=3, global_attn_indexes=[1], output_channels=32, num_pos_feats=16)
PC = dict(hidden_size=32, image_size=128, image_embedding_size=8, mask_input_channels=8)
DC = dict(hidden_size=32, mlp_dim=64, num_hidden_layers=2, num_attention_heads=4, iou_head_hidden_dim=32)


@pytest.fixture(scope="module")
def pair():
    torch.manual_seed(0)
    hc = transformers.SamConfig(vision_config=VC, prompt_encoder_config=PC, mask_decoder_config=DC)
    hm = transformers.SamModel(hc).eval()
    sd = {k: (v + 0.05 * torch.randn_like(v)) if v.dtype.is_floating_point else v for k, v in hm.state_dict().items()}
    # the prompt encoder's Fourier table is tied to the image one in the checkpoints
    sd["prompt_encoder.shared_embedding.positional_embedding"] = sd["shared_image_embedding.positional_embedding"]
    hm.load_state_dict(sd)
    return hc, hm, sd, SamModel(SamConfig.from_dict(hc.to_dict()), sd)


def test_image_embeddings(pair):
    _, hm, _, m = pair
    px = torch.randn(2, 3, 128, 128)
    with torch.no_grad():
        ref = hm.get_image_embeddings(px)
    torch.testing.assert_close(m.image_embeddings(px), ref, atol=1e-4, rtol=1e-4)


PROMPTS = {
    "points": lambda: dict(input_points=torch.rand(2, 3, 2, 2) * 128,
                           input_labels=torch.tensor([[[1, 0], [1, 1], [0, -1]]] * 2)),
    "boxes": lambda: dict(input_boxes=torch.rand(2, 3, 4) * 128),
    "points+boxes": lambda: dict(input_points=torch.rand(2, 3, 2, 2) * 128,
                                 input_labels=torch.tensor([[[1, 1], [1, 0], [0, 1]]] * 2),
                                 input_boxes=torch.rand(2, 3, 4) * 128),
    "points+mask": lambda: dict(input_points=torch.rand(2, 1, 1, 2) * 128, input_labels=torch.ones(2, 1, 1).int(),
                                input_masks=torch.randn(2, 1, 32, 32)),
}


@pytest.mark.parametrize("prompt", list(PROMPTS))
@pytest.mark.parametrize("multimask", [True, False])
def test_masks_match_transformers(pair, prompt, multimask):
    _, hm, _, m = pair
    torch.manual_seed(1)
    kw = PROMPTS[prompt]()
    px = torch.randn(2, 3, 128, 128)
    with torch.no_grad():
        out = hm(pixel_values=px, multimask_output=multimask, **kw)
    mk, iou = m.segment(pixels=px, points=kw.get("input_points"), labels=kw.get("input_labels"),
                        boxes=kw.get("input_boxes"), masks=kw.get("input_masks"), multimask=multimask)
    assert mk.shape == out.pred_masks.shape and iou.shape == out.iou_scores.shape
    scale = out.pred_masks.abs().max().item()
    torch.testing.assert_close(mk, out.pred_masks, atol=1e-4 * scale, rtol=1e-4)
    torch.testing.assert_close(iou, out.iou_scores, atol=1e-5, rtol=1e-4)


def test_upscale_masks_matches_processor():
    proc = transformers.SamImageProcessor(pad_size={"height": 128, "width": 128})
    low = torch.randn(2, 3, 32, 32)
    ref = proc.post_process_masks([low], [(90, 120)], [(96, 128)], binarize=False)[0]
    got = upscale_masks(low, (90, 120), (96, 128), pad_size=128, binarize=False)
    torch.testing.assert_close(got, ref, atol=1e-5, rtol=1e-5)


def test_load_segmenter(pair, tmp_path):
    import numpy as np

    from rlx_models_b200.api import load_segmenter
    from rlx_models_b200.weights.safetensors_io import save_file
    hc, _, sd, m = pair
    d = tmp_path / "sam"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(hc.to_dict()))
    save_file({k: v.contiguous() for k, v in sd.items()}, str(d / "model.safetensors"))
    seg = load_segmenter(str(d), device="cpu")
    img = np.random.default_rng(0).integers(0, 256, (60, 80, 3), dtype=np.uint8)
    masks, iou = seg.segment(img, points=[[[40.0, 30.0]]], labels=[[1]])
    assert masks.shape == (1, 3, 60, 80) and masks.dtype == torch.bool and iou.shape == (1, 3)
    px, orig, resized = seg.preprocess(img)
    assert orig == (60, 80) and resized == (96, 128) and px.shape == (1, 3, 128, 128)
    pts = torch.tensor([[[[40.0 * 128 / 80, 30.0 * 96 / 60]]]])
    low, iou2 = m.segment(pixels=px, points=pts, labels=torch.ones(1, 1, 1).int())
    torch.testing.assert_close(iou, iou2[0])
    masks2, _ = seg.segment(boxes=[[10.0, 10.0, 50.0, 40.0]], multimask=False)   # reuses the image
    assert masks2.shape == (1, 1, 60, 80)
