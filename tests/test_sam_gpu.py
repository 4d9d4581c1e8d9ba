"""SAM v1 on the GPU (encoder GEMMs on the tcgen05 linear, bf16) against the
fp32 CPU model: image embeddings, then masks and IoU scores for point and box
prompts."""
import pytest
import torch

from rlx_models_b200.models.sam import SamConfig, SamModel

pytestmark = pytest.mark.gpu


def test_sam_gpu_matches_cpu():
    transformers = pytest.importorskip("transformers")
    torch.manual_seed(0)
    hc = transformers.SamConfig(
        vision_config=dict(hidden_size=128, num_hidden_layers=4, num_attention_heads=4, mlp_dim=256, image_size=256,
                           patch_size=16, window_size=7, global_attn_indexes=[1, 3], output_channels=64,
                           num_pos_feats=32),
        prompt_encoder_config=dict(hidden_size=64, image_size=256, image_embedding_size=16, mask_input_channels=16),
        mask_decoder_config=dict(hidden_size=64, mlp_dim=128, num_hidden_layers=2, num_attention_heads=4,
                                 iou_head_hidden_dim=64))
    hm = transformers.SamModel(hc)
    sd = {k: (v + 0.05 * torch.randn_like(v)) if v.dtype.is_floating_point else v for k, v in hm.state_dict().items()}
    sd["prompt_encoder.shared_embedding.positional_embedding"] = sd["shared_image_embedding.positional_embedding"]
    cfg = SamConfig.from_dict(hc.to_dict())
    cpu, gpu = SamModel(cfg, sd), SamModel(cfg, sd, device="cuda")
    px = torch.randn(2, 3, 256, 256)
    e_ref, e = cpu.image_embeddings(px), gpu.image_embeddings(px).cpu()
    assert (e - e_ref).norm() / e_ref.norm() < 3e-2
    pts = torch.rand(2, 2, 1, 2) * 256
    boxes = torch.rand(2, 2, 4) * 256
    m_ref, iou_ref = cpu.segment(image_embeddings=e_ref, points=pts, boxes=boxes)
    m, iou = gpu.segment(pixels=px, points=pts, boxes=boxes)
    assert (m.cpu() - m_ref).norm() / m_ref.norm() < 5e-2
    assert (iou.cpu() - iou_ref).abs().max() < 5e-2 * iou_ref.abs().max() + 1e-3
