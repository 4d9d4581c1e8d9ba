"""Encoder families on the GPU (bf16 GEMMs) against their CPU fp32 paths:
NomicBERT text embeddings, CLIP and DINOv2 image embeddings, Parakeet CTC logits, Moonshine decoder logits."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rand(m):
    torch.manual_seed(0)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p[0].numel()))
            else:
                p.normal_(1.0 if n.endswith("weight") else 0.0, 0.1)
    return m.eval()


def _cos(a, b):
    return torch.nn.functional.cosine_similarity(a.float().cpu(), b.float().cpu(), dim=-1)


def test_nomic_bert_gpu_matches_cpu(cuda):
    from transformers import NomicBertConfig as HFC, NomicBertModel
    from rlx_models_b200.models.bert import NomicBertConfig, NomicBertEncoder
    hc = HFC(vocab_size=128, hidden_size=256, num_hidden_layers=2, num_attention_heads=4, intermediate_size=512)
    sd = {k: v.detach() for k, v in _rand(NomicBertModel(hc)).state_dict().items()}
    cfg = NomicBertConfig.from_dict(hc.to_dict())
    ids = torch.randint(1, 128, (3, 20), generator=torch.Generator().manual_seed(1))
    mask = torch.ones(3, 20, dtype=torch.long)
    mask[2, 11:] = 0
    ref = NomicBertEncoder(cfg, sd).embed(ids, mask)
    got = NomicBertEncoder(cfg, sd, device=cuda).embed(ids, mask)
    assert _cos(got, ref).min() > 0.999


def test_clip_vision_gpu_matches_cpu(cuda):
    from transformers import CLIPVisionConfig, CLIPVisionModelWithProjection
    from rlx_models_b200.models.vit import VisionConfig, VisionEncoder
    from rlx_models_b200.utils.preprocess import preprocess_image
    hc = CLIPVisionConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                          image_size=64, patch_size=16, projection_dim=128)
    sd = {k: v.detach() for k, v in _rand(CLIPVisionModelWithProjection(hc)).state_dict().items()}
    cfg = VisionConfig.from_dict(hc.to_dict())
    rng = np.random.default_rng(0)
    px = torch.stack([preprocess_image(rng.integers(0, 256, (70, 90, 3), dtype=np.uint8), size=64, crop=64)
                      for _ in range(2)])
    ref = VisionEncoder(cfg, sd).embed(px)
    got = VisionEncoder(cfg, sd, device=cuda).embed(px)
    assert _cos(got, ref).min() > 0.999


@pytest.mark.parametrize("registers", [False, True])
def test_dinov2_gpu_matches_cpu(cuda, registers):
    import transformers as T
    from rlx_models_b200.models.vit import Dinov2Config, Dinov2Encoder
    kw = dict(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, image_size=56, patch_size=14)
    if registers:
        hc = T.Dinov2WithRegistersConfig(num_register_tokens=4, **kw)
        m = T.Dinov2WithRegistersModel(hc)
    else:
        hc = T.Dinov2Config(**kw)
        m = T.Dinov2Model(hc)
    sd = {k: v.detach() for k, v in _rand(m).state_dict().items()}
    cfg = Dinov2Config.from_dict(hc.to_dict())
    px = torch.randn(2, 3, 112, 112, generator=torch.Generator().manual_seed(2))
    ref = Dinov2Encoder(cfg, sd).embed(px)
    got = Dinov2Encoder(cfg, sd, device=cuda).embed(px)
    assert _cos(got, ref).min() > 0.999


def test_parakeet_ctc_gpu_matches_cpu(cuda):
    import transformers as T
    from rlx_models_b200.models.parakeet import ParakeetConfig, ParakeetCTC
    enc = dict(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, intermediate_size=512,
               conv_kernel_size=9, subsampling_factor=8, subsampling_conv_channels=32, num_mel_bins=80)
    hc = T.ParakeetCTCConfig(encoder_config=enc, vocab_size=129, pad_token_id=128)
    sd = {k: v.detach() for k, v in _rand(T.ParakeetForCTC(hc)).state_dict().items()}
    cfg = ParakeetConfig.from_dict(hc.to_dict())
    feats = torch.randn(2, 200, 80, generator=torch.Generator().manual_seed(3))
    ref, _ = ParakeetCTC(cfg, sd).logits(feats, torch.tensor([200, 150]))
    got, n = ParakeetCTC(cfg, sd, device=cuda).logits(feats, torch.tensor([200, 150]))
    assert _cos(got[0], ref[0]).min() > 0.995
    assert _cos(got[1, :int(n[1])], ref[1, :int(n[1])]).min() > 0.995


def test_dinov3_gpu_matches_cpu(cuda):
    import transformers as T
    from rlx_models_b200.models.vit import Dinov3Config, Dinov3Encoder
    hc = T.DINOv3ViTConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                           image_size=64, patch_size=16, num_register_tokens=4, use_gated_mlp=True, hidden_act="silu")
    sd = {k: v.detach() for k, v in _rand(T.DINOv3ViTModel(hc)).state_dict().items() if v.numel()}
    cfg = Dinov3Config.from_dict(hc.to_dict())
    px = torch.randn(2, 3, 96, 96, generator=torch.Generator().manual_seed(2))
    ref = Dinov3Encoder(cfg, sd).embed(px)
    got = Dinov3Encoder(cfg, sd, device=cuda).embed(px)
    assert _cos(got, ref).min() > 0.999


def test_moonshine_gpu_matches_cpu(cuda):
    import transformers as T
    from rlx_models_b200.models.moonshine import MoonshineConfig, MoonshineModel
    hc = T.MoonshineConfig(vocab_size=256, hidden_size=256, intermediate_size=512, encoder_num_hidden_layers=2,
                           decoder_num_hidden_layers=2, encoder_num_attention_heads=4, decoder_num_attention_heads=4,
                           encoder_num_key_value_heads=4, decoder_num_key_value_heads=4)
    sd = {k: v.detach() for k, v in _rand(T.MoonshineForConditionalGeneration(hc)).state_dict().items()}
    cfg = MoonshineConfig.from_dict(hc.to_dict())
    audio = torch.randn(1, 32000, generator=torch.Generator().manual_seed(4)) * 0.3
    ids = torch.tensor([[1, 7, 19, 200, 42]])
    ref_m, got_m = MoonshineModel(cfg, sd), MoonshineModel(cfg, sd, device=cuda)
    ref = ref_m.decode_step(ids, 0, [None] * 2, ref_m._cross_kv(ref_m.encode(audio)))
    got = got_m.decode_step(ids, 0, [None] * 2, got_m._cross_kv(got_m.encode(audio)))
    assert _cos(got[0], ref[0]).min() > 0.995
