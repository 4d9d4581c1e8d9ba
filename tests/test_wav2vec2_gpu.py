"""wav2vec 2.0 CTC on the GPU (GELU-fused channels-last conv front end on the
tcgen05 GEMM, instance-norm kernel, bf16 encoder linears) against the fp32 CPU
model, for both norm layouts and a padded batch."""
import pytest
import torch

from rlx_models_b200.models.wav2vec2 import Wav2Vec2Config, Wav2Vec2CTC

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kw", [{}, dict(feat_extract_norm="layer", do_stable_layer_norm=True, conv_bias=True)])
def test_wav2vec2_gpu_matches_cpu(kw):
    transformers = pytest.importorskip("transformers")
    torch.manual_seed(0)
    hc = transformers.Wav2Vec2Config(hidden_size=128, num_hidden_layers=2, num_attention_heads=4,
                                     intermediate_size=256, conv_dim=[64] * 7, num_conv_pos_embeddings=16,
                                     num_conv_pos_embedding_groups=4, vocab_size=32, **kw)
    hm = transformers.Wav2Vec2ForCTC(hc)
    sd = {k: (v + 0.05 * torch.randn_like(v)) if v.dtype.is_floating_point else v for k, v in hm.state_dict().items()}
    cfg = Wav2Vec2Config.from_dict(hc.to_dict())
    cpu, gpu = Wav2Vec2CTC(cfg, sd), Wav2Vec2CTC(cfg, sd, device="cuda")
    x = torch.randn(2, 16000)
    x[1, 9000:] = 0
    lens = [16000, 9000]
    ref, n_ref = cpu.logits(x, lengths=lens)
    lg, n = gpu.logits(x, lengths=lens)
    assert n.tolist() == n_ref.tolist()
    for b in range(2):
        r, g = ref[b, :n[b]], lg[b, :n[b]].cpu()
        assert (g - r).norm() / r.norm() < 3e-2, b
