"""EnCodec on the GPU (convs on the activation-fused im2col + tcgen05 GEMM,
LSTM on linear_acc + lstm_cell) against the fp32 CPU model: latents, codes
and the audio decoded from the same codes, for the 24 kHz and 48 kHz layouts."""
import pytest
import torch

from rlx_models_b200.models.encodec import EncodecConfig, EncodecModel, random_weights

pytestmark = pytest.mark.gpu

BASE = dict(num_filters=16, hidden_size=32, upsampling_ratios=[4, 2], codebook_size=64,
            target_bandwidths=[2.4, 9.6], sampling_rate=3200)


@pytest.mark.parametrize("kw", [{}, dict(norm_type="time_group_norm", use_causal_conv=False, audio_channels=2,
                                         normalize=True, chunk_length_s=0.25, overlap=0.1)])
def test_encodec_gpu_matches_cpu(kw):
    cfg = EncodecConfig(**BASE, **kw)
    w = random_weights(cfg, 3)
    cpu, gpu = EncodecModel(cfg, w), EncodecModel(cfg, w, device="cuda")
    torch.manual_seed(0)
    x = 0.3 * torch.randn(2, cfg.audio_channels, 1600)
    z_ref, z = cpu.encode_latents(x), gpu.encode_latents(x).cpu()
    assert z.shape == z_ref.shape
    assert (z - z_ref).norm() / z_ref.norm() < 3e-2
    codes_ref, scales, pad = cpu.encode(x, bandwidth=9.6)
    codes = gpu.encode(x, bandwidth=9.6)[0].cpu()
    assert codes.shape == codes_ref.shape
    assert (codes[:, :, 0] == codes_ref[:, :, 0]).float().mean() > 0.85
    a_ref = cpu.decode(codes_ref, scales, pad)
    a = gpu.decode(codes_ref.cuda(), [None if s is None else s.cuda() for s in scales], pad).cpu()
    assert a.shape == a_ref.shape
    assert (a - a_ref).norm() / a_ref.norm() < 5e-2
