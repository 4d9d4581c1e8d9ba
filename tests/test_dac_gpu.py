"""Codec kernels and the DAC model on the GPU: the activation-fused channels-last
im2col (vector and scalar paths, zero and reflect padding), the transposed-conv
fold and the LSTM cell against their fp32 torch statements, and the bf16 codec
against the fp32 CPU model."""
import math

import pytest
import torch

from rlx_models_b200.models.dac import DacConfig, DacModel, random_weights
from rlx_models_b200.ops import reference as R

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("C,k,s,p,pr,d", [(16, 7, 1, 3, 3, 1), (16, 7, 1, 27, 27, 9), (32, 4, 2, 1, 1, 1),
                                           (24, 10, 5, 3, 3, 1), (1, 7, 1, 3, 3, 1), (3, 3, 1, 1, 1, 1),
                                           (64, 1, 1, 0, 0, 1), (16, 7, 1, 6, 0, 1), (8, 16, 8, 4, 5, 1)])
@pytest.mark.parametrize("act", [None, "snake", "elu", "gelu"])
@pytest.mark.parametrize("reflect", [False, True])
def test_act_im2col(C, k, s, p, pr, d, act, reflect):
    from rlx_models_b200 import ops
    torch.manual_seed(0)
    x = torch.randn(2, 301, C, device="cuda").bfloat16()
    a = (torch.rand(C, device="cuda") + 0.5) if act == "snake" else None
    got = ops.act_im2col(x, k, stride=s, pad=p, pad_right=pr, dil=d, act=act, alpha=a, reflect=reflect)
    ref = R.act_im2col(x.float(), k, s, p, pr, d, act, a, reflect)
    assert got.shape == ref.shape
    torch.testing.assert_close(got.float(), ref, atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("s,O,p,pr", [(2, 8, 1, 1), (5, 16, 3, 3), (8, 24, 4, 4), (4, 8, 0, 4), (5, 16, 1, 4)])
def test_convt_fold(s, O, p, pr):
    from rlx_models_b200 import ops
    torch.manual_seed(0)
    k = 2 * s
    Y = torch.randn(2, 37, k * O, device="cuda")
    b = torch.randn(O, device="cuda")
    got = ops.convt_fold(Y, b, O, stride=s, pad=p, pad_right=pr)
    ref = R.convt_fold(Y, b, O, s, p, pr)
    assert got.shape == ref.shape
    torch.testing.assert_close(got.float(), ref, atol=3e-2, rtol=1e-2)


def test_lstm_cell():
    from rlx_models_b200 import ops
    torch.manual_seed(0)
    B, H = 3, 64
    G = 2 * torch.randn(B, 4 * H, device="cuda")
    c = torch.randn(B, H, device="cuda")
    h_ref, c_ref = R.lstm_cell(G, c.clone())
    h = torch.empty(B, H, dtype=torch.bfloat16, device="cuda")
    y = torch.empty_like(h)
    ops.lstm_cell(G, c, h, y)
    torch.testing.assert_close(c, c_ref, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(h.float(), h_ref, atol=1e-2, rtol=1e-2)
    assert torch.equal(h, y)


def test_dac_gpu_matches_cpu():
    cfg = DacConfig(encoder_hidden_size=16, downsampling_ratios=[2, 4, 5], decoder_hidden_size=128,
                    upsampling_ratios=[5, 4, 2], n_codebooks=4, codebook_size=64, codebook_dim=8, hidden_size=64,
                    hop_length=40, sampling_rate=16000)
    w = random_weights(cfg, 1)
    cpu, gpu = DacModel(cfg, w), DacModel(cfg, w, device="cuda")
    torch.manual_seed(0)
    x = 0.3 * torch.randn(2, 4000)
    z_ref, z = cpu.encode_latents(x), gpu.encode_latents(x).cpu()
    rel = (z - z_ref).norm() / z_ref.norm()
    assert rel < 3e-2, rel
    codes_ref = cpu.encode(x)
    codes = gpu.encode(x).cpu()
    assert (codes[:, 0] == codes_ref[:, 0]).float().mean() > 0.9
    y_ref = cpu._conv(cpu._dec_body(cpu.dequantize(codes_ref)), "decoder.conv2", "decoder.snake1", pad=3)
    y = gpu._conv(gpu._dec_body(gpu.dequantize(codes_ref)), "decoder.conv2", "decoder.snake1", pad=3).float().cpu()
    assert y.shape == y_ref.shape
    assert (y - y_ref).norm() / y_ref.norm() < 5e-2
    pcm = gpu.decode(codes_ref.cuda())
    assert pcm.shape == (2, cpu.decode(codes_ref).shape[1]) and torch.isfinite(pcm).all()
