"""DAC codec on CPU against transformers' DacModel (the fp32 oracle): encoder
latents, RVQ codes, dequantised latents and decoded audio; weight-norm folding
in both serialised forms; the original Descript checkpoint names; the torch
statements of the snake-im2col / transposed-conv fold kernels against
F.conv1d / F.conv_transpose1d."""
import math
import re

import pytest
import torch
import torch.nn.functional as F

from rlx_models_b200.models.dac import DacConfig, DacModel, random_weights
from rlx_models_b200.ops import reference as R

transformers = pytest.importorskip("transformers")

HF_CFG = dict(encoder_hidden_size=8, downsampling_ratios=[2, 4, 5], decoder_hidden_size=64,
              upsampling_ratios=[5, 4, 2], n_codebooks=4, codebook_size=32, codebook_dim=8, hidden_size=48,
              hop_length=40, sampling_rate=16000)


def _hf(w, weight_norm=False):
    hm = transformers.DacModel(transformers.DacConfig(**HF_CFG)).eval()
    if weight_norm:
        hm.apply_weight_norm()
    hm.load_state_dict(w, strict=True)
    return hm


@pytest.mark.parametrize("k,s,p,pr,d", [(7, 1, 3, 3, 1), (7, 1, 9, 9, 3), (4, 2, 1, 1, 1), (10, 5, 3, 3, 1),
                                        (3, 1, 1, 1, 1), (7, 1, 6, 0, 1), (4, 2, 2, 3, 1)])
@pytest.mark.parametrize("act", [None, "snake", "elu", "gelu"])
@pytest.mark.parametrize("reflect", [False, True])
def test_act_im2col_is_conv1d(k, s, p, pr, d, act, reflect):
    torch.manual_seed(0)
    B, T, C, O = 2, 37, 5, 6
    x, a = torch.randn(B, T, C), torch.rand(C) + 0.5
    W, b = torch.randn(O, C, k), torch.randn(O)
    xa = {"snake": lambda t: R.snake(t, a), "elu": F.elu, "gelu": F.gelu, None: lambda t: t}[act](x)
    xp = F.pad(xa.transpose(1, 2), (p, pr), mode="reflect" if reflect else "constant")
    ref = F.conv1d(xp, W, b, stride=s, dilation=d).transpose(1, 2)
    cols = R.act_im2col(x, k, s, p, pr, d, act, a, reflect)
    assert cols.shape[1] % 8 == 0
    Wg = F.pad(W.permute(0, 2, 1).reshape(O, k * C), (0, cols.shape[1] - k * C))
    torch.testing.assert_close((cols @ Wg.t() + b).reshape(B, -1, O), ref, atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("s,p,pr", [(2, 1, 1), (5, 3, 3), (8, 4, 4), (4, 0, 4), (5, 1, 4)])
def test_convt_fold_is_conv_transpose(s, p, pr):
    torch.manual_seed(0)
    B, T, C, O = 2, 11, 8, 6
    k = 2 * s
    x, W, b = torch.randn(B, T, C), torch.randn(C, O, k), torch.randn(O)
    full = F.conv_transpose1d(x.transpose(1, 2), W, b, stride=s).transpose(1, 2)
    ref = full[:, p:full.shape[1] - pr]
    Y = (x.reshape(-1, C) @ W.permute(2, 1, 0).reshape(k * O, C).t()).reshape(B, T, k * O)
    torch.testing.assert_close(R.convt_fold(Y, b, O, s, p, pr), ref, atol=1e-4, rtol=1e-4)


def test_lstm_cell_is_torch_lstm():
    torch.manual_seed(0)
    T, B, H = 9, 3, 16
    lstm = torch.nn.LSTM(H, H, 1)
    x = torch.randn(T, B, H)
    with torch.no_grad():
        ref = lstm(x)[0]
        G = x @ lstm.weight_ih_l0.t() + lstm.bias_ih_l0 + lstm.bias_hh_l0
        h, c = torch.zeros(B, H), torch.zeros(B, H)
        out = []
        for t in range(T):
            h, c = R.lstm_cell(G[t] + h @ lstm.weight_hh_l0.t(), c)
            out.append(h)
    torch.testing.assert_close(torch.stack(out), ref, atol=1e-5, rtol=1e-5)


def test_dac_matches_transformers():
    cfg = DacConfig.from_dict(HF_CFG)
    w = random_weights(cfg, 1)
    hm, m = _hf(w), DacModel(cfg, w)
    torch.manual_seed(0)
    x = 0.3 * torch.randn(2, 400)
    with torch.no_grad():
        enc = hm.encode(x[:, None])
        z_ref = hm.encoder(x[:, None]).transpose(1, 2)
        pre = hm.decoder.conv2(hm.decoder.snake1(
            torch.nn.Sequential(hm.decoder.conv1, *hm.decoder.block)(enc.quantized_representation)))
    z = m.encode_latents(x)
    torch.testing.assert_close(z, z_ref, atol=1e-3 * z_ref.abs().max().item(), rtol=1e-4)
    codes, zq = m.quantize(z)
    assert torch.equal(codes, enc.audio_codes)
    torch.testing.assert_close(zq, enc.quantized_representation.transpose(1, 2), atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(m.dequantize(codes), zq, atol=1e-4, rtol=1e-4)
    with torch.no_grad():
        a_ref = hm.decode(audio_codes=enc.audio_codes).audio_values
    a = m.decode(codes)
    assert a.shape == a_ref.shape
    torch.testing.assert_close(a, a_ref, atol=1e-3, rtol=1e-3)
    # the pre-tanh signal too (tanh saturates with random weights)
    y = m._conv(m._dec_body(zq), "decoder.conv2", "decoder.snake1", pad=3)[..., 0]
    torch.testing.assert_close(y, pre[:, 0], atol=1e-4 * pre.abs().max().item(), rtol=1e-4)


def test_dac_fewer_quantizers_and_roundtrip():
    cfg = DacConfig.from_dict(HF_CFG)
    w = random_weights(cfg, 2)
    hm, m = _hf(w), DacModel(cfg, w)
    x = 0.3 * torch.randn(1, 390)   # not a multiple of the hop: right-padded to 400
    with torch.no_grad():
        enc = hm.encode(F.pad(x, (0, 10))[:, None], n_quantizers=2)
    codes = m.encode(x, n_quantizers=2)
    assert codes.shape == (1, 2, 10) and torch.equal(codes, enc.audio_codes)
    codes_all, rec = m.roundtrip(x[0])
    assert codes_all.shape == (1, 4, 10) and rec.shape == (1, 390)


def test_weight_norm_folding():
    cfg = DacConfig.from_dict(HF_CFG)
    wn = random_weights(cfg, 3, weight_norm=True)
    param = {re.sub(r"\.weight_g$", ".parametrizations.weight.original0",
                    re.sub(r"\.weight_v$", ".parametrizations.weight.original1", k)): v for k, v in wn.items()}
    hm = _hf(param, weight_norm=True)
    x = 0.3 * torch.randn(1, 200)
    with torch.no_grad():
        z_ref = hm.encoder(x[:, None]).transpose(1, 2)
    for src in (wn, param):
        z = DacModel(cfg, src).encode_latents(x)
        torch.testing.assert_close(z, z_ref, atol=1e-3 * z_ref.abs().max().item(), rtol=1e-4)


def _to_descript(name: str, n_enc: int, n_dec: int) -> str:
    res = {"snake1": 0, "conv1": 1, "snake2": 2, "conv2": 3}
    m = re.match(r"encoder\.block\.(\d+)\.res_unit(\d)\.(\w+)\.(.*)$", name)
    if m:
        return f"encoder.block.{int(m[1]) + 1}.block.{int(m[2]) - 1}.block.{res[m[3]]}.{m[4]}"
    m = re.match(r"encoder\.block\.(\d+)\.(snake1|conv1)\.(.*)$", name)
    if m:
        return f"encoder.block.{int(m[1]) + 1}.block.{3 if m[2] == 'snake1' else 4}.{m[3]}"
    m = re.match(r"decoder\.block\.(\d+)\.res_unit(\d)\.(\w+)\.(.*)$", name)
    if m:
        return f"decoder.model.{int(m[1]) + 1}.block.{int(m[2]) + 1}.block.{res[m[3]]}.{m[4]}"
    m = re.match(r"decoder\.block\.(\d+)\.(snake1|conv_t1)\.(.*)$", name)
    if m:
        return f"decoder.model.{int(m[1]) + 1}.block.{0 if m[2] == 'snake1' else 1}.{m[3]}"
    top = {"encoder.conv1": "encoder.block.0", "encoder.snake1": f"encoder.block.{n_enc + 1}",
           "encoder.conv2": f"encoder.block.{n_enc + 2}", "decoder.conv1": "decoder.model.0",
           "decoder.snake1": f"decoder.model.{n_dec + 1}", "decoder.conv2": f"decoder.model.{n_dec + 2}"}
    for a, b in top.items():
        if name.startswith(a + "."):
            return b + name[len(a):]
    return name


def test_descript_checkpoint_names():
    cfg = DacConfig.from_dict({"encoder_dim": 8, "encoder_rates": [2, 4, 5], "decoder_dim": 64,
                               "decoder_rates": [5, 4, 2], "latent_dim": 48, "n_codebooks": 4,
                               "codebook_size": 32, "codebook_dim": 8, "sample_rate": 16000})
    assert cfg.hop_length == 40 and cfg.hidden_size == 48
    w = random_weights(cfg, 4, weight_norm=True)
    d = {_to_descript(k, 3, 3): v for k, v in w.items()}
    assert any(k.startswith("decoder.model.4.") for k in d)
    x = 0.3 * torch.randn(1, 200)
    a, b = DacModel(cfg, w), DacModel(cfg, d)
    torch.testing.assert_close(b.encode_latents(x), a.encode_latents(x))
    codes = a.encode(x)
    torch.testing.assert_close(b.decode(codes), a.decode(codes))


def test_load_codec(tmp_path):
    import json
    from rlx_models_b200.api import load_codec
    from rlx_models_b200.weights.safetensors_io import save_file
    cfg = DacConfig.from_dict(HF_CFG)
    w = random_weights(cfg, 5, weight_norm=True)
    d = tmp_path / "dac"
    d.mkdir()
    (d / "config.json").write_text(json.dumps({**HF_CFG, "model_type": "dac"}))
    save_file({k: v.contiguous() for k, v in w.items()}, str(d / "model.safetensors"))
    codec = load_codec(str(d), device="cpu")
    x = 0.3 * torch.randn(1, 120)
    torch.testing.assert_close(codec.encode(x), DacModel(cfg, w).encode(x))
