"""EnCodec on CPU against transformers' EncodecModel (the fp32 oracle): the
24 kHz layout (causal, reflect padding, weight norm), a non-causal zero-padded
variant and the 48 kHz layout (stereo, time_group_norm, RMS normalisation,
overlapping chunks): encoder latents, codes at two bandwidths, decoded audio;
a signal shorter than the padding; ``load_codec``."""
import json

import pytest
import torch

from rlx_models_b200.models.encodec import EncodecConfig, EncodecModel, random_weights

transformers = pytest.importorskip("transformers")

BASE = dict(num_filters=8, hidden_size=16, upsampling_ratios=[4, 2], codebook_size=32,
            target_bandwidths=[1.0, 2.0], sampling_rate=1600)
VARIANTS = {
    "24khz": {},
    "noncausal_zero": dict(use_causal_conv=False, pad_mode="constant"),
    "48khz": dict(norm_type="time_group_norm", use_causal_conv=False, audio_channels=2, normalize=True,
                  chunk_length_s=0.1, overlap=0.1),
}


def _pair(kw, seed=1):
    hc = transformers.EncodecConfig(**BASE, **kw)
    cfg = EncodecConfig.from_dict(hc.to_dict())
    w = random_weights(cfg, seed)
    hm = transformers.EncodecModel(hc).eval()
    hm.load_state_dict(w, strict=True)
    return cfg, w, hm, EncodecModel(cfg, w)


@pytest.mark.parametrize("variant", list(VARIANTS))
@pytest.mark.parametrize("bandwidth", [1.0, 2.0])
def test_encodec_matches_transformers(variant, bandwidth):
    cfg, _, hm, m = _pair(VARIANTS[variant])
    torch.manual_seed(0)
    x = 0.3 * torch.randn(2, cfg.audio_channels, 333)
    with torch.no_grad():
        z_ref = hm.encoder(x).transpose(1, 2)
        out = hm.encode(x, bandwidth=bandwidth)
        a_ref = hm.decode(out.audio_codes, out.audio_scales,
                          last_frame_pad_length=out.last_frame_pad_length).audio_values
    torch.testing.assert_close(m.encode_latents(x), z_ref, atol=1e-4, rtol=1e-4)
    codes, scales, pad = m.encode(x, bandwidth=bandwidth)
    assert torch.equal(codes, out.audio_codes) and pad == out.last_frame_pad_length
    assert codes.shape[2] == cfg.quantizers_for(bandwidth)
    for s, r in zip(scales, out.audio_scales):
        assert (s is None) == (r is None)
        if s is not None:
            torch.testing.assert_close(s, r)
    a = m.decode(codes, scales, pad)
    assert a.shape == a_ref.shape
    torch.testing.assert_close(a, a_ref, atol=1e-4, rtol=1e-4)


def test_encodec_signal_shorter_than_padding():
    cfg, _, hm, m = _pair({})
    x = 0.3 * torch.randn(1, 1, 5)          # the 7-tap stem pads 6 samples by reflection
    with torch.no_grad():
        z_ref = hm.encoder(x).transpose(1, 2)
    torch.testing.assert_close(m.encode_latents(x), z_ref, atol=1e-4, rtol=1e-4)


def test_load_codec_encodec(tmp_path):
    from rlx_models_b200.api import load_codec
    from rlx_models_b200.weights.safetensors_io import save_file
    hc = transformers.EncodecConfig(**BASE)
    cfg = EncodecConfig.from_dict(hc.to_dict())
    w = random_weights(cfg, 7)
    d = tmp_path / "encodec"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(hc.to_dict()))
    save_file({k: v.contiguous() for k, v in w.items()}, str(d / "model.safetensors"))
    codec = load_codec(str(d), device="cpu")
    assert isinstance(codec, EncodecModel)
    x = 0.3 * torch.randn(1, 1, 160)
    assert torch.equal(codec.encode(x)[0], EncodecModel(cfg, w).encode(x)[0])
