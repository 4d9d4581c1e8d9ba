"""Image and audio front-end helpers against transformers' CLIP / SigLIP
image processors and audio_utils (mel filter banks, spectrograms)."""
import numpy as np
import pytest
import torch

from rlx_models_b200.utils import preprocess as P


def _image(h=211, w=317, seed=0):
    from PIL import Image
    rng = np.random.default_rng(seed)
    return Image.fromarray(rng.integers(0, 256, (h, w, 3), dtype=np.uint8))


def _close(got, ref):
    """Equal up to one 8-bit step of the resized image on a few pixels (the
    resampler's rounding), exact elsewhere."""
    d = (got - ref).abs()
    assert got.shape == ref.shape and d.max() < 1.01 / 255 / min(P.CLIP_STD)
    assert (d > 1e-4).float().mean() < 0.01


@pytest.mark.parametrize("hw", [(211, 317), (400, 150)])
def test_clip_and_siglip_preprocessing(hw):
    from transformers import CLIPImageProcessor, SiglipImageProcessor
    img = _image(*hw)
    ref = CLIPImageProcessor(size={"shortest_edge": 224}, crop_size={"height": 224, "width": 224})(
        img, return_tensors="pt")["pixel_values"][0]
    got = P.preprocess_image(img, size=224, crop=224)
    _close(got, ref)
    ref = SiglipImageProcessor(size={"height": 224, "width": 224})(img, return_tensors="pt")["pixel_values"][0]
    got = P.preprocess_image(img, size=(224, 224), crop=None, mean=P.HALF, std=P.HALF)
    _close(got, ref)


def test_patchify_matches_conv():
    t = torch.randn(3, 32, 48)
    w = torch.randn(5, 3, 16, 16)
    conv = torch.nn.functional.conv2d(t[None], w, stride=16)[0]  # [5, 2, 3]
    rows = P.patchify(t, 16) @ w.reshape(5, -1).t()  # [6, 5]
    assert torch.allclose(rows.t().reshape(5, 2, 3), conv, atol=1e-4)


@pytest.mark.parametrize("scale,norm", [("htk", None), ("slaney", "slaney"), ("htk", "slaney")])
def test_mel_filter_bank(scale, norm):
    from transformers.audio_utils import mel_filter_bank
    ref = mel_filter_bank(num_frequency_bins=201, num_mel_filters=40, min_frequency=20.0, max_frequency=7600.0,
                          sampling_rate=16000, norm=norm, mel_scale=scale)
    got = P.mel_filter_bank(201, 40, 20.0, 7600.0, 16000, norm, scale)
    assert np.allclose(got.numpy(), ref, atol=1e-6)


def test_log_mel_spectrogram():
    from transformers.audio_utils import mel_filter_bank, spectrogram, window_function
    rng = np.random.default_rng(1)
    audio = rng.standard_normal(16000).astype(np.float32) * 0.1
    fb = mel_filter_bank(num_frequency_bins=201, num_mel_filters=64, min_frequency=0.0, max_frequency=8000.0,
                         sampling_rate=16000, norm="slaney", mel_scale="slaney")
    ref = spectrogram(audio, window_function(400, "hann"), frame_length=400, hop_length=160, power=2.0,
                      mel_filters=fb, log_mel="log10", mel_floor=1e-10)
    got = P.log_mel_spectrogram(torch.from_numpy(audio), 16000, 400, 160, 64, norm="slaney", mel_scale="slaney")
    assert got.shape == ref.shape and np.abs(got.numpy() - ref).max() < 1e-3
