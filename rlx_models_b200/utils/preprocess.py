"""Image and audio front-end helpers for the vision / audio model families.

Images (PIL in, fp32 CHW tensors out), in the order the CLIP / SigLIP
processors apply them: resize (shortest edge to ``size`` keeping the aspect
ratio, or to a fixed (h, w)) with PIL's resampling filters on the 8-bit
image, center crop, rescale by 1/255, per-channel normalisation; plus ViT
patchification.

Audio: mel filter banks (HTK or Slaney mel scale, optional Slaney area
normalisation) built from the mel-scale formulas, a power / magnitude STFT
(reflect-padded, periodic Hann window), and log-mel spectrograms.

Reference: crates/rlx-models-core src/image_preprocess.rs (518 lines),
src/audio_ops_ir.rs (mel / STFT ops); transformers' image processors and
``audio_utils`` are the CPU oracles in the tests.
"""
from __future__ import annotations

import math

import torch

CLIP_MEAN = (0.48145466, 0.4578275, 0.40821073)
CLIP_STD = (0.26862954, 0.26130258, 0.27577711)
IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)
HALF = (0.5, 0.5, 0.5)

_RESAMPLE = {"nearest": 0, "bilinear": 2, "bicubic": 3, "lanczos": 1}


# ---------------------------------------------------------------------------
# images
# ---------------------------------------------------------------------------

def load_image(img):
    """A path, PIL image or HWC uint8 array -> RGB PIL image."""
    from PIL import Image
    if isinstance(img, str):
        img = Image.open(img)
    elif not isinstance(img, Image.Image):
        import numpy as np
        img = Image.fromarray(np.asarray(img))
    return img.convert("RGB")


def resize(img, size, resample: str = "bicubic"):
    """``size`` int: the shortest edge becomes ``size`` (the other edge scales
    with it, truncated); (h, w): exact size."""
    w, h = img.size
    if isinstance(size, int):
        if w <= h:
            new_w, new_h = size, int(size * h / w)
        else:
            new_h, new_w = size, int(size * w / h)
    else:
        new_h, new_w = size
    return img.resize((new_w, new_h), resample=_RESAMPLE[resample])


def center_crop(img, size):
    h, w = (size, size) if isinstance(size, int) else size
    W, H = img.size
    top, left = (H - h) // 2, (W - w) // 2
    return img.crop((left, top, left + w, top + h))


def to_tensor(img, rescale: float = 1.0 / 255.0) -> torch.Tensor:
    """PIL RGB -> fp32 [3, H, W] scaled by ``rescale``."""
    import numpy as np
    a = torch.from_numpy(np.asarray(img, dtype=np.uint8).copy())
    return a.permute(2, 0, 1).float() * rescale


def normalize(t: torch.Tensor, mean, std) -> torch.Tensor:
    m = torch.tensor(mean, dtype=t.dtype)[:, None, None]
    s = torch.tensor(std, dtype=t.dtype)[:, None, None]
    return (t - m) / s


def preprocess_image(img, size=224, crop=224, mean=CLIP_MEAN, std=CLIP_STD, resample: str = "bicubic"):
    """load -> resize -> (center crop) -> rescale -> normalise: [3, H, W] fp32.
    CLIP: size=224 (shortest edge), crop=224; SigLIP: size=(224, 224), crop=None,
    mean=std=(0.5, 0.5, 0.5)."""
    img = resize(load_image(img), size, resample)
    if crop is not None:
        img = center_crop(img, crop)
    return normalize(to_tensor(img), mean, std)


def patchify(t: torch.Tensor, patch: int) -> torch.Tensor:
    """[C, H, W] -> [(H/p)(W/p), C p p] patch rows (row-major over the grid,
    channel-major within a patch, the order of a stride-p conv's weights)."""
    C, H, W = t.shape
    x = t.view(C, H // patch, patch, W // patch, patch).permute(1, 3, 0, 2, 4)
    return x.reshape((H // patch) * (W // patch), C * patch * patch)


# ---------------------------------------------------------------------------
# audio
# ---------------------------------------------------------------------------

def hz_to_mel(f, scale: str = "htk"):
    f = torch.as_tensor(f, dtype=torch.float64)
    if scale == "htk":
        return 2595.0 * torch.log10(1.0 + f / 700.0)
    # Slaney: linear below 1 kHz, logarithmic above
    lin = f / (200.0 / 3)
    log = 15.0 + torch.log(f / 1000.0) / (math.log(6.4) / 27.0)
    return torch.where(f >= 1000.0, log, lin)


def mel_to_hz(m, scale: str = "htk"):
    m = torch.as_tensor(m, dtype=torch.float64)
    if scale == "htk":
        return 700.0 * (10.0 ** (m / 2595.0) - 1.0)
    lin = m * (200.0 / 3)
    log = 1000.0 * torch.exp((math.log(6.4) / 27.0) * (m - 15.0))
    return torch.where(m >= 15.0, log, lin)


def mel_filter_bank(n_freqs: int, n_mels: int, f_min: float, f_max: float, sample_rate: int,
                    norm: str | None = None, mel_scale: str = "htk") -> torch.Tensor:
    """[n_freqs, n_mels] triangular filters over the FFT bins 0 .. sr/2: mel
    centres equally spaced between f_min and f_max (n_mels + 2 edges); with
    norm="slaney" each filter is divided by its width in Hz / 2 (equal area)."""
    edges = mel_to_hz(torch.linspace(float(hz_to_mel(f_min, mel_scale)), float(hz_to_mel(f_max, mel_scale)),
                                     n_mels + 2, dtype=torch.float64), mel_scale)
    fft = torch.linspace(0, sample_rate / 2, n_freqs, dtype=torch.float64)
    lo, mid, hi = edges[:-2], edges[1:-1], edges[2:]
    up = (fft[:, None] - lo[None]) / (mid - lo)[None]
    down = (hi[None] - fft[:, None]) / (hi - mid)[None]
    fb = torch.clamp(torch.minimum(up, down), min=0.0)
    if norm == "slaney":
        fb = fb * (2.0 / (hi - lo))[None]
    return fb.float()


def stft(audio: torch.Tensor, n_fft: int, hop: int, power: float = 2.0, center: bool = True) -> torch.Tensor:
    """|STFT|^power [n_fft/2 + 1, frames] with a periodic Hann window and
    reflect padding of n_fft / 2 on both sides when ``center``."""
    win = torch.hann_window(n_fft, periodic=True, dtype=torch.float64)
    spec = torch.stft(audio.double(), n_fft, hop, window=win, center=center, pad_mode="reflect", return_complex=True)
    return spec.abs().pow(power).float()


def log_mel_spectrogram(audio: torch.Tensor, sample_rate: int, n_fft: int, hop: int, n_mels: int,
                        f_min: float = 0.0, f_max: float | None = None, norm: str | None = None,
                        mel_scale: str = "htk", floor: float = 1e-10) -> torch.Tensor:
    """log10(max(mel power, floor)) [n_mels, frames]."""
    fb = mel_filter_bank(n_fft // 2 + 1, n_mels, f_min, f_max or sample_rate / 2, sample_rate, norm, mel_scale)
    mel = fb.t() @ stft(audio, n_fft, hop)
    return torch.log10(torch.clamp(mel, min=floor))
