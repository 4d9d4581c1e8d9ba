"""Whisper speech recognition (the ``transcribe`` task), HF
``WhisperForConditionalGeneration`` tensor layout.

Front end: 16 kHz audio padded / trimmed to 30 s, 400-point Hann STFT with hop
160, power spectrum through a Slaney-scale, Slaney-normalised mel filter bank
(80 or 128 bins), log10 clamped at 1e-10, floored 8 decades below the
maximum, mapped as (x + 4) / 4.

Encoder: two convolutions (k3; the second with stride 2) with GELU, fixed
sinusoidal positions, pre-LayerNorm transformer blocks (q / v / out biases,
no k bias), final LayerNorm. Decoder: token + learned positions, pre-LN
blocks with causal self-attention, cross-attention over the encoder states
and a GELU MLP, final LayerNorm, output projection tied to the token
embedding. ``transcribe`` decodes greedily from the forced prefix
(<|startoftranscript|>, language, task, <|notimestamps|>) to <|endoftext|>,
with self-attention K/V cached across steps and cross-attention K/V computed
once.

GEMMs run on this package's tcgen05 linear on CUDA (bf16); attention and the
convolutions use torch (one encoder pass per 30 s window).

Reference: the reference's ASR families (crates/rlx-whisper and the audio
helpers of rlx-models-core src/audio_ops_ir.rs: mel / STFT).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .flux_text import _linear

SAMPLE_RATE = 16000
N_FFT = 400
HOP = 160
CHUNK_SECONDS = 30


@dataclass
class WhisperConfig:
    vocab_size: int = 51865
    num_mel_bins: int = 80
    d_model: int = 384
    encoder_layers: int = 4
    decoder_layers: int = 4
    encoder_attention_heads: int = 6
    decoder_attention_heads: int = 6
    encoder_ffn_dim: int = 1536
    decoder_ffn_dim: int = 1536
    max_source_positions: int = 1500
    max_target_positions: int = 448
    decoder_start_token_id: int = 50258
    eos_token_id: int = 50257
    scale_embedding: bool = False

    @classmethod
    def from_dict(cls, d: dict) -> "WhisperConfig":
        return cls(**{k: d[k] for k in cls.__dataclass_fields__ if k in d})


# ---------------------------------------------------------------------------
# log-mel front end
# ---------------------------------------------------------------------------

def _hz_to_mel(f):
    """Slaney mel scale: linear below 1 kHz, logarithmic above."""
    f = torch.as_tensor(f, dtype=torch.float64)
    lin = 3.0 * f / 200.0
    log = 15.0 + torch.log(f / 1000.0) / (math.log(6.4) / 27.0)
    return torch.where(f >= 1000.0, log, lin)


def _mel_to_hz(m):
    m = torch.as_tensor(m, dtype=torch.float64)
    lin = 200.0 * m / 3.0
    log = 1000.0 * torch.exp((math.log(6.4) / 27.0) * (m - 15.0))
    return torch.where(m >= 15.0, log, lin)


def mel_filters(n_mels: int = 80, n_fft: int = N_FFT, sr: int = SAMPLE_RATE) -> torch.Tensor:
    """[n_fft // 2 + 1, n_mels] triangular filters, Slaney area normalisation."""
    fft_freqs = torch.linspace(0, sr / 2, n_fft // 2 + 1, dtype=torch.float64)
    mels = torch.linspace(float(_hz_to_mel(0.0)), float(_hz_to_mel(sr / 2)), n_mels + 2, dtype=torch.float64)
    pts = _mel_to_hz(mels)
    fdiff = pts[1:] - pts[:-1]
    slopes = pts[None, :] - fft_freqs[:, None]  # [F, n_mels + 2]
    down = -slopes[:, :-2] / fdiff[:-1]
    up = slopes[:, 2:] / fdiff[1:]
    fb = torch.clamp(torch.minimum(down, up), min=0.0)
    enorm = 2.0 / (pts[2:n_mels + 2] - pts[:n_mels])
    return (fb * enorm[None, :]).float()


def log_mel(audio: torch.Tensor, n_mels: int = 80, pad_to: int | None = SAMPLE_RATE * CHUNK_SECONDS) -> torch.Tensor:
    """audio [n] (16 kHz, float) -> [n_mels, frames] (3000 frames for 30 s)."""
    x = audio.float().flatten()
    if pad_to is not None:
        x = F.pad(x, (0, max(0, pad_to - x.numel())))[:pad_to]
    win = torch.hann_window(N_FFT, periodic=True, dtype=torch.float32, device=x.device)
    spec = torch.stft(x, N_FFT, HOP, window=win, center=True, pad_mode="reflect", return_complex=True)
    power = spec[:, :-1].abs() ** 2  # drop the last frame, as Whisper does
    mel = mel_filters(n_mels).to(x.device).t() @ power
    lg = torch.clamp(mel, min=1e-10).log10()
    lg = torch.maximum(lg, lg.max() - 8.0)
    return (lg + 4.0) / 4.0


def sinusoids(length: int, channels: int, max_timescale: float = 10000.0) -> torch.Tensor:
    inc = math.log(max_timescale) / (channels // 2 - 1)
    inv = torch.exp(-inc * torch.arange(channels // 2, dtype=torch.float32))
    t = torch.arange(length, dtype=torch.float32)[:, None] * inv[None, :]
    return torch.cat([t.sin(), t.cos()], 1)


# ---------------------------------------------------------------------------
# model
# ---------------------------------------------------------------------------

class WhisperModel:
    """``encoder_only``: load just the audio encoder (audio LLMs that reuse it)."""

    def __init__(self, cfg: WhisperConfig, weights, device="cpu", dtype: torch.dtype | None = None,
                 encoder_only: bool = False):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype or (torch.bfloat16 if self.device.type == "cuda" else torch.float32)
        get = (lambda n: weights.take(n)) if hasattr(weights, "take") else (lambda n: weights[n])
        has = lambda n: n in weights  # noqa: E731
        dv = lambda t: t.to(self.device, self.dtype).contiguous()  # noqa: E731
        e, d = "model.encoder.", "model.decoder."
        self.conv1 = (dv(get(e + "conv1.weight")), dv(get(e + "conv1.bias")))
        self.conv2 = (dv(get(e + "conv2.weight")), dv(get(e + "conv2.bias")))
        self.enc_pos = dv(get(e + "embed_positions.weight")) if has(e + "embed_positions.weight") else \
            dv(sinusoids(cfg.max_source_positions, cfg.d_model))

        def attn(p):  # Whisper's k projections carry no bias
            return dict(q=(dv(get(p + "q_proj.weight")), dv(get(p + "q_proj.bias"))),
                        k=(dv(get(p + "k_proj.weight")), None),
                        v=(dv(get(p + "v_proj.weight")), dv(get(p + "v_proj.bias"))),
                        o=(dv(get(p + "out_proj.weight")), dv(get(p + "out_proj.bias"))))

        def ln(p):
            return dv(get(p + ".weight")), dv(get(p + ".bias"))

        def mlp(p):
            return dict(fc1=(dv(get(p + "fc1.weight")), dv(get(p + "fc1.bias"))),
                        fc2=(dv(get(p + "fc2.weight")), dv(get(p + "fc2.bias"))))

        self.enc = [dict(ln1=ln(e + f"layers.{i}.self_attn_layer_norm"), att=attn(e + f"layers.{i}.self_attn."),
                         ln2=ln(e + f"layers.{i}.final_layer_norm"), **mlp(e + f"layers.{i}."))
                    for i in range(cfg.encoder_layers)]
        self.enc_ln = ln(e + "layer_norm")
        if encoder_only:
            return
        self.tok = dv(get(d + "embed_tokens.weight"))
        self.dec_pos = dv(get(d + "embed_positions.weight"))
        self.dec = [dict(ln1=ln(d + f"layers.{i}.self_attn_layer_norm"), att=attn(d + f"layers.{i}.self_attn."),
                         lnx=ln(d + f"layers.{i}.encoder_attn_layer_norm"),
                         xatt=attn(d + f"layers.{i}.encoder_attn."),
                         ln2=ln(d + f"layers.{i}.final_layer_norm"), **mlp(d + f"layers.{i}."))
                    for i in range(cfg.decoder_layers)]
        self.dec_ln = ln(d + "layer_norm")
        self.head = dv(get("proj_out.weight")) if has("proj_out.weight") else self.tok

    def _ln(self, x, p):
        return F.layer_norm(x.float(), (x.shape[-1],), p[0].float(), p[1].float(), 1e-5).to(x.dtype)

    def _proj(self, x, wb):
        return _linear(x, wb[0], wb[1])

    def _heads(self, x, nh):
        B, L, D = x.shape
        return x.view(B, L, nh, D // nh).transpose(1, 2)

    @torch.no_grad()
    def encode(self, mel: torch.Tensor) -> torch.Tensor:
        """mel [B, n_mels, frames] -> encoder states [B, frames / 2, d]."""
        c = self.cfg
        x = mel.to(self.device, self.dtype)
        x = F.gelu(F.conv1d(x, *self.conv1, padding=1))
        x = F.gelu(F.conv1d(x, *self.conv2, stride=2, padding=1)).transpose(1, 2)
        x = x + self.enc_pos[:x.shape[1]]
        nh = c.encoder_attention_heads
        for ly in self.enc:
            h = self._ln(x, ly["ln1"])
            q, k, v = (self._heads(self._proj(h, ly["att"][n]), nh) for n in "qkv")
            a = F.scaled_dot_product_attention(q, k, v)
            x = x + self._proj(a.transpose(1, 2).reshape(x.shape), ly["att"]["o"])
            h = self._ln(x, ly["ln2"])
            x = x + self._proj(F.gelu(self._proj(h, ly["fc1"])), ly["fc2"])
        return self._ln(x, self.enc_ln)

    def cross_kv(self, enc: torch.Tensor):
        nh = self.cfg.decoder_attention_heads
        return [(self._heads(self._proj(enc, ly["xatt"]["k"]), nh), self._heads(self._proj(enc, ly["xatt"]["v"]), nh))
                for ly in self.dec]

    @torch.no_grad()
    def decode(self, ids: torch.Tensor, xkv, cache: list | None = None, offset: int = 0):
        """ids [B, T] continuing ``cache`` (list of per-layer (k, v) or None) at
        position ``offset`` -> (logits [B, T, V] fp32, new cache)."""
        c = self.cfg
        nh = c.decoder_attention_heads
        ids = ids.to(self.device)
        T = ids.shape[1]
        x = self.tok[ids] * (math.sqrt(c.d_model) if c.scale_embedding else 1.0) + self.dec_pos[offset:offset + T]
        new = []
        for i, ly in enumerate(self.dec):
            h = self._ln(x, ly["ln1"])
            q, k, v = (self._heads(self._proj(h, ly["att"][n]), nh) for n in "qkv")
            if cache is not None and cache[i] is not None:
                k = torch.cat([cache[i][0], k], 2)
                v = torch.cat([cache[i][1], v], 2)
            new.append((k, v))
            if T > 1:  # causal within the new tokens, full over the cached prefix
                mask = torch.ones(T, k.shape[2], dtype=torch.bool, device=x.device).tril(k.shape[2] - T)
                a = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
            else:
                a = F.scaled_dot_product_attention(q, k, v)
            x = x + self._proj(a.transpose(1, 2).reshape(x.shape), ly["att"]["o"])
            h = self._ln(x, ly["lnx"])
            q = self._heads(self._proj(h, ly["xatt"]["q"]), nh)
            a = F.scaled_dot_product_attention(q, xkv[i][0], xkv[i][1])
            x = x + self._proj(a.transpose(1, 2).reshape(x.shape), ly["xatt"]["o"])
            h = self._ln(x, ly["ln2"])
            x = x + self._proj(F.gelu(self._proj(h, ly["fc1"])), ly["fc2"])
        x = self._ln(x, self.dec_ln)
        return _linear(x, self.head).float(), new

    @torch.no_grad()
    def generate(self, mel: torch.Tensor, prefix: list[int], max_new_tokens: int = 100) -> list[list[int]]:
        """Greedy decoding after the forced ``prefix``; stops at end-of-text."""
        enc = self.encode(mel)
        xkv = self.cross_kv(enc)
        B = enc.shape[0]
        ids = torch.tensor([prefix] * B)
        logits, cache = self.decode(ids, xkv)
        out = [[] for _ in range(B)]
        done = [False] * B
        pos = len(prefix)
        for _ in range(max_new_tokens):
            nxt = logits[:, -1].argmax(-1)
            for b in range(B):
                if not done[b]:
                    t = int(nxt[b])
                    if t == self.cfg.eos_token_id:
                        done[b] = True
                    else:
                        out[b].append(t)
            if all(done) or pos >= self.cfg.max_target_positions:
                break
            logits, cache = self.decode(nxt.view(B, 1), xkv, cache, pos)
            pos += 1
        return out


class SpeechToText:
    """``transcribe(audio)``: 30 s windows through Whisper, decoded greedily."""

    def __init__(self, model: WhisperModel, tokenizer=None, language: str | None = "en", task: str = "transcribe"):
        self.model, self.tok = model, tokenizer
        self.language, self.task = language, task

    def prefix(self) -> list[int]:
        c = self.model.cfg
        if self.tok is None:
            return [c.decoder_start_token_id]
        ids = [c.decoder_start_token_id]
        for t in ([f"<|{self.language}|>"] if self.language else []) + [f"<|{self.task}|>", "<|notimestamps|>"]:
            tid = self.tok.convert_tokens_to_ids(t)
            if tid is not None and tid != getattr(self.tok, "unk_token_id", None):
                ids.append(tid)
        return ids

    def transcribe(self, audio: torch.Tensor, sample_rate: int = SAMPLE_RATE, max_new_tokens: int = 200):
        if sample_rate != SAMPLE_RATE:
            n = int(round(audio.numel() * SAMPLE_RATE / sample_rate))
            audio = F.interpolate(audio.float().view(1, 1, -1), size=n, mode="linear", align_corners=False).flatten()
        # the encoder's window: 2 * max_source_positions frames of HOP samples (30 s for Whisper)
        win = 2 * self.model.cfg.max_source_positions * HOP
        pieces = []
        for s in range(0, max(1, audio.numel()), win):
            mel = log_mel(audio[s:s + win], self.model.cfg.num_mel_bins, pad_to=win).unsqueeze(0)
            toks = self.model.generate(mel, self.prefix(), max_new_tokens)[0]
            pieces.append(self.tok.decode(toks, skip_special_tokens=True) if self.tok is not None else toks)
        return "".join(pieces) if self.tok is not None else [t for p in pieces for t in p]
