"""VibeVoice-ASR: speech recognition from two causal ConvNeXt tokenizer
encoders (acoustic and semantic) and a Qwen2 LM (transformers
``vibevoice_asr``).

    encoder  24 kHz audio -> stem (causal conv + ConvNeXt blocks) -> per stage a
             strided causal conv (kernel 2 r, stride r) + ConvNeXt blocks -> head
             causal conv -> latents [T / prod(r), hidden]
    block    x += gamma * dwconv(rmsnorm(x));  x += ffn_gamma * W2 act(W1 rmsnorm(x))
             (depthwise causal conv, left padding (k - 1) d - (s - 1))
    project  features = L2a(rmsnorm(L1a(acoustic))) + L2s(rmsnorm(L1s(semantic)))
    prompt   the LM's embeddings at the audio-token positions are replaced by the
             features, in order (one multimodal segment per contiguous run)

The released acoustic path adds Gaussian noise of std ``vae_std`` to its
latents (a VAE sample); ``sample_noise=False`` (the default here) uses the
mean, which is what recognition wants and what makes the output
deterministic. Causal convolutions over the whole signal equal the chunked
streaming pass with padding caches (chunks a multiple of the hop length).

Linear layers (the blocks' FFNs, the projector) run on the package's tcgen05
GEMM in bf16 on the GPU; the convolutions are torch conv1d; the LM is the
package's decoder on the GPU and the fp32 oracle on CPU.

Reference: crates/rlx-vibevoice-asr (VibeVoice-ASR: acoustic and semantic
ConvNeXt VAEs -> speech connectors -> summed features -> Qwen2.5 LM);
transformers' VibeVoiceAsrForConditionalGeneration is the CPU oracle.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from ..config import DecoderConfig
from .flux_text import _linear


@dataclass
class VibeVoiceEncoderConfig:
    channels: int = 1
    kernel_size: int = 7
    num_filters: int = 32
    downsampling_ratios: list = field(default_factory=lambda: [2, 2, 4, 5, 5, 8])
    depths: list = field(default_factory=lambda: [3, 3, 3, 3, 3, 3, 8])
    hidden_size: int = 64
    ffn_expansion: int = 4
    hidden_act: str = "gelu"
    rms_norm_eps: float = 1e-5
    vae_std: float = 0.625

    @property
    def hop_length(self) -> int:
        return int(math.prod(self.downsampling_ratios))

    @classmethod
    def from_dict(cls, d: dict) -> "VibeVoiceEncoderConfig":
        return cls(**{k: d[k] for k in cls.__dataclass_fields__ if k in d and d[k] is not None})


def _act(name, x):
    if name == "gelu":
        return F.gelu(x)
    if name in ("gelu_pytorch_tanh", "gelu_new"):
        return F.gelu(x, approximate="tanh")
    if name == "silu":
        return F.silu(x)
    raise NotImplementedError(f"activation {name!r}")


class VibeVoiceEncoder:
    """One tokenizer encoder (acoustic or semantic) over audio [B, C, S]."""

    def __init__(self, cfg: VibeVoiceEncoderConfig, weights, prefix: str, device="cpu"):
        self.cfg, self.device = cfg, torch.device(device)
        self.dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])
        self._get = lambda n: get(prefix + n)  # noqa: E731
        c = cfg
        self.stem = self._conv("stem.conv.conv", 1)
        self.stages = [[self._block(f"stem.stage.{j}.") for j in range(c.depths[0])]]
        self.downs = []
        for s, r in enumerate(c.downsampling_ratios):
            self.downs.append(self._conv(f"conv_layers.{s}.conv.conv", r))
            self.stages.append([self._block(f"conv_layers.{s}.stage.{j}.") for j in range(c.depths[s + 1])])
        self.head = self._conv("head.conv", 1)

    def _t(self, n, dt=torch.float32):
        return self._get(n).to(self.device, dt).contiguous()

    def _conv(self, n, stride, groups=1):
        w = self._t(n + ".weight", self.dtype)
        return dict(w=w, b=self._t(n + ".bias", self.dtype), stride=stride, groups=groups,
                    pad=(w.shape[-1] - 1) - (stride - 1))

    def _block(self, p):
        return dict(n1=self._t(p + "norm.weight"), n2=self._t(p + "ffn_norm.weight"), g1=self._t(p + "gamma"),
                    g2=self._t(p + "ffn_gamma"), mix=self._conv(p + "mixer.conv", 1, groups=-1),
                    w1=self._t(p + "ffn.linear1.weight", self.dtype), b1=self._t(p + "ffn.linear1.bias", self.dtype),
                    w2=self._t(p + "ffn.linear2.weight", self.dtype), b2=self._t(p + "ffn.linear2.bias", self.dtype))

    @staticmethod
    def _apply_conv(cv, x):  # x [B, C, S] in the compute dtype
        groups = x.shape[1] if cv["groups"] == -1 else cv["groups"]
        return F.conv1d(F.pad(x, (cv["pad"], 0)), cv["w"], cv["b"], stride=cv["stride"], groups=groups)

    def _rms(self, x, w):  # over channels of [B, C, S]
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(1, keepdim=True) + self.cfg.rms_norm_eps) * w[None, :, None])

    def _run_block(self, L, x):
        x = x + L["g1"][None, :, None] * self._apply_conv(L["mix"], self._rms(x, L["n1"]).to(self.dtype)).float()
        B, C, S = x.shape
        h = self._rms(x, L["n2"]).transpose(1, 2).reshape(B * S, C).to(self.dtype).contiguous()
        h = _act(self.cfg.hidden_act, _linear(h, L["w1"], L["b1"]).float()).to(self.dtype)
        y = _linear(h, L["w2"], L["b2"]).float().view(B, S, C).transpose(1, 2)
        return x + L["g2"][None, :, None] * y

    @torch.no_grad()
    def latents(self, audio: torch.Tensor) -> torch.Tensor:
        """audio [B, C, S] (or [B, S]) -> latents [B, ceil-ish(S / hop), hidden] fp32."""
        x = audio.to(self.device, torch.float32)
        if x.dim() == 2:
            x = x[:, None]
        x = self._apply_conv(self.stem, x.to(self.dtype)).float()
        for L in self.stages[0]:
            x = self._run_block(L, x)
        for down, stage in zip(self.downs, self.stages[1:]):
            x = self._apply_conv(down, x.to(self.dtype)).float()
            for L in stage:
                x = self._run_block(L, x)
        return self._apply_conv(self.head, x.to(self.dtype)).float().transpose(1, 2)


@dataclass
class VibeVoiceAsrConfig:
    acoustic: VibeVoiceEncoderConfig
    semantic: VibeVoiceEncoderConfig
    text: DecoderConfig
    audio_token_id: int = 151648

    @classmethod
    def from_dict(cls, d: dict) -> "VibeVoiceAsrConfig":
        tc = dict(d.get("text_config") or {})
        tc.setdefault("model_type", "qwen2")
        return cls(acoustic=VibeVoiceEncoderConfig.from_dict(d.get("acoustic_tokenizer_encoder_config") or {}),
                   semantic=VibeVoiceEncoderConfig.from_dict(d.get("semantic_tokenizer_encoder_config") or {}),
                   text=DecoderConfig.from_hf_dict(tc), audio_token_id=int(d.get("audio_token_id", 151648)))


class _Prefixed:
    """The LM's tensors (``language_model.*`` / ``model.language_model.*``) under decoder names."""

    def __init__(self, weights):
        self.w = weights
        self.map = {}
        for k in weights.keys():
            for pre, new in (("model.language_model.", "model."), ("language_model.model.", "model."),
                             ("language_model.lm_head.", "lm_head."), ("lm_head.", "lm_head.")):
                if k.startswith(pre):
                    self.map[new + k[len(pre):]] = k
                    break

    def keys(self):
        return list(self.map)

    def __contains__(self, n):
        return n in self.map

    def __getitem__(self, n):
        return self.w.take(self.map[n]) if hasattr(self.w, "take") else self.w[self.map[n]]

    def take(self, n, dtype=None, device=None):
        t = self[n]
        return t if dtype is None and device is None else t.to(device=device, dtype=dtype)

    def dict(self):
        return {k: self[k] for k in self.map}


class VibeVoiceAsr:
    takes_waveform = True  # the served audio is the 24 kHz waveform, not log-mel windows

    def __init__(self, cfg: VibeVoiceAsrConfig, weights, device="cpu", lm=None):
        self.cfg, self.device = cfg, torch.device(device)
        pre = "model." if any(k.startswith("model.acoustic_tokenizer_encoder.") for k in weights.keys()) else ""
        self.acoustic = VibeVoiceEncoder(cfg.acoustic, weights, pre + "acoustic_tokenizer_encoder.", device)
        self.semantic = VibeVoiceEncoder(cfg.semantic, weights, pre + "semantic_tokenizer_encoder.", device)
        dt = self.acoustic.dtype
        g = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])
        p = pre + "multi_modal_projector."
        dv = lambda n: g(p + n).to(self.device, dt).contiguous()  # noqa: E731
        self.proj = {s: dict(l1=(dv(f"{s}_linear_1.weight"), dv(f"{s}_linear_1.bias")),
                             n=g(p + f"{s}_norm.weight").to(self.device, torch.float32),
                             l2=(dv(f"{s}_linear_2.weight"), dv(f"{s}_linear_2.bias")))
                     for s in ("acoustic", "semantic")}
        text = _Prefixed(weights)
        if lm is not None:
            self.lm = lm
        elif self.device.type == "cuda":
            from ..registry import build_model
            self.lm = build_model(cfg.text, text, device=self.device)
        else:
            from .oracle import DecoderOracle
            self.lm = DecoderOracle(cfg.text, {k: v.float() for k, v in text.dict().items()}, device=self.device)

    def _connector(self, s: str, lat: torch.Tensor) -> torch.Tensor:
        P = self.proj[s]
        h = _linear(lat.to(self.acoustic.dtype).contiguous(), *P["l1"]).float()
        h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-6) * P["n"]
        return _linear(h.to(self.acoustic.dtype), *P["l2"]).float()

    @torch.no_grad()
    def audio_features(self, audio: torch.Tensor, sample_noise: bool = False,
                       generator: torch.Generator | None = None) -> torch.Tensor:
        """audio [S] or [B, S] at 24 kHz -> features [B, T, H_text] fp32."""
        a = audio if audio.dim() >= 2 else audio[None]
        ac = self.acoustic.latents(a)
        if sample_noise:
            std = self.cfg.acoustic.vae_std * torch.randn(ac.shape[0], generator=generator).to(ac.device)
            ac = ac + std[:, None, None] * torch.randn(ac.shape, generator=generator).to(ac.device)
        sm = self.semantic.latents(a)
        B, T, _ = ac.shape
        f = self._connector("acoustic", ac.reshape(B * T, -1)) + self._connector("semantic", sm.reshape(B * T, -1))
        return f.view(B, T, -1)

    @torch.no_grad()
    def mm_segments(self, ids: list[int], audio: torch.Tensor) -> list[tuple[int, torch.Tensor]]:
        """(first position, rows) of every contiguous run of audio tokens in ``ids``, filled in
        order with the clip's features (``audio``: one clip [S] or a batch [B, S] of equal length)."""
        feats = self.audio_features(audio).reshape(-1, self.cfg.text.hidden_size)
        rows = [i for i, t in enumerate(ids) if t == self.cfg.audio_token_id]
        if len(rows) != feats.shape[0]:
            raise ValueError(f"prompt has {len(rows)} audio tokens; the audio gives {feats.shape[0]}")
        segs, start = [], 0
        for j in range(1, len(rows) + 1):
            if j == len(rows) or rows[j] != rows[j - 1] + 1:
                segs.append((rows[start], feats[start:j]))
                start = j
        return segs

    @torch.no_grad()
    def oracle_logits(self, ids: list[int], audio: torch.Tensor) -> torch.Tensor:
        segs = self.mm_segments(ids, audio)
        rows = torch.cat([torch.arange(p, p + e.shape[0]) for p, e in segs])
        emb = torch.cat([e for _, e in segs]).float()
        lg, _ = self.lm.forward(torch.tensor(ids), mm=(rows, emb))
        return lg
