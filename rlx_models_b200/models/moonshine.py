"""Moonshine speech recognition (encoder-decoder over raw 16 kHz audio).

    encoder  conv1d(1 -> H, k 127, stride 64, no bias) -> tanh -> GroupNorm(1 group)
             -> conv1d(H -> 2H, k 7, stride 3) -> GELU -> conv1d(2H -> H, k 3, stride 2) -> GELU
             -> pre-LayerNorm blocks (bias-free LayerNorms): non-causal self-attention with
                partial RoPE on interleaved pairs, GELU MLP -> final LayerNorm
    decoder  token embedding -> blocks: causal self-attention (partial RoPE), cross-attention
             to the encoder output (no RoPE), SwiGLU-style MLP (fc1 -> [x | gate] ->
             silu(gate) * x -> fc2) -> LayerNorm -> output projection (tied to the embedding)
    decode   greedy from ``decoder_start_token_id`` with a self-attention KV cache and the
             cross-attention K / V computed once per utterance

Linear layers run on the package's GEMM (bf16 on CUDA), the rest in torch;
transformers' MoonshineForConditionalGeneration is the CPU oracle.

Reference: crates/rlx-moonshine (encoder-decoder over raw PCM).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .flux_text import _linear


@dataclass
class MoonshineConfig:
    vocab_size: int = 32768
    hidden_size: int = 288
    intermediate_size: int = 1152
    encoder_num_hidden_layers: int = 6
    decoder_num_hidden_layers: int = 6
    encoder_num_attention_heads: int = 8
    decoder_num_attention_heads: int = 8
    encoder_hidden_act: str = "gelu"
    decoder_hidden_act: str = "silu"
    partial_rotary_factor: float = 0.9
    rope_theta: float = 10000.0
    attention_bias: bool = False
    decoder_start_token_id: int = 1
    eos_token_id: int = 2
    tie_word_embeddings: bool = True

    @classmethod
    def from_dict(cls, d: dict) -> "MoonshineConfig":
        kw = {k: d[k] for k in cls.__dataclass_fields__ if k in d and d[k] is not None}
        rp = d.get("rope_parameters") or {}
        if isinstance(rp, dict):
            kw.setdefault("rope_theta", float(rp.get("rope_theta", d.get("rope_theta", 10000.0))))
            if "partial_rotary_factor" in rp:
                kw["partial_rotary_factor"] = float(rp["partial_rotary_factor"])
        if isinstance(kw.get("eos_token_id"), list):
            kw["eos_token_id"] = kw["eos_token_id"][0]
        return cls(**kw)


def _act(name: str, x: torch.Tensor) -> torch.Tensor:
    return F.silu(x) if name in ("silu", "swish") else F.gelu(x)


class MoonshineModel:
    def __init__(self, cfg: MoonshineConfig, weights, device="cpu", dtype: torch.dtype | None = None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype or (torch.bfloat16 if self.device.type == "cuda" else torch.float32)
        get = (lambda n: weights.take(n)) if hasattr(weights, "take") else (lambda n: weights[n])
        has = lambda n: n in weights  # noqa: E731
        dv = lambda t: t.to(self.device, self.dtype).contiguous()  # noqa: E731
        f32 = lambda t: t.to(self.device, torch.float32).contiguous()  # noqa: E731
        opt = lambda n: dv(get(n)) if has(n) else None  # noqa: E731
        e, d = "model.encoder.", "model.decoder."
        self.conv1 = f32(get(e + "conv1.weight"))
        self.conv2 = (f32(get(e + "conv2.weight")), f32(get(e + "conv2.bias")))
        self.conv3 = (f32(get(e + "conv3.weight")), f32(get(e + "conv3.bias")))
        self.gn = (f32(get(e + "groupnorm.weight")), f32(get(e + "groupnorm.bias")))

        def attn(p):
            names = ("q_proj", "k_proj", "v_proj", "o_proj")
            return {n: (dv(get(p + n + ".weight")), opt(p + n + ".bias")) for n in names}

        def lin(p):
            return (dv(get(p + ".weight")), opt(p + ".bias"))
        self.enc = [dict(ln1=f32(get(e + f"layers.{i}.input_layernorm.weight")),
                         ln2=f32(get(e + f"layers.{i}.post_attention_layernorm.weight")),
                         att=attn(e + f"layers.{i}.self_attn."), fc1=lin(e + f"layers.{i}.mlp.fc1"),
                         fc2=lin(e + f"layers.{i}.mlp.fc2")) for i in range(cfg.encoder_num_hidden_layers)]
        self.enc_norm = f32(get(e + "layer_norm.weight"))
        self.embed = dv(get(d + "embed_tokens.weight"))
        self.dec = [dict(ln1=f32(get(d + f"layers.{i}.input_layernorm.weight")),
                         ln2=f32(get(d + f"layers.{i}.post_attention_layernorm.weight")),
                         ln3=f32(get(d + f"layers.{i}.final_layernorm.weight")),
                         att=attn(d + f"layers.{i}.self_attn."), xatt=attn(d + f"layers.{i}.encoder_attn."),
                         fc1=lin(d + f"layers.{i}.mlp.fc1"), fc2=lin(d + f"layers.{i}.mlp.fc2"))
                    for i in range(cfg.decoder_num_hidden_layers)]
        self.dec_norm = f32(get(d + "norm.weight"))
        self.head = self.embed if cfg.tie_word_embeddings or not has("proj_out.weight") else dv(get("proj_out.weight"))

    # -- pieces ---------------------------------------------------------------
    def _ln(self, x, w):
        return F.layer_norm(x.float(), (x.shape[-1],), w, None, 1e-5)

    def _rope(self, x: torch.Tensor, pos: torch.Tensor, heads: int) -> torch.Tensor:
        """x [B, L, heads * D]: rotate interleaved pairs of the first rotary dims of every head."""
        B, L, _ = x.shape
        D = x.shape[-1] // heads
        rd = int(D * self.cfg.partial_rotary_factor)
        rd -= rd % 2
        inv = 1.0 / (self.cfg.rope_theta ** (torch.arange(0, rd, 2, device=x.device).float() / rd))
        ang = pos.float()[:, None] * inv[None, :]  # [L, rd / 2]
        cos, sin = ang.cos()[None, :, None, :], ang.sin()[None, :, None, :]
        t = x.float().view(B, L, heads, D)
        r, rest = t[..., :rd], t[..., rd:]
        a, b = r[..., 0::2], r[..., 1::2]
        r = torch.stack([a * cos - b * sin, a * sin + b * cos], -1).flatten(-2)
        return torch.cat([r, rest], -1).reshape(B, L, heads * D)

    def _proj(self, x, p):
        return _linear(x.to(self.dtype), *p).float()

    def _attend(self, q, k, v, heads, causal):
        B, Lq, H = q.shape
        D = H // heads
        q, k, v = (t.reshape(B, -1, heads, D).transpose(1, 2) for t in (q, k, v))
        o = F.scaled_dot_product_attention(q, k, v, is_causal=causal and Lq > 1)
        return o.transpose(1, 2).reshape(B, Lq, H)

    # -- encoder --------------------------------------------------------------
    @torch.no_grad()
    def encode(self, audio: torch.Tensor) -> torch.Tensor:
        """audio [B, N] float 16 kHz -> encoder states [B, T, H] fp32."""
        c = self.cfg
        x = audio.to(self.device, torch.float32)[:, None]
        x = torch.tanh(F.conv1d(x, self.conv1, stride=64))
        x = F.group_norm(x, 1, *self.gn, eps=1e-5)
        x = F.gelu(F.conv1d(x, *self.conv2, stride=3))
        x = F.gelu(F.conv1d(x, *self.conv3, stride=2)).transpose(1, 2)  # [B, T, H]
        nh = c.encoder_num_attention_heads
        pos = torch.arange(x.shape[1], device=self.device)
        for ly in self.enc:
            y = self._ln(x, ly["ln1"])
            a = ly["att"]
            q, k, v = (self._proj(y, a[n]) for n in ("q_proj", "k_proj", "v_proj"))
            q, k = self._rope(q, pos, nh), self._rope(k, pos, nh)
            x = x + self._proj(self._attend(q, k, v, nh, False), a["o_proj"])
            y = self._ln(x, ly["ln2"])
            x = x + self._proj(_act(c.encoder_hidden_act, self._proj(y, ly["fc1"])), ly["fc2"])
        return self._ln(x, self.enc_norm)

    # -- decoder --------------------------------------------------------------
    def _cross_kv(self, enc: torch.Tensor):
        return [(self._proj(enc, ly["xatt"]["k_proj"]), self._proj(enc, ly["xatt"]["v_proj"])) for ly in self.dec]

    @torch.no_grad()
    def decode_step(self, ids: torch.Tensor, start: int, cache: list, cross: list) -> torch.Tensor:
        """ids [B, L] new tokens at positions start..; ``cache`` holds each layer's
        self-attention (k, v) [B, start, H] (updated in place); returns fp32 logits [B, L, V]."""
        c = self.cfg
        nh = c.decoder_num_attention_heads
        x = self.embed[ids.to(self.device)].float()
        L = ids.shape[1]
        pos = torch.arange(start, start + L, device=self.device)
        for i, ly in enumerate(self.dec):
            y = self._ln(x, ly["ln1"])
            a = ly["att"]
            q, k, v = (self._proj(y, a[n]) for n in ("q_proj", "k_proj", "v_proj"))
            q, k = self._rope(q, pos, nh), self._rope(k, pos, nh)
            if cache[i] is not None:
                k, v = torch.cat([cache[i][0], k], 1), torch.cat([cache[i][1], v], 1)
            cache[i] = (k, v)
            if L > 1 and start > 0:  # a multi-token continuation: explicit causal mask over the cache
                B = x.shape[0]
                D = k.shape[-1] // nh
                qh, kh, vh = (t.reshape(B, -1, nh, D).transpose(1, 2) for t in (q, k, v))
                m = torch.arange(k.shape[1], device=self.device)[None, :] <= pos[:, None]
                o = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=m).transpose(1, 2).reshape(B, L, -1)
            else:
                o = self._attend(q, k, v, nh, start == 0)
            x = x + self._proj(o, a["o_proj"])
            y = self._ln(x, ly["ln2"])
            xa = ly["xatt"]
            o = self._attend(self._proj(y, xa["q_proj"]), cross[i][0], cross[i][1], nh, False)
            x = x + self._proj(o, xa["o_proj"])
            y = self._ln(x, ly["ln3"])
            h, gate = self._proj(y, ly["fc1"]).chunk(2, -1)
            x = x + self._proj(_act(c.decoder_hidden_act, gate) * h, ly["fc2"])
        x = self._ln(x, self.dec_norm)
        return _linear(x.to(self.dtype), self.head).float()

    @torch.no_grad()
    def greedy(self, audio: torch.Tensor, max_new_tokens: int | None = None) -> list[list[int]]:
        """Greedy transcription token ids per utterance (without the start token,
        up to and excluding the end token). Default length limit: 6.5 tokens per
        second of audio, the release's rule of thumb."""
        c = self.cfg
        audio = torch.as_tensor(audio, dtype=torch.float32)
        if audio.dim() == 1:
            audio = audio[None]
        B = audio.shape[0]
        if max_new_tokens is None:
            max_new_tokens = max(4, math.ceil(audio.shape[1] / 16000 * 6.5))
        enc = self.encode(audio)
        cross = self._cross_kv(enc)
        cache = [None] * len(self.dec)
        ids = torch.full((B, 1), c.decoder_start_token_id, dtype=torch.long, device=self.device)
        out = [[] for _ in range(B)]
        done = [False] * B
        pos = 0
        for _ in range(max_new_tokens):
            lg = self.decode_step(ids, pos, cache, cross)[:, -1]
            pos += ids.shape[1]
            nxt = lg.argmax(-1)
            for b in range(B):
                t = int(nxt[b])
                if not done[b]:
                    if t == c.eos_token_id:
                        done[b] = True
                    else:
                        out[b].append(t)
            if all(done):
                break
            ids = nxt[:, None]
        return out


class MoonshineTranscriber:
    """``transcribe(audio, sample_rate)`` over a MoonshineModel."""

    def __init__(self, model: MoonshineModel, tokenizer=None):
        self.model, self.tokenizer = model, tokenizer

    def transcribe(self, audio, sample_rate: int = 16000):
        a = torch.as_tensor(audio, dtype=torch.float32)
        if a.dim() > 1:
            a = a.mean(-1)
        if sample_rate != 16000:
            a = F.interpolate(a[None, None], scale_factor=16000 / sample_rate, mode="linear",
                              align_corners=False)[0, 0]
        ids = self.model.greedy(a)[0]
        return self.tokenizer.decode(ids) if self.tokenizer is not None else ids
