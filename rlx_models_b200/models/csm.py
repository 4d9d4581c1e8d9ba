"""CSM (Sesame's conversational speech model): text-to-speech as two Llama
decoders over Mimi codec frames.

    prompt    text tokens (embed_text_tokens) and, optionally, audio frames of
              context speech: a frame embeds as the sum over codebooks k of
              embed_audio_tokens[code_k + k * codebook_size]
    backbone  Llama (RMSNorm, RoPE, GQA, SwiGLU) over the prompt and the frames
              generated so far; lm_head on its last hidden state h -> codebook 0
    depth     a small Llama over [h, code_0, code_1, ...] (h projected from the
              backbone width; code_j embedded with offset j * vocab) predicts codebook
              j + 1 from position j + 1 with a codebook-specific head
    stop      a frame whose codebooks (all but the last) are the codebook EOS id ends
              generation; the frames decode to 24 kHz audio with Mimi

Both decoders keep K / V caches; linears run on the package's tcgen05 GEMM in
bf16 on the GPU, attention is torch SDPA; greedy decoding (argmax) is what the
tests pin against transformers.

Checkpoint names: transformers' CsmForConditionalGeneration (``backbone_model.*``,
``depth_decoder.model.*``, ``depth_decoder.codebooks_head.weight``,
``embed_text_tokens.weight``, ``lm_head.weight``, ``codec_model.*``).

Reference: crates/rlx-sesame (Sesame CSM speech generation); transformers'
CsmForConditionalGeneration is the CPU oracle.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from .flux_text import _linear


@dataclass
class LlamaStackCfg:
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    intermediate_size: int
    rms_norm_eps: float = 1e-5
    rope_theta: float = 500000.0
    rope_scaling: dict | None = None

    @classmethod
    def from_dict(cls, d: dict) -> "LlamaStackCfg":
        rp = dict(d.get("rope_parameters") or {})
        theta = float(rp.pop("rope_theta", d.get("rope_theta", 500000.0)))
        kind = rp.get("rope_type", "default")
        return cls(hidden_size=d["hidden_size"], num_hidden_layers=d["num_hidden_layers"],
                   num_attention_heads=d["num_attention_heads"],
                   num_key_value_heads=d.get("num_key_value_heads") or d["num_attention_heads"],
                   head_dim=d.get("head_dim") or d["hidden_size"] // d["num_attention_heads"],
                   intermediate_size=d["intermediate_size"], rms_norm_eps=d.get("rms_norm_eps", 1e-5),
                   rope_theta=theta, rope_scaling=None if kind == "default" else rp)


class _LlamaStack:
    """A Llama decoder stack (no embedding, no head) with a growing K / V cache."""

    def __init__(self, cfg: LlamaStackCfg, get, prefix: str, device, dt):
        from .. import ops
        self.cfg, self.dt, self.device = cfg, dt, device
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            p = f"{prefix}layers.{i}."
            cat = lambda names: torch.cat([get(p + n) for n in names]).to(device, dt).contiguous()  # noqa: E731
            self.layers.append(dict(
                qkv=cat(["self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight"]),
                o=get(p + "self_attn.o_proj.weight").to(device, dt).contiguous(),
                gu=cat(["mlp.gate_proj.weight", "mlp.up_proj.weight"]),
                down=get(p + "mlp.down_proj.weight").to(device, dt).contiguous(),
                ln1=get(p + "input_layernorm.weight").to(device, torch.float32),
                ln2=get(p + "post_attention_layernorm.weight").to(device, torch.float32)))
        self.norm = get(prefix + "norm.weight").to(device, torch.float32)
        inv, mult = ops.rope_inv_freq(cfg.head_dim, cfg.rope_theta, cfg.rope_scaling)
        self.inv, self.mult = inv.to(device), float(mult)

    def _rms(self, x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.cfg.rms_norm_eps) * w

    def _rope(self, x, pos):
        ang = pos[:, None].float() * self.inv[None]
        cos = torch.cat([ang.cos()] * 2, -1) * self.mult
        sin = torch.cat([ang.sin()] * 2, -1) * self.mult
        h = x.shape[-1] // 2
        return x * cos + torch.cat([-x[..., h:], x[..., :h]], -1) * sin

    def _lin(self, x, w):
        shp = x.shape
        return _linear(x.reshape(-1, shp[-1]).to(self.dt).contiguous(), w).float().view(*shp[:-1], -1)

    def forward(self, x: torch.Tensor, start: int, cache: list) -> torch.Tensor:
        """x [B, T, H] fp32 at positions start .. start + T - 1 -> normed hidden [B, T, H]."""
        c = self.cfg
        B, T, _ = x.shape
        nh, nkv, hd = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        pos = torch.arange(start, start + T, device=self.device)
        for i, L in enumerate(self.layers):
            h = self._rms(x, L["ln1"])
            q, k, v = self._lin(h, L["qkv"]).split([nh * hd, nkv * hd, nkv * hd], -1)
            q = self._rope(q.view(B, T, nh, hd).transpose(1, 2), pos)
            k = self._rope(k.view(B, T, nkv, hd).transpose(1, 2), pos)
            v = v.view(B, T, nkv, hd).transpose(1, 2)
            if len(cache) > i:
                k = torch.cat([cache[i][0], k], 2)
                v = torch.cat([cache[i][1], v], 2)
                cache[i] = (k, v)
            else:
                cache.append((k, v))
            kk, vv = k.repeat_interleave(nh // nkv, 1), v.repeat_interleave(nh // nkv, 1)
            o = F.scaled_dot_product_attention(q.to(self.dt), kk.to(self.dt), vv.to(self.dt),
                                               is_causal=T > 1 and start == 0)
            if T > 1 and start > 0:
                raise NotImplementedError("multi-token steps after a cached prefix")
            x = x + self._lin(o.transpose(1, 2).reshape(B, T, nh * hd).float(), L["o"])
            g, u = self._lin(self._rms(x, L["ln2"]), L["gu"]).chunk(2, -1)
            x = x + self._lin(F.silu(g) * u, L["down"])
        return self._rms(x, self.norm)


@dataclass
class CsmConfig:
    backbone: LlamaStackCfg
    depth: LlamaStackCfg
    num_codebooks: int = 32
    vocab_size: int = 2051
    codebook_size: int = 2051
    codebook_eos_token_id: int = 0
    codebook_pad_token_id: int = 2050
    audio_token_id: int = 128002
    audio_eos_token_id: int = 128003
    codec: dict = field(default_factory=dict)

    @classmethod
    def from_dict(cls, d: dict) -> "CsmConfig":
        dd = dict(d.get("depth_decoder_config") or {})
        return cls(backbone=LlamaStackCfg.from_dict(d), depth=LlamaStackCfg.from_dict(dd),
                   num_codebooks=int(d.get("num_codebooks", 32)), vocab_size=int(d.get("vocab_size", 2051)),
                   codebook_size=int(d.get("codebook_size", d.get("vocab_size", 2051))),
                   codebook_eos_token_id=int(d.get("codebook_eos_token_id", 0)),
                   codebook_pad_token_id=int(d.get("codebook_pad_token_id", 2050)),
                   audio_token_id=int(d.get("audio_token_id", 128002)),
                   audio_eos_token_id=int(d.get("audio_eos_token_id", 128003)),
                   codec=dict(d.get("codec_config") or {}))


class _Prefixed:
    def __init__(self, weights, prefix):
        self.w, self.p = weights, prefix
        self.get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])

    def keys(self):
        return [k[len(self.p):] for k in self.w.keys() if k.startswith(self.p)]

    def __contains__(self, k):
        return (self.p + k) in self.w

    def __getitem__(self, k):
        return self.get(self.p + k)


class CsmModel:
    def __init__(self, cfg: CsmConfig, weights, device="cpu", codec: bool = True):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dt = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])
        dev, dt = self.device, self.dt
        self.backbone = _LlamaStack(cfg.backbone, get, "backbone_model.", dev, dt)
        self.depth = _LlamaStack(cfg.depth, get, "depth_decoder.model.", dev, dt)
        self.embed_text = get("embed_text_tokens.weight").to(dev, torch.float32)
        self.embed_audio = get("backbone_model.embed_tokens.embed_audio_tokens.weight").to(dev, torch.float32)
        self.depth_embed = get("depth_decoder.model.embed_tokens.weight").to(dev, torch.float32)
        self.depth_proj = get("depth_decoder.model.inputs_embeds_projector.weight").to(dev, dt).contiguous()
        self.head0 = get("lm_head.weight").to(dev, dt).contiguous()
        # per-codebook heads [K - 1, H_depth, V] -> as linear weights [K - 1][V, H_depth]
        self.heads = get("depth_decoder.codebooks_head.weight").to(dev, torch.float32).transpose(1, 2).to(dt).contiguous()
        self.offsets = torch.arange(cfg.num_codebooks, device=dev) * cfg.codebook_size
        self.codec = None
        if codec and any(k.startswith("codec_model.") for k in weights.keys()):
            from .mimi import MimiConfig, MimiModel
            self.codec = MimiModel(MimiConfig.from_dict(cfg.codec), _Prefixed(weights, "codec_model."), device=device)

    def embed_frames(self, codes: torch.Tensor) -> torch.Tensor:
        """codes [..., K] -> frame embeddings [..., H] (sum over codebooks)."""
        return self.embed_audio[codes.to(self.device).long() + self.offsets].sum(-2)

    def _lin(self, x, w):
        return _linear(x.reshape(-1, x.shape[-1]).to(self.dt).contiguous(), w).float()

    @torch.no_grad()
    def depth_codes(self, h: torch.Tensor, c0: torch.Tensor) -> torch.Tensor:
        """Backbone last hidden states h [B, H] and codebook-0 codes [B] -> all
        codebooks [B, K] (greedy depth decoding)."""
        c = self.cfg
        B = h.shape[0]
        cache: list = []
        x = torch.stack([h, self.depth_embed[c0.long()]], 1)             # positions 0 (h) and 1 (code 0)
        y = self.depth.forward(self._lin(x, self.depth_proj).view(B, 2, -1), 0, cache)
        codes = [c0.long()]
        for j in range(1, c.num_codebooks):
            lg = self._lin(y[:, -1], self.heads[j - 1]).view(B, -1)
            nxt = lg.argmax(-1)
            codes.append(nxt)
            if j == c.num_codebooks - 1:
                break
            e = self.depth_embed[nxt + j * c.vocab_size]
            y = self.depth.forward(self._lin(e[:, None], self.depth_proj).view(B, 1, -1), j + 1, cache)
        return torch.stack(codes, 1)

    @torch.no_grad()
    def generate_frames(self, prompt_embeds: torch.Tensor, max_frames: int = 125) -> torch.Tensor:
        """prompt_embeds [B, T, H] -> frames [B, n, K] (greedy; the EOS frame ends a
        sequence and is dropped, finished sequences are padded with codebook_pad)."""
        c = self.cfg
        B = prompt_embeds.shape[0]
        cache: list = []
        h = self.backbone.forward(prompt_embeds.to(self.device).float(), 0, cache)[:, -1]
        pos = prompt_embeds.shape[1]
        frames, done = [], torch.zeros(B, dtype=torch.bool, device=self.device)
        for _ in range(max_frames):
            c0 = self._lin(h, self.head0).argmax(-1)
            codes = self.depth_codes(h, c0)
            codes = torch.where(done[:, None], torch.full_like(codes, c.codebook_pad_token_id), codes)
            eos = (codes[:, :-1] == c.codebook_eos_token_id).all(-1)
            done = done | eos
            frames.append(codes)
            if bool(done.all()):
                break
            h = self.backbone.forward(self.embed_frames(codes)[:, None], pos, cache)[:, -1]
            pos += 1
        out = torch.stack(frames, 1)
        return out

    @torch.no_grad()
    def text_prompt(self, ids: torch.Tensor) -> torch.Tensor:
        return self.embed_text[ids.to(self.device).long()]

    @torch.no_grad()
    def speak(self, text_ids: torch.Tensor, max_frames: int = 125) -> torch.Tensor:
        """Token ids of a formatted prompt [T] (e.g. "[0]text" with the checkpoint's
        tokenizer) -> 24 kHz audio [samples] through the Mimi codec."""
        frames = self.generate_frames(self.text_prompt(text_ids.view(1, -1)), max_frames)[0]
        keep = ~((frames[:, :-1] == self.cfg.codebook_eos_token_id).all(-1))
        frames = frames[keep]
        if self.codec is None:
            raise ValueError("checkpoint has no codec_model.* tensors")
        return self.codec.decode(frames.t()[None])[0, 0]
