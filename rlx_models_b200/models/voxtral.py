"""Voxtral (Mistral's audio LLM): a Whisper-style audio encoder, a projector
over groups of encoder frames, and a Llama / Mistral decoder whose prompt
carries audio placeholder tokens.

    audio     log-mel features of 30 s windows [n_mels, 3000] -> encoder (two convs with
              GELU, learned positions, pre-LN blocks, final LN) -> [1500, d]
    projector consecutive frames regrouped to rows of ``intermediate_size`` (4 x d in the
              releases) -> linear -> GELU -> linear (no biases) -> one LM token per group
    prompt    the text ids with one ``audio_token_id`` per audio token; the LM's
              input embeddings at those positions are replaced by the projected rows

The encoder is this package's Whisper encoder (``models/whisper.py``,
``encoder_only``); the LM is the package's decoder on the GPU (or the fp32
oracle on CPU) taking the audio rows through ``ForwardBatch.mm_rows`` /
``mm_embeds``, the same injection the LLaVA VLMs use (``models/llava.py``),
so the serving engine places them into whichever prefill chunk holds them.

Checkpoint names: transformers' VoxtralForConditionalGeneration (``audio_tower.*``,
``multi_modal_projector.*``, ``language_model.*``).

Reference: crates/rlx-voxtral (Voxtral audio understanding / transcription);
transformers' VoxtralForConditionalGeneration is the CPU oracle.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from ..config import DecoderConfig
from .flux_text import _linear
from .llava import _View
from .whisper import WhisperConfig, WhisperModel


@dataclass
class VoxtralConfig:
    audio: WhisperConfig
    text: DecoderConfig
    intermediate_size: int = 5120
    audio_token_id: int = 24
    projector_hidden_act: str = "gelu"

    @classmethod
    def from_dict(cls, d: dict) -> "VoxtralConfig":
        ac = dict(d.get("audio_config") or {})
        # the serialised encoder config uses the generic names
        for src, dst in (("hidden_size", "d_model"), ("num_hidden_layers", "encoder_layers"),
                         ("num_attention_heads", "encoder_attention_heads"), ("intermediate_size", "encoder_ffn_dim")):
            if src in ac and dst not in ac:
                ac[dst] = ac[src]
        tc = dict(d.get("text_config") or {})
        tc.setdefault("model_type", "llama")
        return cls(audio=WhisperConfig.from_dict(ac), text=DecoderConfig.from_hf_dict(tc),
                   intermediate_size=int(ac.get("intermediate_size", ac.get("encoder_ffn_dim", 5120))),
                   audio_token_id=int(d.get("audio_token_id", 24)),
                   projector_hidden_act=d.get("projector_hidden_act", "gelu"))


class _EncoderNames:
    """``audio_tower.X`` under the names the Whisper encoder reads (``model.encoder.X``)."""

    def __init__(self, weights):
        self.w = weights
        self.get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])

    def _map(self, n):
        return "audio_tower." + n[len("model.encoder."):] if n.startswith("model.encoder.") else n

    def __contains__(self, n):
        return self._map(n) in self.w

    def __getitem__(self, n):
        return self.get(self._map(n))

    def take(self, n, **kw):
        return self[n]

    def keys(self):
        return ["model.encoder." + k[len("audio_tower."):] for k in self.w.keys() if k.startswith("audio_tower.")]


class VoxtralModel:
    def __init__(self, cfg: VoxtralConfig, weights, device="cpu", lm=None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.encoder = WhisperModel(cfg.audio, _EncoderNames(weights), device=device, encoder_only=True)
        dt = self.encoder.dtype
        get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])
        self.p1 = get("multi_modal_projector.linear_1.weight").to(self.device, dt).contiguous()
        self.p2 = get("multi_modal_projector.linear_2.weight").to(self.device, dt).contiguous()
        text = _View(weights, "text")
        if lm is not None:
            self.lm = lm
        elif self.device.type == "cuda":
            from ..registry import build_model
            self.lm = build_model(cfg.text, text, device=self.device)
        else:
            from .oracle import DecoderOracle
            self.lm = DecoderOracle(cfg.text, {k: v.float() for k, v in text.dict().items()}, device=self.device)

    @torch.no_grad()
    def audio_embeds(self, mel: torch.Tensor) -> torch.Tensor:
        """Log-mel windows [B, n_mels, 2 * max_source_positions] -> projected audio
        tokens [B * frames / group, H_text] (window after window)."""
        h = self.encoder.encode(mel)
        rows = h.reshape(-1, self.cfg.intermediate_size).contiguous()
        act = F.gelu if self.cfg.projector_hidden_act == "gelu" else F.silu
        x = act(_linear(rows, self.p1).float()).to(rows.dtype)
        return _linear(x.contiguous(), self.p2)

    def mm_segments(self, ids: list[int], mel: torch.Tensor) -> list[tuple[int, torch.Tensor]]:
        """(first position, rows) of each contiguous run of audio placeholders in
        ``ids``, filled in order with the projected audio tokens."""
        emb = self.audio_embeds(mel)
        rows = [i for i, t in enumerate(ids) if t == self.cfg.audio_token_id]
        if len(rows) != emb.shape[0]:
            raise ValueError(f"prompt has {len(rows)} audio placeholders; the audio gives {emb.shape[0]} tokens")
        segs, start, used = [], 0, 0
        for j in range(1, len(rows) + 1):
            if j == len(rows) or rows[j] != rows[j - 1] + 1:
                n = j - start
                segs.append((rows[start], emb[used:used + n]))
                used += n
                start = j
        return segs

    @torch.no_grad()
    def oracle_logits(self, ids: list[int], mel: torch.Tensor) -> torch.Tensor:
        """fp32 logits [T, V] of the whole prompt (the CPU oracle path)."""
        segs = self.mm_segments(ids, mel)
        rows = torch.cat([torch.arange(p, p + e.shape[0]) for p, e in segs])
        emb = torch.cat([e for _, e in segs]).float()
        lg, _ = self.lm.forward(torch.tensor(ids), mm=(rows, emb))
        return lg
