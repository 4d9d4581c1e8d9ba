"""LFM2-VL (Liquid AI's vision-language models): a SigLIP 2 NaFlex image tower,
a pixel-unshuffle projector and the LFM2 hybrid (short-conv + attention) LM.

    image    NaFlex patches at the image's aspect ratio -> SigLIP 2 tower (last
             hidden state after its post-norm) -> the valid patches as an [h, w, C]
             grid -> pixel unshuffle by 2 ([h/2, w/2, 4C]) -> LayerNorm -> linear ->
             GELU -> linear -> one LM token per 2 x 2 patch block
    prompt   the text ids with one ``image_token_id`` per image token (the
             processor's tiles / thumbnails each bring their own run); the LM's input
             embeddings at those positions are replaced by the image tokens, in order

The tower is ``models/vit.py`` ``Siglip2Encoder``; the LM is ``models/lfm2.py``
(``Lfm2LM`` on the GPU through the engine with ``ForwardBatch.mm_rows``, the
fp32 ``Lfm2Oracle`` on CPU).

Checkpoint names: transformers' Lfm2VlForConditionalGeneration.

Reference: crates/rlx-lfm-vl (LFM2-VL); transformers'
Lfm2VlForConditionalGeneration is the CPU oracle.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .flux_text import _linear
from .llava import _View
from .vit import Siglip2Encoder, VisionConfig


@dataclass
class Lfm2VlConfig:
    vision: VisionConfig
    text: dict
    image_token_id: int = 396
    downsample_factor: int = 2
    projector_use_layernorm: bool = True
    projector_hidden_act: str = "gelu"

    @classmethod
    def from_dict(cls, d: dict) -> "Lfm2VlConfig":
        vc = dict(d.get("vision_config") or {})
        vc.setdefault("model_type", "siglip2_vision_model")
        return cls(vision=VisionConfig.from_dict(vc), text=dict(d.get("text_config") or {}),
                   image_token_id=int(d.get("image_token_id", 396)),
                   downsample_factor=int(d.get("downsample_factor", 2)),
                   projector_use_layernorm=bool(d.get("projector_use_layernorm", True)),
                   projector_hidden_act=d.get("projector_hidden_act", "gelu"))


class _Prefix:
    def __init__(self, weights, prefix):
        self.w, self.p = weights, prefix
        self.get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])

    def keys(self):
        return [k[len(self.p):] for k in self.w.keys() if k.startswith(self.p)]

    def __contains__(self, k):
        return (self.p + k) in self.w

    def __getitem__(self, k):
        return self.get(self.p + k)

    def take(self, k, **kw):
        return self[k]


class Lfm2VlModel:
    def __init__(self, cfg: Lfm2VlConfig, weights, device="cpu", lm=None):
        from .lfm2 import Lfm2Config
        self.cfg = cfg
        self.device = torch.device(device)
        self.vision = Siglip2Encoder(cfg.vision, _Prefix(weights, "model.vision_tower."), device=device)
        dt = self.vision.dtype
        get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])
        names = set(weights.keys())
        p = "model.multi_modal_projector."
        dv = lambda n: get(n).to(self.device, dt).contiguous() if n in names else None  # noqa: E731
        f32 = lambda n: get(n).to(self.device, torch.float32) if n in names else None  # noqa: E731
        self.ln = (f32(p + "layer_norm.weight"), f32(p + "layer_norm.bias")) if cfg.projector_use_layernorm else None
        self.p1 = (dv(p + "linear_1.weight"), dv(p + "linear_1.bias"))
        self.p2 = (dv(p + "linear_2.weight"), dv(p + "linear_2.bias"))
        text = _View(weights, "text")
        tcfg = Lfm2Config.from_dict({**cfg.text, "model_type": "lfm2"})
        if lm is not None:
            self.lm = lm
        elif self.device.type == "cuda":
            from .lfm2 import Lfm2LM
            self.lm = Lfm2LM(tcfg, text, device=self.device)
        else:
            from .lfm2 import Lfm2Oracle
            self.lm = Lfm2Oracle(tcfg, {k: v.float() for k, v in text.dict().items()}, device=self.device)

    def _unshuffle(self, g: torch.Tensor) -> torch.Tensor:
        """[h, w, C] -> [h/f, w/f, f*f*C], the released projector's channel order."""
        f = self.cfg.downsample_factor
        h, w, C = g.shape
        x = g.reshape(h, w // f, C * f).permute(1, 0, 2).reshape(w // f, h // f, C * f * f)
        return x.permute(1, 0, 2)

    @torch.no_grad()
    def image_features(self, patches, shapes, valid) -> list:
        """NaFlex inputs of a batch of images -> per image its LM tokens [n, H_text]."""
        x, _ = self.vision.forward_patches(patches, shapes, valid)
        out = []
        act = F.gelu if self.cfg.projector_hidden_act == "gelu" else F.silu
        for i, (h, w) in enumerate(shapes.tolist()):
            g = self._unshuffle(x[i, :h * w].float().reshape(h, w, -1))
            g = g.reshape(-1, g.shape[-1])
            if self.ln is not None:
                g = F.layer_norm(g, (g.shape[-1],), *self.ln, 1e-5)
            y = act(_linear(g.to(self.vision.dtype).contiguous(), *self.p1).float())
            out.append(_linear(y.to(self.vision.dtype).contiguous(), *self.p2))
        return out

    def mm_segments(self, ids: list[int], patches, shapes, valid) -> list[tuple[int, torch.Tensor]]:
        """(first position, rows) of each contiguous run of image placeholders,
        filled in order with the images' tokens."""
        feats = torch.cat(self.image_features(patches, shapes, valid))
        rows = [i for i, t in enumerate(ids) if t == self.cfg.image_token_id]
        if len(rows) != feats.shape[0]:
            raise ValueError(f"prompt has {len(rows)} image placeholders; the images give {feats.shape[0]} tokens")
        segs, start, used = [], 0, 0
        for j in range(1, len(rows) + 1):
            if j == len(rows) or rows[j] != rows[j - 1] + 1:
                n = j - start
                segs.append((rows[start], feats[used:used + n]))
                used += n
                start = j
        return segs

    def segments_for_images(self, ids: list[int], images, max_patches: int = 256):
        """Images (paths / PIL / arrays, in placeholder order) -> ``mm_segments``."""
        patches, shapes, valid = self.vision.patchify(list(images), max_patches)
        return self.mm_segments(ids, patches, shapes, valid)

    def image_tokens(self, height: int, width: int, max_patches: int = 256) -> int:
        """LM tokens one image of this size brings (placeholders the prompt needs)."""
        from .vit import naflex_size
        p, f = self.cfg.vision.patch_size, self.cfg.downsample_factor
        th, tw = naflex_size(height, width, p, max_patches)
        return (th // p // f) * (tw // p // f)

    @torch.no_grad()
    def oracle_logits(self, ids: list[int], patches, shapes, valid) -> torch.Tensor:
        segs = self.mm_segments(ids, patches, shapes, valid)
        rows = torch.cat([torch.arange(p, p + e.shape[0]) for p, e in segs])
        emb = torch.cat([e for _, e in segs]).float()
        return self.lm.logits(ids, mm=(rows, emb))
