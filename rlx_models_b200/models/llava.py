"""Vision-language models of the LLaVA form: a ViT vision tower, a projector,
and a decoder LM whose prompt carries image placeholder tokens.

    features = vision tower hidden state of layer ``vision_feature_layer``
               (HF hidden_states indexing: k = after k blocks, negative from the end),
               the CLS token dropped ("default") or kept ("full")
    tokens   = linear_2(act(linear_1(features)))          (projector, H_vision -> H_text)
    prompt   = the text ids with each image's placeholder run (``image_token_index``,
               one per image token, as the processors expand them); the LM's input
               embeddings at those positions are replaced by ``tokens``, in order

The vision tower and projector run once per image (``image_features``); the
LM is this package's decoder (``models/decoder.py``) on the GPU, or the fp32
oracle on CPU, both taking the replacement rows through ``ForwardBatch.mm_rows``
/ ``mm_embeds`` (``DecoderOracle.forward(..., mm=...)``). The engine places an
image's rows into whichever prefill chunk holds their positions
(``LLMEngine.add_request(..., mm=[(position, embeds)])``).

Checkpoint names: transformers 5 (``model.vision_tower.*``,
``model.multi_modal_projector.*``, ``model.language_model.*``, ``lm_head``) and
the earlier release layout (``vision_tower.*``, ``multi_modal_projector.*``,
``language_model.model.*``, ``language_model.lm_head``).

Reference: the reference's VLM runners share one vision-language base
(crates/rlx-vlm-base) over their vision towers and LMs (crates/rlx-qwen3-vl/src/vl_runner.rs:39,
crates/rlx-minicpm-v); transformers' LlavaForConditionalGeneration is the CPU oracle.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from ..config import DecoderConfig
from .flux_text import _linear
from .vit import VisionConfig, VisionEncoder


@dataclass
class LlavaConfig:
    vision: VisionConfig
    text: DecoderConfig
    image_token_index: int = 32000
    vision_feature_layer: int = -2
    vision_feature_select_strategy: str = "default"   # "default" (drop CLS) | "full"
    projector_hidden_act: str = "gelu"

    @classmethod
    def from_dict(cls, d: dict) -> "LlavaConfig":
        vc = dict(d.get("vision_config") or {})
        vc.setdefault("model_type", "clip_vision_model")
        tc = dict(d.get("text_config") or {})
        tc.setdefault("model_type", "llama")
        layer = d.get("vision_feature_layer", -2)
        if isinstance(layer, (list, tuple)):
            raise NotImplementedError("multi-layer vision features (a list of layers) are not supported")
        return cls(vision=VisionConfig.from_dict(vc), text=DecoderConfig.from_hf_dict(tc),
                   image_token_index=int(d.get("image_token_index", d.get("image_token_id", 32000))),
                   vision_feature_layer=int(layer),
                   vision_feature_select_strategy=d.get("vision_feature_select_strategy", "default"),
                   projector_hidden_act=d.get("projector_hidden_act", "gelu"))


_PREFIXES = {
    "vision": ("model.vision_tower.", "vision_tower."),
    "proj": ("model.multi_modal_projector.", "multi_modal_projector."),
    "text": ("model.language_model.", "language_model.model."),
}


class _View:
    """One part of a LLaVA checkpoint under the names its component reads."""

    def __init__(self, weights, part: str):
        self.w = weights
        self.get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])
        self.map: dict[str, str] = {}
        for k in weights.keys():
            for pre in _PREFIXES[part]:
                if k.startswith(pre):
                    rest = k[len(pre):]
                    self.map["model." + rest if part == "text" else rest] = k
            if part == "text" and k in ("lm_head.weight", "language_model.lm_head.weight"):
                self.map["lm_head.weight"] = k

    def keys(self):
        return list(self.map)

    def __contains__(self, name):
        return name in self.map

    def __getitem__(self, name):
        return self.get(self.map[name])

    def take(self, name, dtype=None, device=None):
        t = self[name]
        return t if dtype is None and device is None else t.to(device=device, dtype=dtype)

    def dict(self) -> dict:
        return {k: self[k] for k in self.map}


class LlavaVLM:
    def __init__(self, cfg: LlavaConfig, weights, device="cpu", lm=None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.vision = VisionEncoder(cfg.vision, _View(weights, "vision"), device=device)
        pv = _View(weights, "proj")
        dt = self.vision.dtype
        dv = lambda n: pv[n].to(self.device, dt).contiguous() if n in pv else None  # noqa: E731
        self.p1 = (dv("linear_1.weight"), dv("linear_1.bias"))
        self.p2 = (dv("linear_2.weight"), dv("linear_2.bias"))
        text = _View(weights, "text")
        if lm is not None:
            self.lm = lm
        elif self.device.type == "cuda":
            from ..registry import build_model
            self.lm = build_model(cfg.text, text, device=self.device)
        else:
            from .oracle import DecoderOracle
            self.lm = DecoderOracle(cfg.text, {k: v.float() for k, v in text.dict().items()}, device=self.device)

    def _act(self, x):
        a = self.cfg.projector_hidden_act
        if a == "gelu":
            return F.gelu(x)
        if a in ("gelu_pytorch_tanh", "gelu_new"):
            return F.gelu(x, approximate="tanh")
        if a == "quick_gelu":
            return x * torch.sigmoid(1.702 * x)
        if a == "silu":
            return F.silu(x)
        raise NotImplementedError(f"projector activation {a!r}")

    @torch.no_grad()
    def image_features(self, pixels: torch.Tensor) -> torch.Tensor:
        """pixels [B, 3, S, S] (preprocessed) -> projected image tokens [B, N, H_text]."""
        x = self.vision.hidden_at(pixels, self.cfg.vision_feature_layer)
        if self.cfg.vision_feature_select_strategy == "default":
            x = x[:, 1:]
        h = self._act(_linear(x, *self.p1).float()).to(x.dtype)
        return _linear(h, *self.p2)

    def placeholder_rows(self, ids: list[int]) -> list[int]:
        return [i for i, t in enumerate(ids) if t == self.cfg.image_token_index]

    @torch.no_grad()
    def mm_segments(self, ids: list[int], pixels: torch.Tensor) -> list[tuple[int, torch.Tensor]]:
        """(first position, rows) of every image's placeholder run in ``ids``,
        filled with that image's projected tokens."""
        feats = self.image_features(pixels)
        rows = self.placeholder_rows(ids)
        n_img, n_tok = feats.shape[0], feats.shape[1]
        if len(rows) != n_img * n_tok:
            raise ValueError(f"prompt has {len(rows)} image placeholders; {n_img} images need {n_img * n_tok}")
        segs = []
        for j in range(n_img):
            r = rows[j * n_tok:(j + 1) * n_tok]
            if r[-1] - r[0] != n_tok - 1:
                raise ValueError(f"image {j}'s placeholders are not one contiguous run")
            segs.append((r[0], feats[j]))
        return segs

    @torch.no_grad()
    def oracle_logits(self, ids: list[int], pixels: torch.Tensor) -> torch.Tensor:
        """fp32 logits [T, V] of the whole prompt (the CPU oracle path)."""
        segs = self.mm_segments(ids, pixels)
        rows = torch.cat([torch.arange(p, p + e.shape[0]) for p, e in segs])
        emb = torch.cat([e for _, e in segs]).float()
        lg, _ = self.lm.forward(torch.tensor(ids), mm=(rows, emb))
        return lg
