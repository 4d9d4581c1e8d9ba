"""CLIP dual encoder: the text tower (``models/flux_text.py``) and the vision
tower (``models/vit.py``) projected into one space, with the learned
temperature; similarity logits = exp(logit_scale) * cos(text, image).

Reference: the reference's embedding / vision families (crates/rlx-vision,
the CLIP text encoder of crates/rlx-flux1); transformers ``CLIPModel`` is the
CPU oracle.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .flux_text import CLIPTextConfig, CLIPTextEncoder, _linear
from .vit import VisionConfig, VisionEncoder


class CLIPDualEncoder:
    def __init__(self, config: dict, weights, device="cpu"):
        get = (lambda n: weights.take(n)) if hasattr(weights, "take") else (lambda n: weights[n])
        self.text = CLIPTextEncoder(CLIPTextConfig.from_dict(config["text_config"]), weights, device=device)
        self.vision = VisionEncoder(VisionConfig.from_dict(config), weights, device=device)
        dt = self.text.dtype
        self.text_proj = get("text_projection.weight").to(self.text.device, dt).contiguous()
        self.logit_scale = float(get("logit_scale").float().reshape(()))

    def embed_text(self, ids: torch.Tensor, normalize: bool = True) -> torch.Tensor:
        _, pooled = self.text(ids)
        e = _linear(pooled.to(self.text.dtype), self.text_proj).float()
        return F.normalize(e, dim=-1) if normalize else e

    def embed_image(self, pixels: torch.Tensor, normalize: bool = True) -> torch.Tensor:
        return self.vision.embed(pixels, normalize=normalize)

    def logits_per_image(self, pixels: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        """[images, texts] similarity logits."""
        i, t = self.embed_image(pixels).cpu(), self.embed_text(ids).cpu()
        return torch.exp(torch.tensor(self.logit_scale)) * i @ t.t()
