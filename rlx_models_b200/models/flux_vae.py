"""FLUX.1 autoencoder decoder (16 latent channels) and the text-to-image
pipeline around the DiT.

The FLUX.1 AE is an LDM ``AutoencoderKL``: conv_in (16 -> 512), a middle block
(ResNet, single-head spatial self-attention, ResNet), four up levels with
channels 512, 512, 256, 128 (three ResNets each, nearest-2x upsample + conv
after all but the last), GroupNorm(32) + SiLU + conv_out (128 -> 3). ResNets
are GroupNorm -> SiLU -> conv3x3, twice, with a 1x1 shortcut when the width
changes. Latents are denormalised as z / 0.3611 + 0.1159 before decoding.

Weights load under diffusers names (``decoder.up_blocks.0.resnets.0...``) or
BFL / LDM names (``decoder.up.3.block.0...``, 1x1-conv attention q/k/v,
up levels in reverse order), mapped by :func:`ldm_to_diffusers`.

The decoder runs once per image (the DiT's 28 steps dominate), so it uses
torch convolutions; the DiT steps are this package's kernels.

Reference: crates/rlx-flux1/src/vae.rs (`flux1_vae_config`, SCALING_FACTOR /
SHIFT_FACTOR, `ldm_to_diffusers`), src/pipeline.rs:215-600.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

SCALING_FACTOR = 0.3611
SHIFT_FACTOR = 0.1159


@dataclass
class VAEConfig:
    latent_channels: int = 16
    out_channels: int = 3
    block_out_channels: list = field(default_factory=lambda: [128, 256, 512, 512])
    layers_per_block: int = 2
    norm_num_groups: int = 32
    scaling_factor: float = SCALING_FACTOR
    shift_factor: float = SHIFT_FACTOR


def ldm_to_diffusers(key: str, num_levels: int = 4) -> str | None:
    """BFL / LDM decoder name -> diffusers name (None if not an LDM decoder key)."""
    if not key.startswith("decoder."):
        return None
    r = key[len("decoder."):]
    if r.startswith("mid."):
        r = r[4:]
        blk, _, rest = r.partition(".")
        if blk in ("block_1", "block_2"):
            return f"decoder.mid_block.resnets.{int(blk[-1]) - 1}.{rest}"
        if blk == "attn_1":
            n, _, p = rest.partition(".")
            n = {"norm": "group_norm", "q": "to_q", "k": "to_k", "v": "to_v", "proj_out": "to_out.0"}.get(n)
            return f"decoder.mid_block.attentions.0.{n}.{p}" if n else None
        return None
    if r.startswith("up."):
        lvl, _, rest = r[3:].partition(".")
        i = num_levels - 1 - int(lvl)
        if rest.startswith("block."):
            j, _, t = rest[6:].partition(".")
            t = t.replace("nin_shortcut", "conv_shortcut")
            return f"decoder.up_blocks.{i}.resnets.{j}.{t}"
        if rest.startswith("upsample.conv."):
            return f"decoder.up_blocks.{i}.upsamplers.0.conv.{rest[len('upsample.conv.'):]}"
        return None
    if r.startswith("norm_out."):
        return "decoder.conv_norm_out." + r[len("norm_out."):]
    if r.startswith(("conv_in.", "conv_out.")):
        return None  # same name in both layouts
    return None


class VAEDecoder:
    def __init__(self, cfg: VAEConfig, weights, device="cpu", dtype: torch.dtype | None = None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype or (torch.bfloat16 if self.device.type == "cuda" else torch.float32)
        names = list(weights.keys())
        w = {}
        for n in names:
            if not n.startswith("decoder."):
                continue
            t = weights.take(n) if hasattr(weights, "take") else weights[n]
            d = ldm_to_diffusers(n, len(cfg.block_out_channels)) or n
            if ".attentions.0.to_" in d and d.endswith(".weight") and t.dim() == 4:
                t = t[:, :, 0, 0]  # LDM 1x1-conv attention projections -> linear
            w[d] = t.to(self.device, self.dtype)
        self.w = w

    def _gn(self, x, name, eps=1e-6):
        return F.group_norm(x, self.cfg.norm_num_groups, self.w[name + ".weight"], self.w[name + ".bias"], eps)

    def _conv(self, x, name, pad=1):
        return F.conv2d(x, self.w[name + ".weight"], self.w[name + ".bias"], padding=pad)

    def _resnet(self, x, p):
        h = self._conv(F.silu(self._gn(x, p + ".norm1")), p + ".conv1")
        h = self._conv(F.silu(self._gn(h, p + ".norm2")), p + ".conv2")
        if p + ".conv_shortcut.weight" in self.w:
            x = self._conv(x, p + ".conv_shortcut", pad=0)
        return x + h

    def _attn(self, x, p):
        B, C, H, W = x.shape
        h = self._gn(x, p + ".group_norm").view(B, C, H * W).transpose(1, 2)
        q = F.linear(h, self.w[p + ".to_q.weight"], self.w[p + ".to_q.bias"])
        k = F.linear(h, self.w[p + ".to_k.weight"], self.w[p + ".to_k.bias"])
        v = F.linear(h, self.w[p + ".to_v.weight"], self.w[p + ".to_v.bias"])
        a = F.scaled_dot_product_attention(q.unsqueeze(1), k.unsqueeze(1), v.unsqueeze(1)).squeeze(1)
        o = F.linear(a, self.w[p + ".to_out.0.weight"], self.w[p + ".to_out.0.bias"])
        return x + o.transpose(1, 2).reshape(B, C, H, W)

    @torch.no_grad()
    def decode(self, z: torch.Tensor) -> torch.Tensor:
        """z [B, 16, h, w] (DiT latents) -> image [B, 3, 8h, 8w] in [-1, 1] (unclamped)."""
        c = self.cfg
        x = (z.to(self.device, self.dtype) / c.scaling_factor + c.shift_factor)
        x = self._conv(x, "decoder.conv_in")
        x = self._resnet(x, "decoder.mid_block.resnets.0")
        x = self._attn(x, "decoder.mid_block.attentions.0")
        x = self._resnet(x, "decoder.mid_block.resnets.1")
        n = len(c.block_out_channels)
        for i in range(n):
            for j in range(c.layers_per_block + 1):
                x = self._resnet(x, f"decoder.up_blocks.{i}.resnets.{j}")
            if i < n - 1:
                x = F.interpolate(x, scale_factor=2.0, mode="nearest")
                x = self._conv(x, f"decoder.up_blocks.{i}.upsamplers.0.conv")
        x = F.silu(self._gn(x, "decoder.conv_norm_out"))
        return self._conv(x, "decoder.conv_out").float()


def vae_tensor_specs(cfg: VAEConfig) -> dict[str, tuple]:
    """Diffusers-named decoder tensor shapes (random init for tests / benches)."""
    ch = list(reversed(cfg.block_out_channels))
    s = {"decoder.conv_in.weight": (ch[0], cfg.latent_channels, 3, 3), "decoder.conv_in.bias": (ch[0],)}

    def res(p, i, o):
        s.update({p + ".norm1.weight": (i,), p + ".norm1.bias": (i,), p + ".conv1.weight": (o, i, 3, 3),
                  p + ".conv1.bias": (o,), p + ".norm2.weight": (o,), p + ".norm2.bias": (o,),
                  p + ".conv2.weight": (o, o, 3, 3), p + ".conv2.bias": (o,)})
        if i != o:
            s.update({p + ".conv_shortcut.weight": (o, i, 1, 1), p + ".conv_shortcut.bias": (o,)})

    res("decoder.mid_block.resnets.0", ch[0], ch[0])
    a = "decoder.mid_block.attentions.0."
    s.update({a + "group_norm.weight": (ch[0],), a + "group_norm.bias": (ch[0],)})
    for n in ("to_q", "to_k", "to_v", "to_out.0"):
        s.update({a + n + ".weight": (ch[0], ch[0]), a + n + ".bias": (ch[0],)})
    res("decoder.mid_block.resnets.1", ch[0], ch[0])
    prev = ch[0]
    for i, o in enumerate(ch):
        for j in range(cfg.layers_per_block + 1):
            res(f"decoder.up_blocks.{i}.resnets.{j}", prev if j == 0 else o, o)
        prev = o
        if i < len(ch) - 1:
            s.update({f"decoder.up_blocks.{i}.upsamplers.0.conv.weight": (o, o, 3, 3),
                      f"decoder.up_blocks.{i}.upsamplers.0.conv.bias": (o,)})
    s.update({"decoder.conv_norm_out.weight": (ch[-1],), "decoder.conv_norm_out.bias": (ch[-1],),
              "decoder.conv_out.weight": (cfg.out_channels, ch[-1], 3, 3), "decoder.conv_out.bias": (cfg.out_channels,)})
    return s


def vae_random_weights(cfg: VAEConfig, seed: int = 0) -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    out = {}
    for n, shp in vae_tensor_specs(cfg).items():
        if "norm" in n:
            out[n] = torch.ones(shp) if n.endswith("weight") else torch.zeros(shp)
        elif n.endswith("bias"):
            out[n] = torch.zeros(shp)
        else:
            fan_in = 1
            for d in shp[1:]:
                fan_in *= d
            out[n] = torch.randn(shp, generator=g) / fan_in ** 0.5
    return out


def to_image(x: torch.Tensor) -> torch.Tensor:
    """[-1, 1] float -> uint8 [B, H, W, 3]."""
    return ((x.clamp(-1, 1) + 1) * 127.5).round().to(torch.uint8).permute(0, 2, 3, 1).cpu()


def save_png(img: torch.Tensor, path: str):
    """uint8 [H, W, 3] -> PNG file (Pillow)."""
    from PIL import Image
    Image.fromarray(img.numpy()).save(path)


class FluxPipeline:
    """Text -> image: T5 context + CLIP pooled vector -> DiT rectified-flow
    sampling (this package's kernels) -> VAE decode."""

    def __init__(self, dit, vae: VAEDecoder, t5=None, clip=None, t5_tokenizer=None, clip_tokenizer=None,
                 max_sequence_length: int = 512):
        self.dit, self.vae, self.t5, self.clip = dit, vae, t5, clip
        self.t5_tok, self.clip_tok = t5_tokenizer, clip_tokenizer
        self.max_len = max_sequence_length

    def encode_prompt(self, prompts: list[str] | None = None, t5_ids=None, clip_ids=None):
        if t5_ids is None:
            t5_ids = torch.tensor([self.t5_tok(p, padding="max_length", max_length=self.max_len,
                                               truncation=True)["input_ids"] for p in prompts])
        if clip_ids is None:
            clip_ids = torch.tensor([self.clip_tok(p, padding="max_length", max_length=77,
                                                   truncation=True)["input_ids"] for p in prompts])
        txt = self.t5(t5_ids)
        _, pooled = self.clip(clip_ids)
        return txt, pooled

    def __call__(self, prompts=None, *, t5_ids=None, clip_ids=None, height=1024, width=1024, steps=28,
                 guidance=3.5, seed=0, txt=None, pooled=None) -> torch.Tensor:
        from .flux import generate_latents
        if txt is None:
            txt, pooled = self.encode_prompt(prompts, t5_ids, clip_ids)
        lat = generate_latents(self.dit, txt.to(self.dit.device, torch.bfloat16),
                               pooled.to(self.dit.device, torch.bfloat16), height=height, width=width, steps=steps,
                               guidance=guidance, seed=seed)
        return self.vae.decode(lat)
