"""fp32 FLUX.1 DiT oracle (plain torch, CPU or any device).

Implements the BFL model semantics that the reference's graph builder
reproduces (rlx-flux1 src/transformer.rs: `double_block` :351, `single_block`
:405, `final_layer` :433, `Flux1Dit::forward` :490; src/embed.rs MLP
embedders): LayerNorm without affine (eps 1e-6), adaLN modulation
``(1 + scale) * LN(x) + shift`` from ``Linear(SiLU(vec))``, per-head RMSNorm
on q and k with learned scales, interleaved-pair 3-axis RoPE, joint
non-causal attention over concat(txt, img), GELU (tanh) MLPs, gated
residuals, and the final adaLN + linear projection.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from ..config import FluxConfig
from .flux_common import apply_rope_interleaved, rope_tables, timestep_embedding


class FluxOracle:
    def __init__(self, cfg: FluxConfig, weights: dict[str, torch.Tensor], device="cpu"):
        self.cfg = cfg
        self.dev = torch.device(device)
        self.w = {k: v.to(self.dev, torch.float32) for k, v in weights.items()}

    def _lin(self, name, x):
        b = self.w.get(name + ".bias")
        return F.linear(x, self.w[name + ".weight"], b)

    def _mlp_embed(self, name, x):
        return self._lin(name + ".out_layer", F.silu(self._lin(name + ".in_layer", x)))

    @staticmethod
    def _ln(x, eps):
        return F.layer_norm(x, (x.shape[-1],), eps=eps)

    def _rms(self, x, scale):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.cfg.eps) * scale

    def _attn(self, q, k, v, cos, sin):
        # q, k, v: [B, heads, L, D]
        q = apply_rope_interleaved(q, cos, sin)
        k = apply_rope_interleaved(k, cos, sin)
        s = q @ k.transpose(-1, -2) / math.sqrt(q.shape[-1])
        o = torch.softmax(s, -1) @ v
        B, Hh, L, D = o.shape
        return o.permute(0, 2, 1, 3).reshape(B, L, Hh * D)

    def _split_heads(self, qkv):
        B, L, _ = qkv.shape
        c = self.cfg
        x = qkv.reshape(B, L, 3, c.num_heads, c.head_dim).permute(2, 0, 3, 1, 4)
        return x[0], x[1], x[2]

    def forward(self, img, img_ids, txt, txt_ids, timesteps, y, guidance=None) -> torch.Tensor:
        """img [B, Li, in], txt [B, Lt, ctx], ids [L, 3] (shared across the batch),
        timesteps/guidance [B], y [B, vec]. Returns the velocity [B, Li, out]."""
        c, d = self.cfg, self.dev
        img, txt, y = img.to(d).float(), txt.to(d).float(), y.to(d).float()
        img = self._lin("img_in", img)
        vec = self._mlp_embed("time_in", timestep_embedding(timesteps).to(d))
        if c.guidance_embed:
            vec = vec + self._mlp_embed("guidance_in", timestep_embedding(guidance).to(d))
        vec = vec + self._mlp_embed("vector_in", y)
        txt = self._lin("txt_in", txt)
        cos, sin = rope_tables(torch.cat([txt_ids, img_ids]), c.axes_dim, c.theta)
        cos, sin = cos.to(d), sin.to(d)
        Lt = txt.shape[1]
        sv = F.silu(vec)[:, None, :]
        for i in range(c.depth):
            p = f"double_blocks.{i}."
            im = self._lin(p + "img_mod.lin", sv).chunk(6, -1)
            tm = self._lin(p + "txt_mod.lin", sv).chunk(6, -1)
            iq, ik, iv = self._split_heads(self._lin(p + "img_attn.qkv", (1 + im[1]) * self._ln(img, c.eps) + im[0]))
            tq, tk, tv = self._split_heads(self._lin(p + "txt_attn.qkv", (1 + tm[1]) * self._ln(txt, c.eps) + tm[0]))
            iq = self._rms(iq, self.w[p + "img_attn.norm.query_norm.scale"])
            ik = self._rms(ik, self.w[p + "img_attn.norm.key_norm.scale"])
            tq = self._rms(tq, self.w[p + "txt_attn.norm.query_norm.scale"])
            tk = self._rms(tk, self.w[p + "txt_attn.norm.key_norm.scale"])
            a = self._attn(torch.cat([tq, iq], 2), torch.cat([tk, ik], 2), torch.cat([tv, iv], 2), cos, sin)
            ta, ia = a[:, :Lt], a[:, Lt:]
            img = img + im[2] * self._lin(p + "img_attn.proj", ia)
            img = img + im[5] * self._lin(p + "img_mlp.2", F.gelu(
                self._lin(p + "img_mlp.0", (1 + im[4]) * self._ln(img, c.eps) + im[3]), approximate="tanh"))
            txt = txt + tm[2] * self._lin(p + "txt_attn.proj", ta)
            txt = txt + tm[5] * self._lin(p + "txt_mlp.2", F.gelu(
                self._lin(p + "txt_mlp.0", (1 + tm[4]) * self._ln(txt, c.eps) + tm[3]), approximate="tanh"))
        x = torch.cat([txt, img], 1)
        H = c.hidden_size
        for i in range(c.depth_single_blocks):
            p = f"single_blocks.{i}."
            shift, scale, gate = self._lin(p + "modulation.lin", sv).chunk(3, -1)
            h = self._lin(p + "linear1", (1 + scale) * self._ln(x, c.eps) + shift)
            q, k, v = self._split_heads(h[..., :3 * H])
            q = self._rms(q, self.w[p + "norm.query_norm.scale"])
            k = self._rms(k, self.w[p + "norm.key_norm.scale"])
            a = self._attn(q, k, v, cos, sin)
            x = x + gate * self._lin(p + "linear2", torch.cat([a, F.gelu(h[..., 3 * H:], approximate="tanh")], -1))
        img = x[:, Lt:]
        shift, scale = self._lin("final_layer.adaLN_modulation.1", sv).chunk(2, -1)
        return self._lin("final_layer.linear", (1 + scale) * self._ln(img, c.eps) + shift)
