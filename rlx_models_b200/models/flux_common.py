"""FLUX.1 pieces shared by the fp32 oracle and the GPU DiT: tensor-name
contract, seeded init, 3-axis RoPE tables, timestep embedding, the shifted
Euler schedule and 2x2 latent packing.

Semantics follow the BFL reference model as the reference framework
implements it (rlx-flux1 src/embed.rs:30-45 timestep embedding,
src/rope.rs:20-78 3-axis RoPE, src/sampler.rs:20-140 schedule / pack /
Euler, src/weights.rs:202 query/key row de-interleave).
"""
from __future__ import annotations

import math

import torch

from ..config import FluxConfig
from ..weights.init import TensorSpec, init_tensor


def flux_tensor_specs(cfg: FluxConfig) -> list[TensorSpec]:
    H, M, D = cfg.hidden_size, cfg.mlp_hidden, cfg.head_dim
    specs: list[TensorSpec] = []

    def lin(name, out, inp, bias=True):
        specs.append(TensorSpec(name + ".weight", (out, inp), "matrix"))
        if bias:
            specs.append(TensorSpec(name + ".bias", (out,), "bias"))

    lin("img_in", H, cfg.in_channels)
    lin("txt_in", H, cfg.context_in_dim)
    lin("time_in.in_layer", H, 256)
    lin("time_in.out_layer", H, H)
    lin("vector_in.in_layer", H, cfg.vec_in_dim)
    lin("vector_in.out_layer", H, H)
    if cfg.guidance_embed:
        lin("guidance_in.in_layer", H, 256)
        lin("guidance_in.out_layer", H, H)
    for i in range(cfg.depth):
        for s in ("img", "txt"):
            p = f"double_blocks.{i}.{s}"
            lin(p + "_mod.lin", 6 * H, H)
            lin(p + "_attn.qkv", 3 * H, H, cfg.qkv_bias)
            lin(p + "_attn.proj", H, H)
            lin(p + "_mlp.0", M, H)
            lin(p + "_mlp.2", H, M)
            specs.append(TensorSpec(p + "_attn.norm.query_norm.scale", (D,), "norm"))
            specs.append(TensorSpec(p + "_attn.norm.key_norm.scale", (D,), "norm"))
    for i in range(cfg.depth_single_blocks):
        p = f"single_blocks.{i}"
        lin(p + ".linear1", 3 * H + M, H)
        lin(p + ".linear2", H, H + M)
        lin(p + ".modulation.lin", 3 * H, H)
        specs.append(TensorSpec(p + ".norm.query_norm.scale", (D,), "norm"))
        specs.append(TensorSpec(p + ".norm.key_norm.scale", (D,), "norm"))
    lin("final_layer.adaLN_modulation.1", 2 * H, H)
    lin("final_layer.linear", cfg.out_channels, H)
    return specs


def flux_random_weights(cfg: FluxConfig, seed: int = 0, device="cpu", dtype=torch.bfloat16,
                        bias_std: float = 0.0) -> dict[str, torch.Tensor]:
    """Seeded N(0, 0.02) matrices, unit norm scales; ``bias_std`` > 0 draws
    biases too (tests), else zeros."""
    out = {}
    for s in flux_tensor_specs(cfg):
        if s.kind == "bias" and bias_std > 0:
            s = TensorSpec(s.name, s.shape, "matrix", s.dtype)
            out[s.name] = init_tensor(s, seed, device, dtype, std=bias_std)
        else:
            out[s.name] = init_tensor(s, seed, device, dtype)
    return out


# -- positions and RoPE ---------------------------------------------------------

def position_ids(txt_len: int, h: int, w: int) -> torch.Tensor:
    """[txt_len + h*w, 3] float64 ids, text first: text rows are (0, 0, 0),
    image row (r, c) is (0, r, c)."""
    ids = torch.zeros(txt_len + h * w, 3, dtype=torch.float64)
    r = torch.arange(h, dtype=torch.float64).repeat_interleave(w)
    c = torch.arange(w, dtype=torch.float64).repeat(h)
    ids[txt_len:, 1] = r
    ids[txt_len:, 2] = c
    return ids


def rope_angles(ids: torch.Tensor, axes_dim=(16, 56, 56), theta: float = 10000.0) -> torch.Tensor:
    """[L, head_dim/2] float64 angles. Pair j of axis a (width w_a) turns at
    theta^(-2j / w_a) times the position along a; axes are concatenated."""
    cols = []
    for a, wdt in enumerate(axes_dim):
        j = torch.arange(wdt // 2, dtype=torch.float64)
        omega = 1.0 / theta ** (2 * j / wdt)
        cols.append(ids[:, a:a + 1] * omega[None, :])
    return torch.cat(cols, 1)


def rope_tables(ids: torch.Tensor, axes_dim=(16, 56, 56), theta: float = 10000.0):
    ang = rope_angles(ids, axes_dim, theta)
    return torch.cos(ang).float(), torch.sin(ang).float()


def apply_rope_interleaved(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """BFL convention: pairs (2j, 2j+1) rotate by angle j. x [..., L, D], cos/sin [L, D/2]."""
    x1, x2 = x[..., 0::2], x[..., 1::2]
    o1 = x1 * cos - x2 * sin
    o2 = x1 * sin + x2 * cos
    return torch.stack([o1, o2], -1).flatten(-2)


def deinterleave_perm(head_dim: int) -> torch.Tensor:
    """Within-head row order that turns interleaved-pair RoPE into the
    half-split form (pair j -> dims j and j + D/2): [0, 2, 4, ..., 1, 3, 5, ...]."""
    return torch.cat([torch.arange(0, head_dim, 2), torch.arange(1, head_dim, 2)])


# -- conditioning ---------------------------------------------------------------

def timestep_embedding(t: torch.Tensor, dim: int = 256, max_period: float = 10000.0,
                       time_factor: float = 1000.0) -> torch.Tensor:
    """[B] -> [B, dim] float32: t * 1000 against exp(-ln(max_period) i / half), [cos | sin]."""
    t = t.double() * time_factor
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float64) / half)
    args = t[:, None] * freqs[None]
    return torch.cat([torch.cos(args), torch.sin(args)], -1).float()


# -- sampling -------------------------------------------------------------------

def schedule(steps: int, image_seq_len: int, shift: bool = True, base_shift: float = 0.5,
             max_shift: float = 1.15) -> list[float]:
    """steps + 1 timesteps from 1 to 0; [dev] shifts them by mu(image_seq_len)
    (linear in the sequence length between 256 -> base_shift and 4096 -> max_shift)."""
    steps = max(1, steps)
    ts = [1.0 - i / steps for i in range(steps + 1)]
    if not shift:
        return ts
    m = (max_shift - base_shift) / (4096 - 256)
    mu = m * image_seq_len + (base_shift - m * 256)
    return [0.0 if t <= 0 else math.exp(mu) / (math.exp(mu) + (1.0 / t - 1.0)) for t in ts]


def pack(latents: torch.Tensor) -> torch.Tensor:
    """[B, C, H, W] -> [B, (H/2)(W/2), C*4], channel order (c, ph, pw)."""
    B, C, H, W = latents.shape
    x = latents.reshape(B, C, H // 2, 2, W // 2, 2).permute(0, 2, 4, 1, 3, 5)
    return x.reshape(B, (H // 2) * (W // 2), C * 4)


def unpack(x: torch.Tensor, C: int, H: int, W: int) -> torch.Tensor:
    B = x.shape[0]
    x = x.reshape(B, H // 2, W // 2, C, 2, 2).permute(0, 3, 1, 4, 2, 5)
    return x.reshape(B, C, H, W)


def euler(x: torch.Tensor, timesteps: list[float], velocity) -> torch.Tensor:
    """x += (t_next - t) * v(x, t) over consecutive timestep pairs."""
    for i in range(len(timesteps) - 1):
        t, tn = timesteps[i], timesteps[i + 1]
        x = x + (tn - t) * velocity(x, t, i)
    return x
