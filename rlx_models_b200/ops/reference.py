"""Plain-PyTorch fp32 restatements of every kernel (test oracles, CPU path).

These follow the HF module semantics that the reference mirrors and are the
spec the CUDA kernels are tested against.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    return (xf * torch.rsqrt(var + eps)) * w.float()


def rmsnorm_hf_bf16(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """Exact HF order for bf16 activations: normalise fp32, cast, scale by weight."""
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    return w * (xf * torch.rsqrt(var + eps)).to(x.dtype)


def rope(x: torch.Tensor, positions: torch.Tensor, inv_freq: torch.Tensor, scale: float = 1.0) -> torch.Tensor:
    """Half-split rotary embedding. x: [T, H, D], positions: [T]. With fewer
    than D/2 frequencies only the first 2 * len(inv_freq) dims rotate
    (partial RoPE); the rest pass through."""
    R = 2 * inv_freq.shape[0]
    if R < x.shape[-1]:
        return torch.cat([rope(x[..., :R], positions, inv_freq, scale), x[..., R:].float()], -1)
    freqs = positions.float()[:, None] * inv_freq.float()[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    cos, sin = emb.cos() * scale, emb.sin() * scale
    xf = x.float()
    half = xf.shape[-1] // 2
    rot = torch.cat([-xf[..., half:], xf[..., :half]], dim=-1)
    return xf * cos[:, None, :] + rot * sin[:, None, :]


def rope_interleaved(x: torch.Tensor, positions: torch.Tensor, inv_freq: torch.Tensor,
                     scale: float = 1.0) -> torch.Tensor:
    """Rotary embedding on interleaved pairs (x[2i], x[2i+1]) rotated by
    positions * inv_freq[i] (Llama-4 / GPT-J layout). x: [T, H, D]."""
    xf = x.float()
    a, b = xf[..., 0::2], xf[..., 1::2]
    ang = positions.float()[:, None] * inv_freq.float().to(x.device)[None, :]
    cos, sin = (ang.cos() * scale)[:, None, :], (ang.sin() * scale)[:, None, :]
    return torch.stack([a * cos - b * sin, a * sin + b * cos], -1).flatten(-2)


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return F.silu(gate.float()) * up.float()


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_pos: torch.Tensor, k_pos: torch.Tensor,
              scale: float, causal: bool = True, window: int = 0, sinks: torch.Tensor | None = None,
              softcap: float = 0.0, chunk: int = 0) -> torch.Tensor:
    """Dense GQA attention. q: [Tq, Hq, D], k/v: [Tk, Hkv, D]; returns [Tq, Hq, D] fp32.
    ``softcap`` > 0: scaled scores become softcap * tanh(s / softcap); ``chunk`` > 0:
    a query sees only keys of its own ``chunk``-token block (chunked attention)."""
    Hq, Hkv = q.shape[1], k.shape[1]
    G = Hq // Hkv
    kf = k.float().repeat_interleave(G, dim=1)
    vf = v.float().repeat_interleave(G, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), kf) * scale
    if softcap > 0:
        s = torch.tanh(s / softcap) * softcap
    mask = torch.ones(q.shape[0], k.shape[0], dtype=torch.bool, device=q.device)
    if causal:
        mask &= k_pos[None, :] <= q_pos[:, None]
    if chunk > 0:
        mask &= (k_pos[None, :] // chunk) == (q_pos[:, None] // chunk)
    if window > 0:
        mask &= k_pos[None, :] > (q_pos[:, None] - window)
        if not causal:  # a bidirectional window: |q - k| < window
            mask &= k_pos[None, :] < (q_pos[:, None] + window)
    s = s.masked_fill(~mask[None], float("-inf"))
    if sinks is not None:
        sk = sinks.float()[:, None, None].expand(Hq, q.shape[0], 1)
        s = torch.cat([s, sk], dim=-1)
        p = torch.softmax(s, dim=-1)[..., :-1]
    else:
        p = torch.softmax(s, dim=-1)
    return torch.einsum("hqk,khd->qhd", p, vf)


def gather_paged(cache: torch.Tensor, block_table: torch.Tensor, length: int) -> torch.Tensor:
    """cache [NB, Hkv, 16, D] + block list -> [length, Hkv, D]."""
    nblk = (length + 15) // 16
    pages = cache[block_table[:nblk].long()]  # [nblk, Hkv, 16, D]
    return pages.permute(0, 2, 1, 3).reshape(nblk * 16, cache.shape[1], cache.shape[3])[:length]


def snake(x: torch.Tensor, alpha: torch.Tensor) -> torch.Tensor:
    """fp32 Snake activation over the last (channel) axis: x + sin(a x)^2 / (a + 1e-9)."""
    xf, a = x.float(), alpha.float()
    return xf + torch.sin(a * xf).pow(2) / (a + 1e-9)


def act_im2col(x: torch.Tensor, k: int, stride: int = 1, pad: int = 0, pad_right: int | None = None, dil: int = 1,
               act: str | None = None, alpha=None, reflect: bool = False) -> torch.Tensor:
    """fp32 channels-last im2col of x [B, T, C] with the activation applied
    first (None, "snake" with ``alpha``, "elu", "gelu"): [B * T_out, round_up(k * C, 8)],
    column j * C + c of row (b, t) = act(x)[b, t * stride - pad + j * dil, c];
    outside the signal zero, or the reflected sample when ``reflect``; zero
    padding columns."""
    B, T, C = x.shape
    pr = pad if pad_right is None else pad_right
    acts = {"snake": lambda t: snake(t, alpha), "elu": torch.nn.functional.elu, "gelu": torch.nn.functional.gelu}
    xs = acts[act](x.float()) if act is not None else x.float()
    if reflect:
        xp = torch.nn.functional.pad(xs.transpose(1, 2), (pad, pr), mode="reflect").transpose(1, 2)
    else:
        xp = torch.nn.functional.pad(xs, (0, 0, pad, pr))
    T_out = (T + pad + pr - dil * (k - 1) - 1) // stride + 1
    t = torch.arange(T_out, device=x.device)[:, None] * stride + torch.arange(k, device=x.device)[None, :] * dil
    cols = xp[:, t].reshape(B * T_out, k * C)        # [B, T_out, k, C] -> rows
    kp = (k * C + 7) // 8 * 8
    return cols if kp == k * C else torch.nn.functional.pad(cols, (0, kp - k * C))


def convt_fold(Y: torch.Tensor, bias, c_out: int, stride: int, pad: int, pad_right: int | None = None) -> torch.Tensor:
    """fp32 overlap-add of a transposed convolution computed as a GEMM: Y [B,
    T_in, k * C_out] (column j * C_out + o = tap j of output o) -> the full
    output [B, (T_in - 1) * stride + k, C_out] (+ bias) with ``pad`` samples cut
    on the left and ``pad_right`` (default ``pad``) on the right."""
    B, T_in, kc = Y.shape
    k = kc // c_out
    pr = pad if pad_right is None else pad_right
    full = torch.zeros(B, (T_in - 1) * stride + k, c_out, dtype=torch.float32, device=Y.device)
    Yr = Y.float().reshape(B, T_in, k, c_out)
    for j in range(k):
        full[:, j:j + (T_in - 1) * stride + 1:stride] += Yr[:, :, j]
    out = full[:, pad:full.shape[1] - pr]
    return out + bias.float() if bias is not None else out


def lstm_cell(G: torch.Tensor, c: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 LSTM step from gate pre-activations G [B, 4H] (order i, f, g, o)
    -> (h, c)."""
    i, f, g, o = G.float().chunk(4, -1)
    c = torch.sigmoid(f) * c + torch.sigmoid(i) * torch.tanh(g)
    return torch.sigmoid(o) * torch.tanh(c), c


def instance_norm(x: torch.Tensor, gamma=None, beta=None, active: int = 0, eps: float = 1e-5) -> torch.Tensor:
    """fp32 instance norm over the last axis with statistics of the first ``active`` steps."""
    xf = x.float()
    a = active if 0 < active <= x.shape[-1] else x.shape[-1]
    mean = xf[..., :a].mean(-1, keepdim=True)
    var = xf[..., :a].var(-1, unbiased=False, keepdim=True)
    y = (xf - mean) * torch.rsqrt(var + eps)
    if gamma is not None:
        y = y * gamma.float()[None, :, None]
    if beta is not None:
        y = y + beta.float()[None, :, None]
    return y
