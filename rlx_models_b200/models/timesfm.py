"""TimesFM: a decoder-only foundation model for time-series forecasting.

    input    context right-aligned to ``context_length`` (front zero padding marked
             in a padding mask) and cut into patches of 32; each series is scaled by
             the mean / std of its first patch with at least 3 observed values
    tokens   residual MLP([patch ; patch padding]) -> hidden, + frequency embedding
             (+ sinusoidal positions shifted to the first observed patch, optional)
    layers   x += attn(RMSNorm(x)) (causal, padded patches masked as keys; queries
             scaled per dimension by softplus(w) / sqrt(d) * 1 / ln 2) then
             x += FFN(LayerNorm(x)) with padded patches' FFN outputs zeroed
    output   residual MLP -> horizon_length x (mean + quantiles) per patch, rescaled;
             the last patch's forecast is appended to the context and the model runs
             again until the horizon is covered; optional trend / residual
             decomposition by a moving average (two series per input, outputs summed)

Linear layers run on the package's tcgen05 GEMM in bf16 on the GPU (fp32 on
CPU); attention is torch SDPA with the causal + padding mask.

Checkpoint names: transformers' TimesFmModelForPrediction.

Reference: crates/rlx-timesfm3 (TimesFM forecasting); transformers'
TimesFmModelForPrediction is the CPU oracle.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from .flux_text import _linear


@dataclass
class TimesFmConfig:
    patch_length: int = 32
    context_length: int = 512
    horizon_length: int = 128
    freq_size: int = 3
    num_hidden_layers: int = 50
    hidden_size: int = 1280
    intermediate_size: int = 1280
    head_dim: int = 80
    num_attention_heads: int = 16
    tolerance: float = 1e-6
    rms_norm_eps: float = 1e-6
    quantiles: list = field(default_factory=lambda: [0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9])
    pad_val: float = 1123581321.0
    use_positional_embedding: bool = False
    min_timescale: float = 1
    max_timescale: float = 10000

    @classmethod
    def from_dict(cls, d: dict) -> "TimesFmConfig":
        names = set(cls.__dataclass_fields__)
        return cls(**{k: v for k, v in d.items() if k in names and v is not None})


class TimesFm:
    def __init__(self, cfg: TimesFmConfig, weights, device="cpu"):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dt = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])
        dev, dt = self.device, self.dt
        lw = lambda n: get(n).to(dev, dt).contiguous()  # noqa: E731
        f32 = lambda n: get(n).to(dev, torch.float32).contiguous()  # noqa: E731

        def block(p):
            return dict(i=(lw(p + "input_layer.weight"), lw(p + "input_layer.bias")),
                        o=(lw(p + "output_layer.weight"), lw(p + "output_layer.bias")),
                        r=(lw(p + "residual_layer.weight"), lw(p + "residual_layer.bias")))

        d = "decoder."
        self.inp = block(d + "input_ff_layer.")
        self.freq = f32(d + "freq_emb.weight")
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            p = f"{d}layers.{i}."
            qkv_w = torch.cat([get(p + f"self_attn.{n}_proj.weight") for n in "qkv"]).to(dev, dt).contiguous()
            qkv_b = torch.cat([get(p + f"self_attn.{n}_proj.bias") for n in "qkv"]).to(dev, dt).contiguous()
            self.layers.append(dict(
                qkv=(qkv_w, qkv_b), o=(lw(p + "self_attn.o_proj.weight"), lw(p + "self_attn.o_proj.bias")),
                qscale=F.softplus(f32(p + "self_attn.scaling")) * (1.442695041 / math.sqrt(cfg.head_dim)),
                rms=f32(p + "input_layernorm.weight"),
                ln=(f32(p + "mlp.layer_norm.weight"), f32(p + "mlp.layer_norm.bias")),
                up=(lw(p + "mlp.gate_proj.weight"), lw(p + "mlp.gate_proj.bias")),
                down=(lw(p + "mlp.down_proj.weight"), lw(p + "mlp.down_proj.bias"))))
        self.head = block("horizon_ff_layer.")
        n = cfg.hidden_size // 2
        inc = math.log(float(cfg.max_timescale) / float(cfg.min_timescale)) / max(n - 1, 1)
        self.inv_timescales = cfg.min_timescale * torch.exp(torch.arange(n, dtype=torch.float32, device=dev) * -inc)

    # -- pieces ------------------------------------------------------------
    def _lin(self, x, wb):
        shp = x.shape
        return _linear(x.reshape(-1, shp[-1]).to(self.dt).contiguous(), *wb).float().view(*shp[:-1], -1)

    def _res_block(self, x, B):
        return self._lin(F.silu(self._lin(x, B["i"])), B["o"]) + self._lin(x, B["r"])

    def _stats(self, x, pad):
        """Mean / std of each series' first patch with >= 3 observed values (else the last patch)."""
        n_obs = (1 - pad).sum(2)
        ok = n_obs >= 3
        idx = torch.where(ok.any(1), ok.int().argmax(1), torch.full_like(ok[:, 0], x.shape[1] - 1, dtype=torch.long))
        b = torch.arange(x.shape[0], device=x.device)
        arr, m = x[b, idx], 1 - pad[b, idx]
        n = m.sum(1).clamp(min=1.0)
        mu = (arr * m).sum(1) / n
        var = (((arr - mu[:, None]) * m) ** 2).sum(1) / n
        return mu, var.clamp(min=0.0).sqrt()

    def _positions(self, pad_patch: torch.Tensor, N: int) -> torch.Tensor:
        """Sinusoidal positions rotated so position 0 lands on the first observed patch."""
        pos = torch.arange(N, dtype=torch.float32, device=self.device)[:, None] * self.inv_timescales[None]
        emb = torch.cat([torch.sin(pos), torch.cos(pos)], 1)
        emb = F.pad(emb, (0, self.cfg.hidden_size % 2))
        obs = pad_patch == 0
        first = torch.where(obs.any(1), obs.int().argmax(1), torch.full_like(obs[:, 0], -1, dtype=torch.long))
        idx = (torch.arange(N, device=self.device)[None] - first[:, None]) % N
        return emb[idx]

    @torch.no_grad()
    def forward_patches(self, values: torch.Tensor, padding: torch.Tensor, freq: torch.Tensor):
        """values / padding [B, L] (L a multiple of the patch), freq [B] ->
        (forecasts [B, N, horizon, 1 + quantiles] fp32, patch padding [B, N])."""
        c = self.cfg
        B = values.shape[0]
        x = values.to(self.device).float().view(B, -1, c.patch_length)
        pad = padding.to(self.device).float().view(B, -1, c.patch_length)
        x = torch.where((pad - 1.0).abs() < c.tolerance, torch.zeros_like(x), x)
        pad = torch.where((x - c.pad_val).abs() < c.tolerance, torch.ones_like(pad), pad)
        mu, sigma = self._stats(x, pad)
        sigma = sigma.clamp(min=c.tolerance)
        xn = (x - mu[:, None, None]) / sigma[:, None, None]
        xn = torch.where((x - c.pad_val).abs() < c.tolerance, torch.full_like(xn, c.pad_val), xn)
        xn = xn * (1.0 - pad)
        h = self._res_block(torch.cat([xn, pad], -1), self.inp)
        pp = pad.min(-1).values                                   # [B, N] padded patches
        N = h.shape[1]
        if c.use_positional_embedding:
            h = h + self._positions(pp, N)
        h = h + self.freq[freq.to(self.device).long().view(B)][:, None]
        # additive mask, as the released model applies it: a query whose keys are all padded
        # (front padding) attends uniformly instead of producing NaNs
        neg = torch.finfo(torch.float32).min
        causal = torch.triu(torch.full((N, N), neg, device=self.device), diagonal=1)
        mask = torch.minimum(pp[:, None, None, :] * neg, causal[None, None]).to(self.dt)
        nh, hd = c.num_attention_heads, c.head_dim
        for L in self.layers:
            y = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + c.rms_norm_eps) * L["rms"]
            q, k, v = self._lin(y, L["qkv"]).split(nh * hd, -1)
            q = q.view(B, N, nh, hd).transpose(1, 2) * L["qscale"]
            k = k.view(B, N, nh, hd).transpose(1, 2)
            v = v.view(B, N, nh, hd).transpose(1, 2)
            o = F.scaled_dot_product_attention(q.to(self.dt), k.to(self.dt), v.to(self.dt), attn_mask=mask,
                                               scale=1.0)
            h = h + self._lin(o.transpose(1, 2).reshape(B, N, nh * hd).float(), L["o"])
            g = F.relu(self._lin(F.layer_norm(h, (h.shape[-1],), *L["ln"], 1e-6), L["up"]))
            h = h + self._lin(g, L["down"]) * (1.0 - pp[:, :, None])
        out = self._res_block(h, self.head).view(B, N, c.horizon_length, len(c.quantiles) + 1)
        return out * sigma[:, None, None, None] + mu[:, None, None, None], pp

    # -- forecasting -------------------------------------------------------
    def _prepare(self, series: list, context_len: int):
        c = self.cfg
        vals, pads = [], []
        for ts in series:
            ts = torch.as_tensor(ts, dtype=torch.float32)
            n = ts.shape[0]
            pad = torch.zeros(n + c.horizon_length)
            if n < context_len:
                ts = torch.cat([torch.zeros(context_len - n), ts])
                pad = torch.cat([torch.ones(context_len - n), pad])
            elif n > context_len:
                ts = ts[-context_len:]
                pad = pad[-(context_len + c.horizon_length):]
            vals.append(ts)
            pads.append(pad)
        return torch.stack(vals), torch.stack(pads)

    @torch.no_grad()
    def forecast(self, series: list, freq: list | None = None, horizon: int | None = None,
                 window_size: int | None = None, context_len: int | None = None, truncate_negative: bool = False):
        """Series (1-D tensors / lists of past values) -> (mean [B, horizon],
        mean + quantiles [B, horizon, 1 + len(quantiles)])."""
        c = self.cfg
        ctx = c.context_length if context_len is None else context_len
        series = [torch.as_tensor(s, dtype=torch.float32)[-ctx:] for s in series]
        inp_min = min(float(s.min()) for s in series)
        freq = [0] * len(series) if freq is None else list(freq)
        if window_size is not None:
            parts, fr = [], []
            for s, f in zip(series, freq):
                sm = F.conv1d(F.pad(s, (window_size - 1, 0))[None, None],
                              torch.full((1, 1, window_size), 1.0 / window_size))[0, 0]
                parts += [sm, s - sm]
                fr += [f, f]
            series, freq = parts, fr
        horizon = c.horizon_length if horizon is None else horizon
        vals, pads = self._prepare(series, ctx)
        steps = (horizon + c.horizon_length - 1) // c.horizon_length
        pads = F.pad(pads, (0, steps * c.horizon_length))    # forecasts appended later are observed
        fr = torch.tensor(freq, dtype=torch.long)
        out_all, cur = [], vals
        for _ in range(steps):
            v = cur[:, -ctx:]
            p = pads[:, :cur.shape[1]][:, -ctx:]
            fc, _ = self.forward_patches(v, p, fr)
            out_all.append(fc[:, -1, :c.horizon_length].cpu())
            cur = torch.cat([cur, fc[:, -1, :c.horizon_length, 0].cpu()], 1)
        full = torch.cat(out_all, 1)[:, :horizon]
        if window_size is not None:
            full = full[0::2] + full[1::2]
        if inp_min >= 0 and truncate_negative:
            full = full.clamp(min=0.0)
        return full[..., 0], full
