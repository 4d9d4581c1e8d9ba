"""V-JEPA 2 video encoder (Meta's self-supervised video model) and its
attentive-probe video classifier.

    patches  tubelets of 2 frames x 16 x 16 pixels (a strided 3-D conv, run here as
             one GEMM over the flattened tubelets) -> tokens in (frame, row, column) order
    blocks   x += proj(attn(LN(x))) with 3-D rotary positions: the head dimension is
             split in three equal even parts rotated by the token's frame, row and
             column index (a fixed 1/10000^(i / (d/2)) frequency table per part; the
             rest passes through); x += MLP(LN(x)); final LayerNorm
    probe    3 self-attention blocks over the tokens, then one cross-attention block
             from a learned query (queries un-normalised, keys / values LayerNormed) ->
             linear classifier

The token grid of the rotary positions is the configured crop (as the released
model computes it). Linear layers run on the package's tcgen05 GEMM in bf16 on
the GPU; attention is torch SDPA.

Checkpoint names: transformers' VJEPA2Model / VJEPA2ForVideoClassification.

Reference: crates/rlx-vjepa2 (V-JEPA 2 video embeddings / classification);
transformers' VJEPA2 modules are the CPU oracle.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .flux_text import _linear


@dataclass
class VJEPA2Config:
    patch_size: int = 16
    crop_size: int = 256
    frames_per_clip: int = 64
    tubelet_size: int = 2
    hidden_size: int = 1024
    in_chans: int = 3
    num_attention_heads: int = 16
    num_hidden_layers: int = 24
    mlp_ratio: float = 4.0
    layer_norm_eps: float = 1e-6
    qkv_bias: bool = True
    hidden_act: str = "gelu"
    num_pooler_layers: int = 3

    @classmethod
    def from_dict(cls, d: dict) -> "VJEPA2Config":
        names = set(cls.__dataclass_fields__)
        return cls(**{k: v for k, v in d.items() if k in names and v is not None})


def _rotate(x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    """The released model's rotation of x [..., N, d] by positions pos [N]: a
    [sin | sin] / [cos | cos] table over d/2 frequencies applied to
    interleaved-pair rotated features."""
    d = x.shape[-1]
    omega = 1.0 / 10000 ** (torch.arange(d // 2, dtype=torch.float32, device=x.device) / (d / 2.0))
    f = pos.float()[:, None] * omega[None]
    sin, cos = f.sin().repeat(1, 2), f.cos().repeat(1, 2)
    y = x.unflatten(-1, (-1, 2))
    y = torch.stack((-y[..., 1], y[..., 0]), -1).flatten(-2)
    return x * cos + y * sin


class VJEPA2:
    def __init__(self, cfg: VJEPA2Config, weights, device="cpu"):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dt = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])
        names = set(weights.keys())
        pre = "vjepa2." if any(k.startswith("vjepa2.") for k in names) else ""
        dev, dt = self.device, self.dt
        lw = lambda n: get(n).to(dev, dt).contiguous()  # noqa: E731
        f32 = lambda n: get(n).to(dev, torch.float32).contiguous()  # noqa: E731
        e = pre + "encoder."
        pw = get(e + "embeddings.patch_embeddings.proj.weight")              # [H, C, t, p, p]
        self.patch_w = pw.reshape(pw.shape[0], -1).to(dev, dt).contiguous()
        self.patch_b = lw(e + "embeddings.patch_embeddings.proj.bias")
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            p = f"{e}layer.{i}."
            qkv_w = torch.cat([get(p + f"attention.{n}.weight") for n in ("query", "key", "value")])
            qkv_b = torch.cat([get(p + f"attention.{n}.bias") for n in ("query", "key", "value")]) \
                if cfg.qkv_bias else None
            self.layers.append(dict(
                ln1=(f32(p + "norm1.weight"), f32(p + "norm1.bias")), ln2=(f32(p + "norm2.weight"), f32(p + "norm2.bias")),
                qkv=(qkv_w.to(dev, dt).contiguous(), None if qkv_b is None else qkv_b.to(dev, dt).contiguous()),
                proj=(lw(p + "attention.proj.weight"), lw(p + "attention.proj.bias")),
                fc1=(lw(p + "mlp.fc1.weight"), lw(p + "mlp.fc1.bias")), fc2=(lw(p + "mlp.fc2.weight"), lw(p + "mlp.fc2.bias"))))
        self.ln = (f32(e + "layernorm.weight"), f32(e + "layernorm.bias"))
        self.pooler = None
        if "pooler.query_tokens" in names:
            def attn(p):
                return {n: (lw(p + f"{n}.weight"), lw(p + f"{n}.bias")) for n in ("q_proj", "k_proj", "v_proj", "out_proj")
                        if p + f"{n}.weight" in names}

            def block(p, a):
                return dict(ln1=(f32(p + "layer_norm1.weight"), f32(p + "layer_norm1.bias")), attn=attn(p + a),
                            ln2=(f32(p + "layer_norm2.weight"), f32(p + "layer_norm2.bias")),
                            fc1=(lw(p + "mlp.fc1.weight"), lw(p + "mlp.fc1.bias")),
                            fc2=(lw(p + "mlp.fc2.weight"), lw(p + "mlp.fc2.bias")))
            self.pooler = dict(query=f32("pooler.query_tokens"),
                               self_layers=[block(f"pooler.self_attention_layers.{i}.", "self_attn.")
                                            for i in range(cfg.num_pooler_layers)],
                               cross=block("pooler.cross_attention_layer.", "cross_attn."))
            self.classifier = (lw("classifier.weight"), lw("classifier.bias")) if "classifier.weight" in names else None

    # -- pieces ------------------------------------------------------------
    def _lin(self, x, wb):
        shp = x.shape
        return _linear(x.reshape(-1, shp[-1]).to(self.dt).contiguous(), *wb).float().view(*shp[:-1], -1)

    def _ln(self, x, wb):
        return F.layer_norm(x, (x.shape[-1],), wb[0], wb[1], self.cfg.layer_norm_eps)

    def _mlp(self, x, L):
        return self._lin(F.gelu(self._lin(x, L["fc1"])), L["fc2"])

    def _positions(self, N: int):
        c = self.cfg
        g = c.crop_size // c.patch_size
        ids = torch.arange(N, device=self.device)
        per_frame = g * g
        f = ids // per_frame
        r = (ids - per_frame * f) // g
        w = ids - per_frame * f - g * r
        return f, r, w

    def _rope3d(self, x, pos):
        hd = x.shape[-1]
        part = 2 * ((hd // 3) // 2)
        out, s = [], 0
        for p in pos:
            out.append(_rotate(x[..., s:s + part], p))
            s += part
        if s < hd:
            out.append(x[..., s:])
        return torch.cat(out, -1)

    # -- encoder -----------------------------------------------------------
    @torch.no_grad()
    def features(self, video: torch.Tensor) -> torch.Tensor:
        """video [B, T, C, H, W] (preprocessed frames) -> tokens [B, T/2 * (H/16) * (W/16), hidden] fp32."""
        c = self.cfg
        x = video.to(self.device, torch.float32).permute(0, 2, 1, 3, 4)          # [B, C, T, H, W]
        if x.shape[2] < c.tubelet_size:
            x = x.repeat(1, 1, c.tubelet_size, 1, 1)
        B, C, T, H, W = x.shape
        t, p = c.tubelet_size, c.patch_size
        tub = x.view(B, C, T // t, t, H // p, p, W // p, p).permute(0, 2, 4, 6, 1, 3, 5, 7)
        rows = tub.reshape(B * (T // t) * (H // p) * (W // p), C * t * p * p)
        h = _linear(rows.to(self.dt).contiguous(), self.patch_w, self.patch_b).float().view(B, -1, c.hidden_size)
        N = h.shape[1]
        pos = self._positions(N)
        nh = c.num_attention_heads
        hd = c.hidden_size // nh
        for L in self.layers:
            y = self._ln(h, L["ln1"])
            q, k, v = self._lin(y, L["qkv"]).view(B, N, 3, nh, hd).permute(2, 0, 3, 1, 4)
            q, k = self._rope3d(q, pos), self._rope3d(k, pos)
            o = F.scaled_dot_product_attention(q.to(self.dt), k.to(self.dt), v.to(self.dt))
            h = h + self._lin(o.transpose(1, 2).reshape(B, N, -1).float(), L["proj"])
            h = h + self._mlp(self._ln(h, L["ln2"]), L)
        return self._ln(h, self.ln)

    # -- attentive probe ---------------------------------------------------
    def _mha(self, a, q_in, kv_in):
        nh = self.cfg.num_attention_heads
        B, Tq, D = q_in.shape
        Tk = kv_in.shape[1]
        sh = lambda x, T: x.view(B, T, nh, D // nh).transpose(1, 2).to(self.dt)  # noqa: E731
        o = F.scaled_dot_product_attention(sh(self._lin(q_in, a["q_proj"]), Tq), sh(self._lin(kv_in, a["k_proj"]), Tk),
                                           sh(self._lin(kv_in, a["v_proj"]), Tk))
        o = o.transpose(1, 2).reshape(B, Tq, D).float()
        return self._lin(o, a["out_proj"]) if "out_proj" in a else o

    @torch.no_grad()
    def pooled(self, video: torch.Tensor) -> torch.Tensor:
        """Attentive-probe embedding [B, hidden] (classification checkpoints)."""
        if self.pooler is None:
            raise ValueError("checkpoint has no attentive pooler")
        P = self.pooler
        h = self.features(video)
        for L in P["self_layers"]:
            y = self._ln(h, L["ln1"])
            h = h + self._mha(L["attn"], y, y)
            h = h + self._mlp(self._ln(h, L["ln2"]), L)
        L = P["cross"]
        q = P["query"].expand(h.shape[0], -1, -1)
        x = q + self._mha(L["attn"], q, self._ln(h, L["ln1"]))
        x = x + self._mlp(self._ln(x, L["ln2"]), L)
        return x[:, 0]

    @torch.no_grad()
    def classify(self, video: torch.Tensor) -> torch.Tensor:
        """Video-classification logits [B, labels]."""
        return self._lin(self.pooled(video), self.classifier)
