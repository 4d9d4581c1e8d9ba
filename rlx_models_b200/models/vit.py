"""Vision transformers for image embeddings: the CLIP and SigLIP vision towers
(HF ``vision_model.*`` names, standalone or inside the full CLIP / SigLIP
checkpoints) and the DINOv2 / DINOv3 self-supervised backbones
(``Dinov2Encoder``, ``Dinov3Encoder``).

    patches  = patchify(pixels) @ W_patch^T (+ bias)      (the stride-p conv as a GEMM)
    tokens   = [CLS] + patches (CLIP) | patches (SigLIP), + position embeddings
    CLIP     : pre-LayerNorm, pre-norm blocks (quick-GELU MLP), pooled = LN(token 0),
               image embedding = visual_projection(pooled)
    SigLIP   : pre-norm blocks (GELU-tanh MLP), post-LayerNorm, pooled by the
               attention-pooling head (a learned probe attends over the tokens,
               then LayerNorm + MLP with a residual)

Runs on the package's GEMM (``_linear``: bf16 on CUDA) or in fp32 on CPU;
attention is non-causal SDPA. Images go through ``utils/preprocess.py``.

Reference: crates/rlx-vision (NomicVision encoder graphs) and the vision
towers of the reference's VLM families; transformers CLIP / SigLIP vision
models are the CPU oracles.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .flux_text import _linear


def _pad_k(w: torch.Tensor) -> torch.Tensor:
    """Zero-pad a patch-embedding weight's input dim to a multiple of 8 (the GEMM's
    16-byte row rule; a 14-pixel patch has 3 * 14 * 14 = 588 inputs)."""
    k = w.shape[1]
    return w if k % 8 == 0 else F.pad(w, (0, 8 - k % 8))


def _patch_rows(pixels: torch.Tensor, patch: int, k_padded: int, dtype) -> torch.Tensor:
    from ..utils.preprocess import patchify
    rows = torch.stack([patchify(p, patch) for p in pixels]).to(dtype)
    return rows if rows.shape[-1] == k_padded else F.pad(rows, (0, k_padded - rows.shape[-1]))


@dataclass
class VisionConfig:
    family: str = "clip"  # "clip" | "siglip"
    hidden_size: int = 768
    intermediate_size: int = 3072
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    image_size: int = 224
    patch_size: int = 32
    layer_norm_eps: float = 1e-5
    projection_dim: int = 0

    @classmethod
    def from_dict(cls, d: dict) -> "VisionConfig":
        mt = d.get("model_type", "clip_vision_model")
        vc = d.get("vision_config") or d
        fam = "siglip" if "siglip" in mt else "clip"
        kw = {k: vc[k] for k in cls.__dataclass_fields__ if k in vc and k != "family"}
        kw["projection_dim"] = d.get("projection_dim", vc.get("projection_dim", 0)) if fam == "clip" else 0
        return cls(family=fam, **kw)


class VisionEncoder:
    def __init__(self, cfg: VisionConfig, weights, device="cpu", dtype: torch.dtype | None = None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype or (torch.bfloat16 if self.device.type == "cuda" else torch.float32)
        get = (lambda n: weights.take(n)) if hasattr(weights, "take") else (lambda n: weights[n])
        has = lambda n: n in weights  # noqa: E731
        dv = lambda t: t.to(self.device, self.dtype).contiguous()  # noqa: E731
        v = "vision_model."
        e = v + "embeddings."
        H = cfg.hidden_size
        self.w_patch = _pad_k(dv(get(e + "patch_embedding.weight").reshape(H, -1)))
        self.b_patch = dv(get(e + "patch_embedding.bias")) if has(e + "patch_embedding.bias") else None
        self.cls = dv(get(e + "class_embedding")) if has(e + "class_embedding") else None
        self.pos = dv(get(e + "position_embedding.weight"))
        ln = lambda p: (dv(get(p + ".weight")), dv(get(p + ".bias")))  # noqa: E731
        self.pre_ln = ln(v + "pre_layrnorm") if has(v + "pre_layrnorm.weight") else None
        self.post_ln = ln(v + "post_layernorm")
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            p = v + f"encoder.layers.{i}."
            a = p + "self_attn."
            self.layers.append(dict(
                ln1=ln(p + "layer_norm1"), ln2=ln(p + "layer_norm2"),
                qkv=dv(torch.cat([get(a + f"{n}_proj.weight") for n in "qkv"], 0)),
                qkv_b=dv(torch.cat([get(a + f"{n}_proj.bias") for n in "qkv"], 0)),
                o=(dv(get(a + "out_proj.weight")), dv(get(a + "out_proj.bias"))),
                fc1=(dv(get(p + "mlp.fc1.weight")), dv(get(p + "mlp.fc1.bias"))),
                fc2=(dv(get(p + "mlp.fc2.weight")), dv(get(p + "mlp.fc2.bias")))))
        self.proj = dv(get("visual_projection.weight")) if has("visual_projection.weight") else None
        self.head = None
        h = v + "head."
        if has(h + "probe"):
            self.head = dict(probe=dv(get(h + "probe")), in_w=dv(get(h + "attention.in_proj_weight")),
                             in_b=dv(get(h + "attention.in_proj_bias")),
                             o=(dv(get(h + "attention.out_proj.weight")), dv(get(h + "attention.out_proj.bias"))),
                             ln=ln(h + "layernorm"), fc1=(dv(get(h + "mlp.fc1.weight")), dv(get(h + "mlp.fc1.bias"))),
                             fc2=(dv(get(h + "mlp.fc2.weight")), dv(get(h + "mlp.fc2.bias"))))

    def _ln(self, x, p):
        return F.layer_norm(x.float(), (x.shape[-1],), p[0].float(), p[1].float(),
                            self.cfg.layer_norm_eps).to(x.dtype)

    def _act(self, x):
        x = x.float()
        return x * torch.sigmoid(1.702 * x) if self.cfg.family == "clip" else F.gelu(x, approximate="tanh")

    def _attend(self, q, k, v, nh):
        B, Lq, H = q.shape
        D = H // nh
        q, k, v = (t.reshape(B, -1, nh, D).transpose(1, 2) for t in (q, k, v))
        return F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B, Lq, H)

    def _blocks(self, pixels: torch.Tensor, n_blocks: int) -> torch.Tensor:
        c = self.cfg
        pixels = pixels.to(self.device, torch.float32)
        B = pixels.shape[0]
        H, nh = c.hidden_size, c.num_attention_heads
        x = _linear(_patch_rows(pixels, c.patch_size, self.w_patch.shape[1], self.dtype), self.w_patch, self.b_patch)
        if self.cls is not None:
            x = torch.cat([self.cls.expand(B, 1, H), x], 1)
        x = x + self.pos[None, :x.shape[1]]
        if self.pre_ln is not None:
            x = self._ln(x, self.pre_ln)
        for ly in self.layers[:n_blocks]:
            q, k, v = _linear(self._ln(x, ly["ln1"]), ly["qkv"], ly["qkv_b"]).split(H, -1)
            x = x + _linear(self._attend(q, k, v, nh), *ly["o"])
            x = x + _linear(self._act(_linear(self._ln(x, ly["ln2"]), *ly["fc1"])).to(x.dtype), *ly["fc2"])
        return x

    @torch.no_grad()
    def hidden_at(self, pixels: torch.Tensor, layer: int) -> torch.Tensor:
        """Hidden states after ``layer`` blocks (HF ``hidden_states[layer]``; negative
        counts from the end: -1 = the last block's output, before any post-norm)."""
        n = len(self.layers)
        k = layer if layer >= 0 else n + 1 + layer
        if not 0 <= k <= n:
            raise ValueError(f"layer {layer} outside 0..{n}")
        return self._blocks(pixels, k)

    @torch.no_grad()
    def __call__(self, pixels: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """pixels [B, 3, S, S] (preprocessed) -> (last hidden [B, L, H], pooled [B, H])."""
        c = self.cfg
        H, nh = c.hidden_size, c.num_attention_heads
        x = self._blocks(pixels, len(self.layers))
        B = x.shape[0]
        if c.family == "clip":
            return x, self._ln(x[:, 0], self.post_ln)
        x = self._ln(x, self.post_ln)
        if self.head is None:
            return x, x.mean(1)
        hd = self.head
        wq, wk, wv = hd["in_w"].split(H, 0)
        bq, bk, bv = hd["in_b"].split(H, 0)
        probe = hd["probe"].expand(B, 1, H)
        h = _linear(self._attend(_linear(probe, wq, bq), _linear(x, wk, bk), _linear(x, wv, bv), nh), *hd["o"])
        h = h + _linear(self._act(_linear(self._ln(h, hd["ln"]), *hd["fc1"])).to(h.dtype), *hd["fc2"])
        return x, h[:, 0]

    def embed(self, pixels: torch.Tensor, normalize: bool = True) -> torch.Tensor:
        """[B, D] fp32 image embeddings: CLIP's projected pooled token (when the
        checkpoint has visual_projection), otherwise the pooled output."""
        _, pooled = self(pixels)
        e = _linear(pooled, self.proj).float() if self.proj is not None else pooled.float()
        return F.normalize(e, dim=-1) if normalize else e


# ---------------------------------------------------------------------------
# DINOv2 (with or without register tokens)
# ---------------------------------------------------------------------------

@dataclass
class Dinov2Config:
    hidden_size: int = 768
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    mlp_ratio: float = 4.0
    image_size: int = 518
    patch_size: int = 14
    layer_norm_eps: float = 1e-6
    use_swiglu_ffn: bool = False
    num_register_tokens: int = 0
    hidden_act: str = "gelu"
    # the with-registers release resizes position grids with the antialiased bicubic
    # filter (a = -0.5), the original one with plain bicubic (a = -0.75)
    antialias: bool = False

    @classmethod
    def from_dict(cls, d: dict) -> "Dinov2Config":
        kw = {k: d[k] for k in cls.__dataclass_fields__ if k in d}
        kw.setdefault("antialias", d.get("model_type") == "dinov2_with_registers")
        return cls(**kw)


class Dinov2Encoder:
    """DINOv2 ViT: [CLS] + register tokens + patch tokens, position embeddings
    on CLS and patches (bicubically resized to the image's patch grid when it
    differs from the pretraining grid), pre-norm blocks with learned per-channel
    layer scales on both residual branches (GELU MLP, or SwiGLU for the giant
    variants), final LayerNorm; pooled output = the normalised CLS token.
    Checkpoint names: ``embeddings.*``, ``encoder.layer.{i}.*``, ``layernorm.*``
    (an optional ``dinov2.`` prefix is accepted).

    Reference: the reference's vision crates (crates/rlx-dinov2); the
    transformers Dinov2Model / Dinov2WithRegistersModel are the CPU oracles."""

    def __init__(self, cfg: Dinov2Config, weights, device="cpu", dtype: torch.dtype | None = None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype or (torch.bfloat16 if self.device.type == "cuda" else torch.float32)
        names = list(weights.keys()) if hasattr(weights, "keys") else list(weights)
        pre = "dinov2." if any(n.startswith("dinov2.") for n in names) else ""
        get = (lambda n: weights.take(pre + n)) if hasattr(weights, "take") else (lambda n: weights[pre + n])
        has = lambda n: (pre + n) in weights  # noqa: E731
        dv = lambda t: t.to(self.device, self.dtype).contiguous()  # noqa: E731
        ln = lambda p: (dv(get(p + ".weight")), dv(get(p + ".bias")))  # noqa: E731
        lin = lambda p: (dv(get(p + ".weight")), dv(get(p + ".bias")))  # noqa: E731
        H = cfg.hidden_size
        e = "embeddings."
        self.w_patch = _pad_k(dv(get(e + "patch_embeddings.projection.weight").reshape(H, -1)))
        self.b_patch = dv(get(e + "patch_embeddings.projection.bias"))
        self.cls = dv(get(e + "cls_token").reshape(1, 1, H))
        self.regs = dv(get(e + "register_tokens")) if has(e + "register_tokens") else None
        self.pos = get(e + "position_embeddings").float().to(self.device)  # [1, 1 + g*g, H], resized per image grid
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            p = f"encoder.layer.{i}."
            a = p + "attention."
            mlp = dict(w_in=lin(p + "mlp.weights_in"), w_out=lin(p + "mlp.weights_out")) if cfg.use_swiglu_ffn \
                else dict(fc1=lin(p + "mlp.fc1"), fc2=lin(p + "mlp.fc2"))
            self.layers.append(dict(
                ln1=ln(p + "norm1"), ln2=ln(p + "norm2"),
                qkv=dv(torch.cat([get(a + f"attention.{n}.weight") for n in ("query", "key", "value")], 0)),
                qkv_b=dv(torch.cat([get(a + f"attention.{n}.bias") for n in ("query", "key", "value")], 0)),
                o=lin(a + "output.dense"),
                ls1=dv(get(p + "layer_scale1.lambda1")), ls2=dv(get(p + "layer_scale2.lambda1")), **mlp))
        self.norm = ln("layernorm")

    def _ln(self, x, p):
        return F.layer_norm(x.float(), (x.shape[-1],), p[0].float(), p[1].float(),
                            self.cfg.layer_norm_eps).to(x.dtype)

    def _pos(self, gh: int, gw: int) -> torch.Tensor:
        n = self.pos.shape[1] - 1
        if gh * gw == n and gh == gw:
            return self.pos
        g = int(round(n ** 0.5))
        H = self.pos.shape[-1]
        grid = self.pos[:, 1:].reshape(1, g, g, H).permute(0, 3, 1, 2)
        grid = F.interpolate(grid, size=(gh, gw), mode="bicubic", align_corners=False, antialias=self.cfg.antialias)
        return torch.cat([self.pos[:, :1], grid.permute(0, 2, 3, 1).reshape(1, gh * gw, H)], 1)

    def _mlp(self, x, ly):
        if "w_in" in ly:
            a, b = _linear(x, *ly["w_in"]).float().chunk(2, -1)
            return _linear((F.silu(a) * b).to(x.dtype), *ly["w_out"])
        h = _linear(x, *ly["fc1"]).float()
        h = F.gelu(h, approximate="tanh" if self.cfg.hidden_act == "gelu_pytorch_tanh" else "none")
        return _linear(h.to(x.dtype), *ly["fc2"])

    @torch.no_grad()
    def __call__(self, pixels: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """pixels [B, 3, h, w] (preprocessed; h, w multiples of the patch size) ->
        (last hidden [B, 1 + registers + patches, H], pooled CLS [B, H])."""
        c = self.cfg
        pixels = pixels.to(self.device, torch.float32)
        B, _, h, w = pixels.shape
        H, nh = c.hidden_size, c.num_attention_heads
        gh, gw = h // c.patch_size, w // c.patch_size
        x = _linear(_patch_rows(pixels, c.patch_size, self.w_patch.shape[1], self.dtype), self.w_patch, self.b_patch)
        x = torch.cat([self.cls.expand(B, 1, H), x], 1)
        x = (x.float() + self._pos(gh, gw)).to(self.dtype)
        if self.regs is not None:
            x = torch.cat([x[:, :1], self.regs.expand(B, -1, H), x[:, 1:]], 1)
        for ly in self.layers:
            q, k, v = _linear(self._ln(x, ly["ln1"]), ly["qkv"], ly["qkv_b"]).split(H, -1)
            D = H // nh
            q, k, v = (t.reshape(B, -1, nh, D).transpose(1, 2) for t in (q, k, v))
            att = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B, -1, H)
            x = x + _linear(att, *ly["o"]) * ly["ls1"]
            x = x + self._mlp(self._ln(x, ly["ln2"]), ly) * ly["ls2"]
        x = self._ln(x, self.norm)
        return x, x[:, 0]

    def embed(self, pixels: torch.Tensor, normalize: bool = True) -> torch.Tensor:
        """[B, H] fp32 image embeddings (the normalised CLS token)."""
        _, pooled = self(pixels)
        e = pooled.float()
        return F.normalize(e, dim=-1) if normalize else e


# ---------------------------------------------------------------------------
# DINOv3 (2-D axial RoPE on the patch tokens, register tokens, LayerScale)
# ---------------------------------------------------------------------------

@dataclass
class Dinov3Config:
    hidden_size: int = 384
    intermediate_size: int = 1536
    num_hidden_layers: int = 12
    num_attention_heads: int = 6
    patch_size: int = 16
    image_size: int = 224
    layer_norm_eps: float = 1e-5
    rope_theta: float = 100.0
    num_register_tokens: int = 0
    use_gated_mlp: bool = False
    hidden_act: str = "gelu"

    @classmethod
    def from_dict(cls, d: dict) -> "Dinov3Config":
        return cls(**{k: d[k] for k in cls.__dataclass_fields__ if k in d})


class Dinov3Encoder:
    """DINOv3 ViT: [CLS] + register tokens + patch tokens (no absolute position
    embedding); in every block, q and k of the patch tokens are rotated by a 2-D
    axial RoPE whose angles are 2 pi * (patch-centre coordinate in [-1, 1]) *
    theta^(-4j / head_dim), the y frequencies then the x frequencies, repeated
    for the two halves of the head (half-split rotation); pre-norm blocks with
    LayerScale on both branches (GELU MLP, or a gated one), final LayerNorm,
    CLS pooling. Checkpoint names: ``embeddings.*``, ``model.layer.{i}.*``
    (or ``layer.{i}.*``), ``norm.*``.

    Reference: crates/rlx-dinov3; transformers' DINOv3ViTModel is the CPU oracle."""

    def __init__(self, cfg: Dinov3Config, weights, device="cpu", dtype: torch.dtype | None = None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype or (torch.bfloat16 if self.device.type == "cuda" else torch.float32)
        get = (lambda n: weights.take(n)) if hasattr(weights, "take") else (lambda n: weights[n])
        has = lambda n: n in weights  # noqa: E731
        dv = lambda t: t.to(self.device, self.dtype).contiguous()  # noqa: E731
        H = cfg.hidden_size
        e = "embeddings."
        self.w_patch = _pad_k(dv(get(e + "patch_embeddings.weight").reshape(H, -1)))
        self.b_patch = dv(get(e + "patch_embeddings.bias"))
        self.cls = dv(get(e + "cls_token").reshape(1, 1, H))
        self.regs = dv(get(e + "register_tokens")) if has(e + "register_tokens") and cfg.num_register_tokens else None
        lp = "model.layer." if has("model.layer.0.norm1.weight") else "layer."
        ln = lambda p: (dv(get(p + ".weight")), dv(get(p + ".bias")))  # noqa: E731
        opt = lambda n: dv(get(n)) if has(n) else None  # noqa: E731
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            p = lp + f"{i}."
            a = p + "attention."
            zero = torch.zeros(H)
            qkv_b = torch.cat([get(a + f"{n}_proj.bias") if has(a + f"{n}_proj.bias") else zero for n in "qkv"])
            mlp = {n: (dv(get(p + f"mlp.{n}_proj.weight")), opt(p + f"mlp.{n}_proj.bias"))
                   for n in (("gate", "up", "down") if cfg.use_gated_mlp else ("up", "down"))}
            self.layers.append(dict(
                ln1=ln(p + "norm1"), ln2=ln(p + "norm2"),
                qkv=dv(torch.cat([get(a + f"{n}_proj.weight") for n in "qkv"], 0)), qkv_b=dv(qkv_b),
                o=(dv(get(a + "o_proj.weight")), opt(a + "o_proj.bias")),
                ls1=dv(get(p + "layer_scale1.lambda1")), ls2=dv(get(p + "layer_scale2.lambda1")), mlp=mlp))
        self.norm = ln("norm")
        D = H // cfg.num_attention_heads
        self.inv = 1.0 / cfg.rope_theta ** torch.arange(0, 1, 4 / D, dtype=torch.float32)  # [D / 4]

    def _ln(self, x, p):
        return F.layer_norm(x.float(), (x.shape[-1],), p[0].float(), p[1].float(),
                            self.cfg.layer_norm_eps).to(x.dtype)

    def _act(self, x):
        a = self.cfg.hidden_act
        return F.gelu(x) if a == "gelu" else (F.silu(x) if a in ("silu", "swish") else F.gelu(x, approximate="tanh"))

    def _rope(self, gh: int, gw: int):
        ch = (torch.arange(0.5, gh) / gh) * 2 - 1
        cw = (torch.arange(0.5, gw) / gw) * 2 - 1
        coords = torch.stack(torch.meshgrid(ch, cw, indexing="ij"), -1).reshape(-1, 2)  # [P, (y, x)]
        ang = (2 * math.pi * coords[:, :, None] * self.inv[None, None, :]).reshape(coords.shape[0], -1).repeat(1, 2)
        return ang.cos().to(self.device), ang.sin().to(self.device)

    @torch.no_grad()
    def __call__(self, pixels: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """pixels [B, 3, h, w] (preprocessed; multiples of the patch size) ->
        (last hidden [B, 1 + registers + patches, H], pooled CLS [B, H])."""
        c = self.cfg
        pixels = pixels.to(self.device, torch.float32)
        B, _, h, w = pixels.shape
        H, nh = c.hidden_size, c.num_attention_heads
        D = H // nh
        gh, gw = h // c.patch_size, w // c.patch_size
        x = _linear(_patch_rows(pixels, c.patch_size, self.w_patch.shape[1], self.dtype), self.w_patch, self.b_patch)
        parts = [self.cls.expand(B, 1, H)] + ([self.regs.expand(B, -1, H)] if self.regs is not None else []) + [x]
        x = torch.cat(parts, 1)
        n_pre = x.shape[1] - gh * gw
        cos, sin = self._rope(gh, gw)

        def rot(t):  # [B, nh, L, D]: rotate the patch tokens only
            pre, pt = t[:, :, :n_pre], t[:, :, n_pre:].float()
            half = D // 2
            r = torch.cat([-pt[..., half:], pt[..., :half]], -1)
            return torch.cat([pre, (pt * cos + r * sin).to(t.dtype)], 2)
        for ly in self.layers:
            q, k, v = _linear(self._ln(x, ly["ln1"]), ly["qkv"], ly["qkv_b"]).split(H, -1)
            q, k, v = (t.reshape(B, -1, nh, D).transpose(1, 2) for t in (q, k, v))
            att = F.scaled_dot_product_attention(rot(q), rot(k), v).transpose(1, 2).reshape(B, -1, H)
            x = x + _linear(att, *ly["o"]) * ly["ls1"]
            y = self._ln(x, ly["ln2"])
            m = ly["mlp"]
            if "gate" in m:
                hdn = (self._act(_linear(y, *m["gate"]).float()) * _linear(y, *m["up"]).float()).to(y.dtype)
            else:
                hdn = self._act(_linear(y, *m["up"]).float()).to(y.dtype)
            x = x + _linear(hdn, *m["down"]) * ly["ls2"]
        x = self._ln(x, self.norm)
        return x, x[:, 0]

    def embed(self, pixels: torch.Tensor, normalize: bool = True) -> torch.Tensor:
        _, pooled = self(pixels)
        e = pooled.float()
        return F.normalize(e, dim=-1) if normalize else e


# ---------------------------------------------------------------------------
# SigLIP 2 (NaFlex: native aspect ratio, variable patch count)
# ---------------------------------------------------------------------------

def naflex_size(height: int, width: int, patch: int, max_patches: int) -> tuple[int, int]:
    """Largest resize of (height, width), each side a multiple of the patch,
    with at most ``max_patches`` patches (the scale found by bisection, as the
    SigLIP 2 processor does)."""
    def side(scale, n):
        return max(patch, int(math.ceil(n * scale / patch) * patch))
    lo, hi = 1e-6, 100.0
    while hi - lo >= 1e-5:
        s = (lo + hi) / 2
        if (side(s, height) / patch) * (side(s, width) / patch) <= max_patches:
            lo = s
        else:
            hi = s
    return side(lo, height), side(lo, width)


class Siglip2Encoder(VisionEncoder):
    """SigLIP 2 vision tower over NaFlex inputs: patches [B, L, p * p * C]
    (row-major patches, channel-last inside each), their grid shapes [B, 2] and
    a validity mask [B, L]. The learned square position table is resized
    (bilinear, antialiased) to each image's grid; padded patches are masked as
    keys in every block and in the attention-pooling head.

    Reference: crates/rlx-siglip2 (SigLIP 2 image tower); transformers'
    Siglip2VisionModel is the CPU oracle."""

    def _positions(self, shapes: torch.Tensor, L: int) -> torch.Tensor:
        n = self.pos.shape[0]
        side = int(round(math.sqrt(n)))
        table = self.pos.float().reshape(side, side, -1).permute(2, 0, 1)[None]
        out = torch.empty(len(shapes), L, table.shape[1], device=self.device)
        for i, (h, w) in enumerate(shapes.tolist()):
            r = F.interpolate(table, size=(h, w), mode="bilinear", align_corners=False, antialias=True)
            r = r.reshape(table.shape[1], h * w).t()
            out[i, :h * w] = r
            out[i, h * w:] = r[0]
        return out

    def _attend_masked(self, q, k, v, nh, mask):
        B, Lq, H = q.shape
        D = H // nh
        q, k, v = (t.reshape(B, -1, nh, D).transpose(1, 2) for t in (q, k, v))
        return F.scaled_dot_product_attention(q, k, v, attn_mask=mask).transpose(1, 2).reshape(B, Lq, H)

    @torch.no_grad()
    def forward_patches(self, patches: torch.Tensor, shapes: torch.Tensor, valid: torch.Tensor):
        """-> (last hidden [B, L, H] after the post-norm, pooled [B, H] or None)."""
        c = self.cfg
        H, nh = c.hidden_size, c.num_attention_heads
        B, L, K = patches.shape
        rows = patches.to(self.device, self.dtype).reshape(B * L, K)
        if rows.shape[1] != self.w_patch.shape[1]:
            rows = F.pad(rows, (0, self.w_patch.shape[1] - rows.shape[1]))
        x = _linear(rows.contiguous(), self.w_patch, self.b_patch).view(B, L, H)
        x = (x.float() + self._positions(shapes, L)).to(self.dtype)
        valid = valid.to(self.device).bool()
        mask = valid[:, None, None, :]
        for ly in self.layers:
            q, k, v = _linear(self._ln(x, ly["ln1"]), ly["qkv"], ly["qkv_b"]).split(H, -1)
            x = x + _linear(self._attend_masked(q, k, v, nh, mask), *ly["o"])
            x = x + _linear(self._act(_linear(self._ln(x, ly["ln2"]), *ly["fc1"])).to(x.dtype), *ly["fc2"])
        x = self._ln(x, self.post_ln)
        if self.head is None:
            return x, None
        hd = self.head
        wq, wk, wv = hd["in_w"].split(H, 0)
        bq, bk, bv = hd["in_b"].split(H, 0)
        probe = hd["probe"].expand(B, 1, H)
        h = _linear(self._attend_masked(_linear(probe, wq, bq), _linear(x, wk, bk), _linear(x, wv, bv), nh, mask),
                    *hd["o"])
        h = h + _linear(self._act(_linear(self._ln(h, hd["ln"]), *hd["fc1"])).to(h.dtype), *hd["fc2"])
        return x, h[:, 0]

    def patchify(self, images, max_patches: int = 256, mean=(0.5, 0.5, 0.5), std=(0.5, 0.5, 0.5)):
        """Images -> (patches [B, max_patches, p * p * 3], shapes [B, 2], valid [B, max_patches]):
        NaFlex resize (bilinear), rescale to [0, 1], normalise, row-major patches."""
        from PIL import Image

        from ..utils.preprocess import load_image, normalize, to_tensor
        p = self.cfg.patch_size
        out, shapes, valid = [], [], []
        for im in images:
            im = load_image(im)
            w0, h0 = im.size
            th, tw = naflex_size(h0, w0, p, max_patches)
            t = normalize(to_tensor(im.resize((tw, th), resample=Image.BILINEAR)), mean, std)    # [3, th, tw]
            gh, gw = th // p, tw // p
            rows = t.view(3, gh, p, gw, p).permute(1, 3, 2, 4, 0).reshape(gh * gw, p * p * 3)
            out.append(F.pad(rows, (0, 0, 0, max_patches - rows.shape[0])))
            shapes.append((gh, gw))
            valid.append(torch.arange(max_patches) < gh * gw)
        return torch.stack(out), torch.tensor(shapes), torch.stack(valid)

    def embed_images(self, images, max_patches: int = 256, normalize: bool = True) -> torch.Tensor:
        patches, shapes, valid = self.patchify(images, max_patches)
        _, pooled = self.forward_patches(patches, shapes, valid)
        e = pooled.float()
        return F.normalize(e, dim=-1) if normalize else e
