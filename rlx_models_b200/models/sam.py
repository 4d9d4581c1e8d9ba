"""Segment Anything (SAM v1): a ViT image encoder with windowed / global
attention and decomposed relative positions, a prompt encoder (points, boxes,
mask) and a two-way transformer mask decoder.

    image encoder  patches (16 px) + absolute position table -> L blocks of
                   x += proj(attn(LN(x)))   (14 x 14 windows, or global in the listed
                                             blocks; scores += q . R_h[qy - ky] + q . R_w[qx - kx])
                   x += MLP(LN(x))
                   -> neck: conv1x1 -> LN2d -> conv3x3 -> LN2d -> [256, 64, 64]
    prompts        points / box corners: random Fourier features of the normalised
                   coordinates + a learned embedding per label (pad point, negative,
                   positive, box corner 1 / 2); mask: two stride-2 convs + LN + GELU + 1x1
                   conv, else a learned "no mask" vector over the grid
    mask decoder   tokens [iou, mask x 4, prompts] and the image grid exchange information
                   in 2 two-way blocks (token self-attention, token->image and image->token
                   cross-attention at half width, MLP) + a final token->image attention;
                   the grid is upsampled x4 by two transposed convs; each mask token's
                   3-layer MLP gives a hypernetwork vector dotted with every upsampled
                   pixel -> low-resolution mask logits [256, 256]; an MLP on the IoU
                   token scores the masks

On the GPU the image encoder (the cost: 4096 tokens through 12 blocks for
ViT-B) runs its GEMMs in bf16 on the package's tcgen05 linear; attention
with the relative-position bias goes through torch SDPA with the bias as an
additive mask; the neck's 3x3 conv, the prompt encoder and the mask decoder
(a few tokens against one 64 x 64 grid) stay in fp32 torch.

Checkpoint names: transformers' SamModel layout.

Reference: the reference's SAM v1 crate (crates/rlx-sam/src/lib.rs:16-40:
preprocessing, encoder with windowed + global attention and decomposed
relative positions, neck; the prompt encoder and mask decoder in its later
phases) and the SAM mask-decoder IR (crates/rlx-sam-ir).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from .flux_text import _linear


@dataclass
class SamVisionCfg:
    hidden_size: int = 768
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    mlp_dim: int = 3072
    image_size: int = 1024
    patch_size: int = 16
    num_channels: int = 3
    window_size: int = 14
    global_attn_indexes: list = field(default_factory=lambda: [2, 5, 8, 11])
    output_channels: int = 256
    num_pos_feats: int = 128
    layer_norm_eps: float = 1e-6
    use_abs_pos: bool = True
    use_rel_pos: bool = True
    qkv_bias: bool = True
    hidden_act: str = "gelu"


@dataclass
class SamPromptCfg:
    hidden_size: int = 256
    image_size: int = 1024
    image_embedding_size: int = 64
    mask_input_channels: int = 16
    layer_norm_eps: float = 1e-6
    hidden_act: str = "gelu"


@dataclass
class SamDecoderCfg:
    hidden_size: int = 256
    mlp_dim: int = 2048
    num_hidden_layers: int = 2
    num_attention_heads: int = 8
    attention_downsample_rate: int = 2
    num_multimask_outputs: int = 3
    iou_head_depth: int = 3
    iou_head_hidden_dim: int = 256
    layer_norm_eps: float = 1e-6
    hidden_act: str = "relu"


@dataclass
class SamConfig:
    vision: SamVisionCfg = field(default_factory=SamVisionCfg)
    prompt: SamPromptCfg = field(default_factory=SamPromptCfg)
    decoder: SamDecoderCfg = field(default_factory=SamDecoderCfg)

    @classmethod
    def from_dict(cls, d: dict) -> "SamConfig":
        def pick(klass, sub):
            names = set(klass.__dataclass_fields__)
            return klass(**{k: v for k, v in (sub or {}).items() if k in names})
        return cls(vision=pick(SamVisionCfg, d.get("vision_config")),
                   prompt=pick(SamPromptCfg, d.get("prompt_encoder_config")),
                   decoder=pick(SamDecoderCfg, d.get("mask_decoder_config")))


def _act(name: str, x: torch.Tensor) -> torch.Tensor:
    if name == "gelu":
        return F.gelu(x)
    if name == "relu":
        return F.relu(x)
    if name in ("gelu_new", "gelu_pytorch_tanh"):
        return F.gelu(x, approximate="tanh")
    raise NotImplementedError(f"activation {name!r}")


def _ln(x, w, b, eps):
    return F.layer_norm(x.float(), (x.shape[-1],), w, b, eps)


def _ln2d(x, w, b, eps):
    """LayerNorm over the channel axis of [B, C, H, W]."""
    return _ln(x.permute(0, 2, 3, 1), w, b, eps).permute(0, 3, 1, 2)


def _rel_table(q_size: int, k_size: int, table: torch.Tensor) -> torch.Tensor:
    """[q_size, k_size, d] relative-position embeddings for every (query, key)
    offset along one axis; the table is linearly resampled when its length is
    not 2 * max(q, k) - 1."""
    n = 2 * max(q_size, k_size) - 1
    if table.shape[0] != n:
        table = F.interpolate(table.float().t()[None], size=n, mode="linear")[0].t()
    q = torch.arange(q_size, device=table.device)[:, None] * max(k_size / q_size, 1.0)
    k = torch.arange(k_size, device=table.device)[None, :] * max(q_size / k_size, 1.0)
    return table[((q - k) + (k_size - 1) * max(q_size / k_size, 1.0)).long()]


class SamModel:
    def __init__(self, cfg: SamConfig, weights, device="cpu"):
        self.cfg = cfg
        self.device = torch.device(device)
        self.fast = self.device.type == "cuda"
        self.vdt = torch.bfloat16 if self.fast else torch.float32
        get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])
        names = set(weights.keys())
        f32 = lambda n: get(n).to(self.device, torch.float32).contiguous()  # noqa: E731
        vd = lambda n: get(n).to(self.device, self.vdt).contiguous()  # noqa: E731
        opt = lambda n, fn: fn(n) if n in names else None  # noqa: E731
        v = cfg.vision
        p = "vision_encoder."
        self.patch_w = vd(p + "patch_embed.projection.weight").reshape(v.hidden_size, -1)
        self.patch_b = vd(p + "patch_embed.projection.bias")
        self.pos_embed = opt(p + "pos_embed", f32)
        self.layers = []
        for i in range(v.num_hidden_layers):
            q = f"{p}layers.{i}."
            self.layers.append(dict(
                ln1=(f32(q + "layer_norm1.weight"), f32(q + "layer_norm1.bias")),
                ln2=(f32(q + "layer_norm2.weight"), f32(q + "layer_norm2.bias")),
                qkv=(vd(q + "attn.qkv.weight"), opt(q + "attn.qkv.bias", vd)),
                proj=(vd(q + "attn.proj.weight"), vd(q + "attn.proj.bias")),
                rel_h=opt(q + "attn.rel_pos_h", f32), rel_w=opt(q + "attn.rel_pos_w", f32),
                lin1=(vd(q + "mlp.lin1.weight"), vd(q + "mlp.lin1.bias")),
                lin2=(vd(q + "mlp.lin2.weight"), vd(q + "mlp.lin2.bias")),
                window=0 if i in v.global_attn_indexes else v.window_size))
        self.neck1 = vd(p + "neck.conv1.weight").reshape(v.output_channels, -1)
        self.neck_ln1 = (f32(p + "neck.layer_norm1.weight"), f32(p + "neck.layer_norm1.bias"))
        self.neck2 = f32(p + "neck.conv2.weight")
        self.neck_ln2 = (f32(p + "neck.layer_norm2.weight"), f32(p + "neck.layer_norm2.bias"))
        self.w = {n: f32(n) for n in names if not n.startswith(p)}
        if "shared_image_embedding.positional_embedding" not in self.w:
            self.w["shared_image_embedding.positional_embedding"] = self.w[
                "prompt_encoder.shared_embedding.positional_embedding"]

    # -- image encoder -----------------------------------------------------
    def _attention(self, x: torch.Tensor, L: dict) -> torch.Tensor:
        """x [N, h, w, C] (one window or the whole grid per row) -> [N, h, w, C]."""
        v = self.cfg.vision
        N, h, w, C = x.shape
        nh, hd = v.num_attention_heads, C // v.num_attention_heads
        qkv = _linear(x.reshape(N * h * w, C), *L["qkv"]).view(N, h * w, 3, nh, hd).permute(2, 0, 3, 1, 4)
        q, k, val = qkv[0], qkv[1], qkv[2]                      # [N, nh, hw, hd]
        bias = None
        if L["rel_h"] is not None:
            Rh = _rel_table(h, h, L["rel_h"])
            Rw = _rel_table(w, w, L["rel_w"])
            qr = q.float().reshape(N * nh, h, w, hd)
            rel_h = torch.einsum("bhwc,hkc->bhwk", qr, Rh)
            rel_w = torch.einsum("bhwc,wkc->bhwk", qr, Rw)
            bias = (rel_h[..., :, None] + rel_w[..., None, :]).reshape(N, nh, h * w, h * w)
        if self.fast:
            o = F.scaled_dot_product_attention(q, k, val, attn_mask=None if bias is None else bias.to(q.dtype))
        else:
            s = (q * hd ** -0.5) @ k.transpose(-2, -1)
            if bias is not None:
                s = s + bias
            o = torch.softmax(s.float(), -1).to(q.dtype) @ val
        o = o.permute(0, 2, 1, 3).reshape(N * h * w, C)
        return _linear(o.contiguous(), *L["proj"]).view(N, h, w, C)

    def _block(self, x: torch.Tensor, L: dict) -> torch.Tensor:
        v = self.cfg.vision
        B, H, W, C = x.shape
        y = _ln(x, *L["ln1"], v.layer_norm_eps).to(self.vdt)
        ws = L["window"]
        if ws > 0:
            ph, pw = (-H) % ws, (-W) % ws
            yp = F.pad(y, (0, 0, 0, pw, 0, ph))
            Hp, Wp = H + ph, W + pw
            win = yp.view(B, Hp // ws, ws, Wp // ws, ws, C).permute(0, 1, 3, 2, 4, 5).reshape(-1, ws, ws, C)
            o = self._attention(win, L)
            o = o.view(B, Hp // ws, Wp // ws, ws, ws, C).permute(0, 1, 3, 2, 4, 5).reshape(B, Hp, Wp, C)
            o = o[:, :H, :W]
        else:
            o = self._attention(y, L)
        x = x + o.float()
        y = _ln(x, *L["ln2"], v.layer_norm_eps).to(self.vdt).reshape(B * H * W, C)
        h = _act(v.hidden_act, _linear(y, *L["lin1"]).float()).to(self.vdt)
        return x + _linear(h, *L["lin2"]).float().view(B, H, W, C)

    @torch.no_grad()
    def image_embeddings(self, pixels: torch.Tensor) -> torch.Tensor:
        """Preprocessed pixels [B, 3, S, S] -> image embeddings [B, 256, S/16, S/16] fp32."""
        v = self.cfg.vision
        x = pixels.to(self.device, torch.float32)
        B, _, S, _ = x.shape
        g, P = S // v.patch_size, v.patch_size
        rows = x.view(B, v.num_channels, g, P, g, P).permute(0, 2, 4, 1, 3, 5).reshape(B * g * g, -1)
        h = _linear(rows.to(self.vdt).contiguous(), self.patch_w, self.patch_b).float().view(B, g, g, -1)
        if self.pos_embed is not None:
            h = h + self.pos_embed
        for L in self.layers:
            h = self._block(h, L)
        y = _linear(h.to(self.vdt).reshape(B * g * g, -1), self.neck1).float().view(B, g, g, -1)
        y = _ln(y, *self.neck_ln1, 1e-6).permute(0, 3, 1, 2)
        y = F.conv2d(y, self.neck2, padding=1)
        return _ln2d(y, *self.neck_ln2, 1e-6)

    # -- prompt encoder ----------------------------------------------------
    def _fourier(self, coords: torch.Tensor) -> torch.Tensor:
        """Coordinates in [0, 1] (last axis x, y) -> [..., 2 * num_pos_feats]."""
        c = (2 * coords - 1) @ self.w["shared_image_embedding.positional_embedding"]
        c = 2 * math.pi * c
        return torch.cat([torch.sin(c), torch.cos(c)], -1)

    def image_positional_embeddings(self) -> torch.Tensor:
        n = self.cfg.prompt.image_embedding_size
        t = (torch.arange(n, device=self.device, dtype=torch.float32) + 0.5) / n
        grid = torch.stack([t[None, :].expand(n, n), t[:, None].expand(n, n)], -1)   # (x, y)
        return self._fourier(grid).permute(2, 0, 1)[None]

    def _embed_points(self, points, labels, pad: bool):
        w, S = self.w, self.cfg.prompt.image_size
        pts = points.float() + 0.5
        labels = labels.to(pts.device)
        if pad:
            pts = torch.cat([pts, torch.zeros_like(pts[:, :, :1])], 2)
            labels = torch.cat([labels, -torch.ones_like(labels[:, :, :1])], 2)
        e = self._fourier(pts / S)
        lab = labels[..., None]
        e = torch.where(lab == -1, w["prompt_encoder.not_a_point_embed.weight"], e)
        e = torch.where(lab != -10, e, torch.zeros_like(e))
        e = torch.where(lab == 0, e + w["prompt_encoder.point_embed.0.weight"], e)
        e = torch.where(lab == 1, e + w["prompt_encoder.point_embed.1.weight"], e)
        return e

    def _embed_boxes(self, boxes):
        w, S = self.w, self.cfg.prompt.image_size
        B, nb = boxes.shape[:2]
        e = self._fourier((boxes.float() + 0.5).view(B, nb, 2, 2) / S)
        corner = torch.stack([w["prompt_encoder.point_embed.2.weight"][0], w["prompt_encoder.point_embed.3.weight"][0]])
        return e + corner

    def _embed_mask(self, masks):
        w, c = self.w, self.cfg.prompt
        p = "prompt_encoder.mask_embed."
        h = F.conv2d(masks.float(), w[p + "conv1.weight"], w[p + "conv1.bias"], stride=2)
        h = _act(c.hidden_act, _ln2d(h, w[p + "layer_norm1.weight"], w[p + "layer_norm1.bias"], c.layer_norm_eps))
        h = F.conv2d(h, w[p + "conv2.weight"], w[p + "conv2.bias"], stride=2)
        h = _act(c.hidden_act, _ln2d(h, w[p + "layer_norm2.weight"], w[p + "layer_norm2.bias"], c.layer_norm_eps))
        return F.conv2d(h, w[p + "conv3.weight"], w[p + "conv3.bias"])

    def prompt_embeddings(self, points=None, labels=None, boxes=None, masks=None):
        """points [B, P, n, 2] (input-image pixels) + labels [B, P, n] (1 positive,
        0 negative, -1 padding, -10 ignored), boxes [B, P, 4] (x0, y0, x1, y1),
        masks [B, 1, 256, 256] -> (sparse [B, P, m, 256] or None, dense [B, 256, 64, 64])."""
        dev = self.device
        sparse, B = None, 1
        if points is not None:
            points = points.to(dev)
            B = points.shape[0]
            if labels is None:
                labels = torch.ones(points.shape[:3], dtype=torch.int32, device=dev)
            sparse = self._embed_points(points, labels.to(dev), pad=boxes is None)
        if boxes is not None:
            boxes = boxes.to(dev)
            B = boxes.shape[0]
            be = self._embed_boxes(boxes)
            sparse = be if sparse is None else torch.cat([sparse, be], 2)
        n = self.cfg.prompt.image_embedding_size
        if masks is not None:
            dense = self._embed_mask(masks.to(dev))
        else:
            dense = self.w["prompt_encoder.no_mask_embed.weight"].reshape(1, -1, 1, 1).expand(B, -1, n, n)
        return sparse, dense

    # -- mask decoder ------------------------------------------------------
    def _attn(self, name, q, k, v, down):
        w, c = self.w, self.cfg.decoder
        lin = lambda x, n: x @ w[f"{name}.{n}.weight"].t() + w[f"{name}.{n}.bias"]  # noqa: E731
        q, k, v = lin(q, "q_proj"), lin(k, "k_proj"), lin(v, "v_proj")
        B, P, T, D = q.shape
        nh = c.num_attention_heads
        hd = D // nh
        sh = lambda x: x.reshape(B * P, x.shape[2], nh, hd).transpose(1, 2)  # noqa: E731
        s = (sh(q) @ sh(k).transpose(-2, -1)) * hd ** -0.5
        o = torch.softmax(s, -1) @ sh(v)
        o = o.transpose(1, 2).reshape(B, P, T, D)
        return lin(o, "out_proj")

    def _ln_dec(self, x, name, eps=None):
        return F.layer_norm(x, (x.shape[-1],), self.w[name + ".weight"], self.w[name + ".bias"],
                            self.cfg.decoder.layer_norm_eps if eps is None else eps)

    def _mlp(self, x, name, n_layers, act="relu"):
        w = self.w
        x = _act(act, x @ w[name + ".proj_in.weight"].t() + w[name + ".proj_in.bias"])
        for j in range(n_layers - 2):
            x = _act(act, x @ w[f"{name}.layers.{j}.weight"].t() + w[f"{name}.layers.{j}.bias"])
        return x @ w[name + ".proj_out.weight"].t() + w[name + ".proj_out.bias"]

    def _two_way(self, tokens, image, image_pe):
        c, w = self.cfg.decoder, self.w
        queries, keys = tokens, image
        for i in range(c.num_hidden_layers):
            p = f"mask_decoder.transformer.layers.{i}."
            if i == 0:
                queries = self._attn(p + "self_attn", queries, queries, queries, 1)
            else:
                q = queries + tokens
                queries = queries + self._attn(p + "self_attn", q, q, queries, 1)
            queries = self._ln_dec(queries, p + "layer_norm1")
            q, k = queries + tokens, keys + image_pe
            queries = queries + self._attn(p + "cross_attn_token_to_image", q, k, keys, c.attention_downsample_rate)
            queries = self._ln_dec(queries, p + "layer_norm2")
            h = _act(c.hidden_act, queries @ w[p + "mlp.lin1.weight"].t() + w[p + "mlp.lin1.bias"])
            queries = self._ln_dec(queries + h @ w[p + "mlp.lin2.weight"].t() + w[p + "mlp.lin2.bias"],
                                   p + "layer_norm3")
            q, k = queries + tokens, keys + image_pe
            keys = self._ln_dec(keys + self._attn(p + "cross_attn_image_to_token", k, q, queries,
                                                  c.attention_downsample_rate), p + "layer_norm4")
        p = "mask_decoder.transformer."
        q, k = queries + tokens, keys + image_pe
        queries = queries + self._attn(p + "final_attn_token_to_image", q, k, keys, c.attention_downsample_rate)
        return self._ln_dec(queries, p + "layer_norm_final_attn", eps=1e-5), keys

    @torch.no_grad()
    def decode_masks(self, image_emb, sparse, dense, multimask: bool = True):
        """-> (low-resolution mask logits [B, P, n, 4S/16, 4S/16], IoU scores [B, P, n])."""
        c, w = self.cfg.decoder, self.w
        B, C, H, W = image_emb.shape
        P = sparse.shape[1] if sparse is not None else 1
        nm = c.num_multimask_outputs + 1
        out_tok = torch.cat([w["mask_decoder.iou_token.weight"], w["mask_decoder.mask_tokens.weight"]])
        tokens = out_tok.expand(B, P, -1, -1)
        if sparse is not None:
            tokens = torch.cat([tokens, sparse], 2)
        img = (image_emb.to(self.device) + dense).repeat_interleave(P, 0)
        pe = self.image_positional_embeddings().expand(B * P, -1, -1, -1)
        img_seq = img.flatten(2).transpose(1, 2).reshape(B, P, H * W, C)
        pe_seq = pe.flatten(2).transpose(1, 2).reshape(B, P, H * W, C)
        hs, keys = self._two_way(tokens, img_seq, pe_seq)
        iou_tok, mask_tok = hs[:, :, 0], hs[:, :, 1:1 + nm]
        grid = keys.reshape(B * P, H, W, C).permute(0, 3, 1, 2)
        p = "mask_decoder."
        up = F.conv_transpose2d(grid, w[p + "upscale_conv1.weight"], w[p + "upscale_conv1.bias"], stride=2)
        up = F.gelu(_ln2d(up, w[p + "upscale_layer_norm.weight"], w[p + "upscale_layer_norm.bias"], 1e-6))
        up = F.gelu(F.conv_transpose2d(up, w[p + "upscale_conv2.weight"], w[p + "upscale_conv2.bias"], stride=2))
        hyper = torch.stack([self._mlp(mask_tok[:, :, i], f"{p}output_hypernetworks_mlps.{i}", 3)
                             for i in range(nm)], 2)                      # [B, P, nm, C/8]
        _, cu, hu, wu = up.shape
        masks = (hyper @ up.reshape(B, P, cu, hu * wu)).reshape(B, P, nm, hu, wu)
        iou = self._mlp(iou_tok, p + "iou_prediction_head", c.iou_head_depth)
        sl = slice(1, None) if multimask else slice(0, 1)
        return masks[:, :, sl], iou[:, :, sl]

    @torch.no_grad()
    def segment(self, pixels=None, points=None, labels=None, boxes=None, masks=None, image_embeddings=None,
                multimask: bool = True):
        """Masks and IoU scores for the prompts (``image_embeddings`` reuse an
        image's encoder output across prompts)."""
        emb = self.image_embeddings(pixels) if image_embeddings is None else image_embeddings.to(self.device)
        sparse, dense = self.prompt_embeddings(points, labels, boxes, masks)
        return self.decode_masks(emb, sparse, dense, multimask)


def upscale_masks(masks: torch.Tensor, original_size: tuple, reshaped_size: tuple, pad_size: int = 1024,
                  binarize: bool = True, threshold: float = 0.0) -> torch.Tensor:
    """Low-resolution logits [..., h, w] -> masks at the original image size:
    upsample to the padded input, cut the padding, resize to the original."""
    lead = masks.shape[:-2]
    m = masks.reshape(-1, 1, *masks.shape[-2:]).float()
    m = F.interpolate(m, (pad_size, pad_size), mode="bilinear", align_corners=False)
    m = m[..., :reshaped_size[0], :reshaped_size[1]]
    m = F.interpolate(m, tuple(original_size), mode="bilinear", align_corners=False)
    m = m.reshape(*lead, *original_size)
    return m > threshold if binarize else m
