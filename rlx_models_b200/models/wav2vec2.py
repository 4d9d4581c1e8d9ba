"""wav2vec 2.0 CTC speech recognition (Wav2Vec2ForCTC checkpoints: base /
large / large-lv60 / XLSR fine-tunes).

    features   raw 16 kHz audio -> 7 strided convs (kernels 10,3,3,3,3,2,2; strides
               5,2,2,2,2,2,2; 512 channels; GELU): the first followed by a per-channel
               norm over time ("group" models) or every conv by a LayerNorm over
               channels ("layer" models)  -> one frame per 20 ms
    projection LayerNorm + linear to the model width
    positions  x += GELU(grouped conv(x), kernel 128, 16 groups, weight-normalised over
               the kernel axis, last output dropped)
    encoder    post-norm blocks (x = LN(x + attn(x)); x = LN(x + FFN(x)), after an
               input LayerNorm) or, for "stable layer norm" models, pre-norm blocks with
               a final LayerNorm
    head       linear to the character vocabulary; greedy CTC (argmax per frame,
               repeats merged, the pad / blank id dropped); padded batches mask the
               attention to each input's frames

The feature convolutions run channels-last as GEMMs on the shared codec
blocks (``models/codec_common.py``: GELU fused into the next conv's operand);
the first conv's per-channel norm is ``ops.instance_norm``; the linears run on
the tcgen05 GEMM in bf16; the grouped positional conv is a torch conv1d and
attention is torch SDPA with a key-padding mask.

Reference: crates/rlx-wav2vec2-asr (wav2vec 2.0 CTC recognition); transformers'
Wav2Vec2ForCTC is the CPU oracle.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from .codec_common import ConvRunner, GemmConv, fold_weight_norm
from .flux_text import _linear


@dataclass
class Wav2Vec2Config:
    hidden_size: int = 768
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    intermediate_size: int = 3072
    hidden_act: str = "gelu"
    layer_norm_eps: float = 1e-5
    feat_extract_norm: str = "group"
    feat_extract_activation: str = "gelu"
    conv_dim: list = field(default_factory=lambda: [512] * 7)
    conv_kernel: list = field(default_factory=lambda: [10, 3, 3, 3, 3, 2, 2])
    conv_stride: list = field(default_factory=lambda: [5, 2, 2, 2, 2, 2, 2])
    conv_bias: bool = False
    num_conv_pos_embeddings: int = 128
    num_conv_pos_embedding_groups: int = 16
    do_stable_layer_norm: bool = False
    vocab_size: int = 32
    pad_token_id: int = 0

    @classmethod
    def from_dict(cls, d: dict) -> "Wav2Vec2Config":
        names = set(cls.__dataclass_fields__)
        return cls(**{k: v for k, v in d.items() if k in names and v is not None})

    def frames(self, samples: int) -> int:
        for k, s in zip(self.conv_kernel, self.conv_stride):
            samples = (samples - k) // s + 1
        return samples


def _act(name, x):
    if name == "gelu":
        return F.gelu(x)
    if name in ("gelu_new", "gelu_pytorch_tanh"):
        return F.gelu(x, approximate="tanh")
    if name == "relu":
        return F.relu(x)
    raise NotImplementedError(f"activation {name!r}")


class Wav2Vec2CTC:
    def __init__(self, cfg: Wav2Vec2Config, weights, device="cpu"):
        self.cfg = cfg
        self.run = ConvRunner(device)
        self.device, self.dtype = self.run.device, self.run.dtype
        get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])
        raw = {k: get(k) for k in weights.keys()}
        pre = "wav2vec2." if any(k.startswith("wav2vec2.") for k in raw) else ""
        w = fold_weight_norm(raw)
        dev, dt = self.device, self.dtype
        f32 = lambda n: w[n].to(dev, torch.float32).contiguous()  # noqa: E731
        lw = lambda n: w[n].to(dev, dt).contiguous()  # noqa: E731
        fe = pre + "feature_extractor.conv_layers."
        self.convs, self.conv_norms = [], []
        for i in range(len(cfg.conv_dim)):
            self.convs.append(GemmConv(w[f"{fe}{i}.conv.weight"], w.get(f"{fe}{i}.conv.bias"), False, dt, dev))
            nw = f"{fe}{i}.layer_norm.weight"
            self.conv_norms.append((f32(nw), f32(f"{fe}{i}.layer_norm.bias")) if nw in w else None)
        fp = pre + "feature_projection."
        self.fp_ln = (f32(fp + "layer_norm.weight"), f32(fp + "layer_norm.bias"))
        self.fp = (lw(fp + "projection.weight"), lw(fp + "projection.bias"))
        en = pre + "encoder."
        self.pos_w = f32(en + "pos_conv_embed.conv.weight")
        self.pos_b = f32(en + "pos_conv_embed.conv.bias")
        self.enc_ln = (f32(en + "layer_norm.weight"), f32(en + "layer_norm.bias"))
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            p = f"{en}layers.{i}."
            qkv_w = torch.cat([w[p + f"attention.{n}_proj.weight"] for n in "qkv"]).to(dev, dt).contiguous()
            qkv_b = torch.cat([w[p + f"attention.{n}_proj.bias"] for n in "qkv"]).to(dev, dt).contiguous()
            self.layers.append(dict(
                qkv=(qkv_w, qkv_b), o=(lw(p + "attention.out_proj.weight"), lw(p + "attention.out_proj.bias")),
                ln=(f32(p + "layer_norm.weight"), f32(p + "layer_norm.bias")),
                ff1=(lw(p + "feed_forward.intermediate_dense.weight"), lw(p + "feed_forward.intermediate_dense.bias")),
                ff2=(lw(p + "feed_forward.output_dense.weight"), lw(p + "feed_forward.output_dense.bias")),
                ln2=(f32(p + "final_layer_norm.weight"), f32(p + "final_layer_norm.bias"))))
        self.head = (lw("lm_head.weight"), lw("lm_head.bias")) if "lm_head.weight" in w else None

    # -- features ----------------------------------------------------------
    def _features(self, audio: torch.Tensor) -> torch.Tensor:
        """[B, samples] -> [B, frames, conv_dim[-1]] fp32."""
        c = self.cfg
        x = audio.to(self.device, self.dtype)[:, :, None].contiguous()
        act = None
        for i, L in enumerate(self.convs):
            x = self.run.conv(x, L, act=act, stride=c.conv_stride[i])
            norm = self.conv_norms[i]
            if norm is not None and c.feat_extract_norm == "group" and i == 0:
                x = self._channel_norm(x, *norm)
            elif norm is not None:
                x = F.layer_norm(x.float(), (x.shape[-1],), *norm, 1e-5).to(self.dtype)
            act = c.feat_extract_activation          # fused into the next conv's operand
        return _act(act, x.float())

    def _channel_norm(self, x, g, b):
        """Per-channel normalisation over time (GroupNorm with one group per channel)."""
        xt = x.transpose(1, 2).contiguous()          # [B, C, T]
        if self.run.fast:
            y = self.run.ops.instance_norm(xt.float(), g, b, eps=1e-5)
        else:
            y = F.group_norm(xt.float(), xt.shape[1], g, b, 1e-5)
        return y.transpose(1, 2).to(self.dtype).contiguous()

    # -- encoder -----------------------------------------------------------
    def _attention(self, x, L, mask):
        c = self.cfg
        B, T, H = x.shape
        nh = c.num_attention_heads
        qkv = _linear(x.to(self.dtype).reshape(B * T, H).contiguous(), *L["qkv"]).view(B, T, 3, nh, H // nh)
        q, k, v = qkv.permute(2, 0, 3, 1, 4)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
        o = o.transpose(1, 2).reshape(B * T, H).contiguous()
        return _linear(o, *L["o"]).float().view(B, T, H)

    def _ffn(self, x, L):
        B, T, H = x.shape
        h = _act(self.cfg.hidden_act, _linear(x.to(self.dtype).reshape(B * T, H).contiguous(), *L["ff1"]).float())
        return _linear(h.to(self.dtype), *L["ff2"]).float().view(B, T, H)

    @torch.no_grad()
    def hidden_states(self, audio: torch.Tensor, lengths=None):
        """audio [B, samples] (zero-padded) -> (encoder output [B, frames, H] fp32,
        valid frames per input)."""
        c = self.cfg
        eps = c.layer_norm_eps
        feats = self._features(audio)
        B, T, _ = feats.shape
        n = torch.full((B,), T, dtype=torch.long) if lengths is None else \
            torch.tensor([c.frames(int(s)) for s in lengths]).clamp(max=T)
        x = F.layer_norm(feats, (feats.shape[-1],), *self.fp_ln, eps)
        x = _linear(x.to(self.dtype).reshape(B * T, -1).contiguous(), *self.fp).float().view(B, T, -1)
        mask = None
        if lengths is not None and bool((n < T).any()):
            valid = torch.arange(T)[None, :] < n[:, None]
            x = x * valid.to(x.device)[..., None]
            mask = valid.to(self.device)[:, None, None, :]
        pad = c.num_conv_pos_embeddings // 2
        pos = F.conv1d(x.transpose(1, 2), self.pos_w, self.pos_b, padding=pad, groups=c.num_conv_pos_embedding_groups)
        if c.num_conv_pos_embeddings % 2 == 0:
            pos = pos[..., :-1]
        x = x + _act(c.feat_extract_activation, pos).transpose(1, 2)
        if not c.do_stable_layer_norm:
            x = F.layer_norm(x, (x.shape[-1],), *self.enc_ln, eps)
        for L in self.layers:
            if c.do_stable_layer_norm:
                x = x + self._attention(F.layer_norm(x, (x.shape[-1],), *L["ln"], eps), L, mask)
                x = x + self._ffn(F.layer_norm(x, (x.shape[-1],), *L["ln2"], eps), L)
            else:
                x = F.layer_norm(x + self._attention(x, L, mask), (x.shape[-1],), *L["ln"], eps)
                x = F.layer_norm(x + self._ffn(x, L), (x.shape[-1],), *L["ln2"], eps)
        if c.do_stable_layer_norm:
            x = F.layer_norm(x, (x.shape[-1],), *self.enc_ln, eps)
        return x, n

    @torch.no_grad()
    def logits(self, audio: torch.Tensor, lengths=None):
        """-> (CTC logits [B, frames, vocab] fp32, valid frames)."""
        x, n = self.hidden_states(audio, lengths)
        B, T, H = x.shape
        return _linear(x.to(self.dtype).reshape(B * T, H).contiguous(), *self.head).float().view(B, T, -1), n

    def greedy(self, audio: torch.Tensor, lengths=None) -> list[list[int]]:
        lg, n = self.logits(audio, lengths)
        out = []
        for b in range(lg.shape[0]):
            best = lg[b, :int(n[b])].argmax(-1).tolist()
            seq, prev = [], None
            for t in best:
                if t != prev and t != self.cfg.pad_token_id:
                    seq.append(t)
                prev = t
            out.append(seq)
        return out


class Wav2Vec2Transcriber:
    """``transcribe(audio, sample_rate)``: zero-mean / unit-variance input
    normalisation (the released feature extractors'), greedy CTC, tokenizer decode."""

    def __init__(self, model: Wav2Vec2CTC, tokenizer=None, normalize: bool = True):
        self.model, self.tokenizer, self.normalize = model, tokenizer, normalize

    def transcribe(self, audio, sample_rate: int = 16000):
        a = torch.as_tensor(audio, dtype=torch.float32)
        if a.dim() > 1:
            a = a.mean(-1)
        if sample_rate != 16000:
            a = F.interpolate(a[None, None], scale_factor=16000 / sample_rate, mode="linear",
                              align_corners=False)[0, 0]
        if self.normalize:
            a = (a - a.mean()) / torch.sqrt(a.var(unbiased=False) + 1e-7)
        ids = self.model.greedy(a[None])[0]
        return self.tokenizer.decode(ids) if self.tokenizer is not None else ids
