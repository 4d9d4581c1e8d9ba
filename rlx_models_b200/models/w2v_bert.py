"""wav2vec 2.0-BERT (w2v-BERT 2.0) Conformer encoder with a CTC head
(transformers ``wav2vec2-bert``).

    input    stacked log-mel filterbank frames [T, 160] (the SeamlessM4T feature
             extractor's output: 80 bins, two frames per row)
    project  x = Linear(LayerNorm(features))
    layer    x += 0.5 FFN1(LN(x));  x += MHSA(LN(x));  x += Conv(x);
             x += 0.5 FFN2(LN(x));  x = LN(x)
    MHSA     scores = q k^T / sqrt(d) + q . E[clamp(j - i, -L, R) + L] / sqrt(d)
             ("relative_key": a learned embedding per clipped key-query distance)
    Conv     LN -> pointwise conv to 2C -> GLU -> causal depthwise conv ->
             LN -> act -> pointwise conv
    head     logits = lm_head(x) -> greedy CTC (blank = pad id)

Linear layers (FFNs, attention projections, pointwise convs, the head) run on
the package's tcgen05 GEMM in bf16 on the GPU (fp32 on CPU); attention with
the distance bias and the depthwise conv are torch ops.

Reference: crates/rlx-wav2vec2-bert (w2v-BERT 2.0 Conformer ASR);
transformers' Wav2Vec2BertForCTC is the CPU oracle.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .flux_text import _linear


@dataclass
class W2vBertConfig:
    hidden_size: int = 1024
    num_hidden_layers: int = 24
    num_attention_heads: int = 16
    intermediate_size: int = 4096
    feature_projection_input_dim: int = 160
    hidden_act: str = "swish"
    layer_norm_eps: float = 1e-5
    conv_depthwise_kernel_size: int = 31
    position_embeddings_type: str | None = "relative_key"
    left_max_position_embeddings: int = 64
    right_max_position_embeddings: int = 8
    vocab_size: int = 32
    pad_token_id: int = 0
    add_adapter: bool = False
    use_intermediate_ffn_before_adapter: bool = False

    @classmethod
    def from_dict(cls, d: dict) -> "W2vBertConfig":
        kw = {k: d[k] for k in cls.__dataclass_fields__ if k in d}
        c = cls(**kw)
        if c.add_adapter:
            raise NotImplementedError("w2v-BERT adapter layers are not built")
        if c.position_embeddings_type not in (None, "relative_key"):
            raise NotImplementedError(f"position_embeddings_type {c.position_embeddings_type!r}")
        return c


def _kaldi_mel_bank(n_mels: int, n_fft: int, sr: int, f_min: float = 20.0) -> torch.Tensor:
    """[n_fft // 2 + 1, n_mels] triangles laid out evenly on Kaldi's mel scale
    1127 ln(1 + f / 700) and evaluated there (no area normalisation)."""
    mel = lambda f: 1127.0 * torch.log1p(torch.as_tensor(f, dtype=torch.float64) / 700.0)  # noqa: E731
    edges = torch.linspace(float(mel(f_min)), float(mel(sr / 2)), n_mels + 2, dtype=torch.float64)
    m = mel(torch.linspace(0, sr / 2, n_fft // 2 + 1, dtype=torch.float64))[:, None]
    lo, c, hi = edges[None, :-2], edges[None, 1:-1], edges[None, 2:]
    return torch.clamp(torch.minimum((m - lo) / (c - lo), (hi - m) / (hi - c)), min=0.0)


def fbank_features(audio, sample_rate: int = 16000, n_mels: int = 80, stride: int = 2) -> torch.Tensor:
    """The w2v-BERT / SeamlessM4T input features of one clip: Kaldi-style log mel
    filterbank (16-bit scale, 25 ms Povey windows every 10 ms, DC offset removed,
    pre-emphasis 0.97, 512-point power spectrum, 80 Kaldi-mel triangles from
    20 Hz, log with a floor of 2^-23), normalised per mel bin (mean, unbiased
    variance + 1e-7), and ``stride`` consecutive frames stacked per row ->
    [frames // stride, n_mels * stride] fp32."""
    x = torch.as_tensor(audio, dtype=torch.float64).flatten() * 2.0 ** 15
    flen, hop, nfft = 400, 160, 512
    n = 1 + (x.numel() - flen) // hop
    fr = x.unfold(0, flen, hop)[:n].clone()
    fr -= fr.mean(-1, keepdim=True)
    fr[:, 1:] -= 0.97 * fr[:, :-1].clone()
    fr[:, 0] *= 1 - 0.97
    win = torch.hann_window(flen, periodic=False, dtype=torch.float64).pow(0.85)
    spec = torch.fft.rfft(fr * win, n=nfft).abs().pow(2)
    feats = torch.log(torch.clamp(spec @ _kaldi_mel_bank(n_mels, nfft, sample_rate), min=1.192092955078125e-07))
    feats = (feats - feats.mean(0, keepdim=True)) / torch.sqrt(feats.var(0, unbiased=True, keepdim=True) + 1e-7)
    T = feats.shape[0] - feats.shape[0] % stride
    return feats[:T].reshape(T // stride, n_mels * stride).float()


def _act(name, x):
    if name in ("swish", "silu"):
        return F.silu(x)
    if name == "gelu":
        return F.gelu(x)
    if name == "relu":
        return F.relu(x)
    raise NotImplementedError(f"activation {name!r}")


class W2vBertCTC:
    def __init__(self, cfg: W2vBertConfig, weights, device="cpu"):
        self.cfg, self.device = cfg, torch.device(device)
        self.dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])
        has = lambda k: k in weights  # noqa: E731
        pre = "wav2vec2_bert."
        lw = lambda n: get(n).to(self.device, self.dtype).contiguous()  # noqa: E731
        f32 = lambda n: get(n).to(self.device, torch.float32).contiguous()  # noqa: E731
        ln = lambda n: (f32(n + ".weight"), f32(n + ".bias"))  # noqa: E731
        lin = lambda n: (lw(n + ".weight"), lw(n + ".bias") if has(n + ".bias") else None)  # noqa: E731
        fp = pre + "feature_projection."
        self.fp_ln, self.fp = ln(fp + "layer_norm"), lin(fp + "projection")
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            p = f"{pre}encoder.layers.{i}."
            a, cv = p + "self_attn.", p + "conv_module."
            L = dict(ln_f1=ln(p + "ffn1_layer_norm"), f1a=lin(p + "ffn1.intermediate_dense"),
                     f1b=lin(p + "ffn1.output_dense"), ln_a=ln(p + "self_attn_layer_norm"),
                     qkv=(torch.cat([lw(a + f"linear_{n}.weight") for n in "qkv"]),
                          torch.cat([lw(a + f"linear_{n}.bias") for n in "qkv"])),
                     out=lin(a + "linear_out"), ln_c=ln(cv + "layer_norm"),
                     pw1=(lw(cv + "pointwise_conv1.weight").squeeze(-1).contiguous(), None),
                     dw=f32(cv + "depthwise_conv.weight"), ln_dw=ln(cv + "depthwise_layer_norm"),
                     pw2=(lw(cv + "pointwise_conv2.weight").squeeze(-1).contiguous(), None),
                     ln_f2=ln(p + "ffn2_layer_norm"), f2a=lin(p + "ffn2.intermediate_dense"),
                     f2b=lin(p + "ffn2.output_dense"), ln_out=ln(p + "final_layer_norm"))
            if cfg.position_embeddings_type == "relative_key":
                L["dist"] = f32(a + "distance_embedding.weight")
            self.layers.append(L)
        self.inter = None
        if cfg.use_intermediate_ffn_before_adapter and has(pre + "intermediate_ffn.intermediate_dense.weight"):
            self.inter = (lin(pre + "intermediate_ffn.intermediate_dense"), lin(pre + "intermediate_ffn.output_dense"))
        self.head = lin("lm_head")

    def _lin(self, x, wb):
        return _linear(x.to(self.dtype).contiguous(), *wb).float()

    def _ln(self, x, wb):
        return F.layer_norm(x, (x.shape[-1],), wb[0], wb[1], self.cfg.layer_norm_eps)

    def _ffn(self, x, a, b, act):
        return self._lin(_act(act, self._lin(x, a)), b)

    def _attn(self, L, x):
        c = self.cfg
        T, C = x.shape
        nh = c.num_attention_heads
        d = C // nh
        q, k, v = self._lin(x, L["qkv"]).view(T, 3, nh, d).unbind(1)
        q, k, v = (t.transpose(0, 1) for t in (q, k, v))  # [nh, T, d]
        bias = None
        if "dist" in L:
            pos = torch.arange(T, device=x.device)
            dist = (pos[None, :] - pos[:, None]).clamp(-c.left_max_position_embeddings,
                                                        c.right_max_position_embeddings)
            E = L["dist"][dist + c.left_max_position_embeddings]  # [T, T, d]
            bias = torch.einsum("hld,lrd->hlr", q, E) / d ** 0.5
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=bias, scale=d ** -0.5)
        return self._lin(o.transpose(0, 1).reshape(T, C), L["out"])

    def _conv(self, L, x):
        c = self.cfg
        h = F.glu(self._lin(self._ln(x, L["ln_c"]), L["pw1"]), dim=-1)  # [T, C]
        K = L["dw"].shape[-1]
        h = F.conv1d(F.pad(h.t()[None], (K - 1, 0)), L["dw"], groups=h.shape[1])[0].t()
        h = _act(c.hidden_act, self._ln(h, L["ln_dw"]))
        return self._lin(h, L["pw2"])

    @torch.no_grad()
    def hidden(self, features: torch.Tensor) -> torch.Tensor:
        """features [T, feature_projection_input_dim] -> encoder output [T, hidden] fp32."""
        c = self.cfg
        x = self._lin(self._ln(features.to(self.device, torch.float32), self.fp_ln), self.fp)
        for L in self.layers:
            x = x + 0.5 * self._ffn(self._ln(x, L["ln_f1"]), L["f1a"], L["f1b"], c.hidden_act)
            x = x + self._attn(L, self._ln(x, L["ln_a"]))
            x = x + self._conv(L, x)
            x = x + 0.5 * self._ffn(self._ln(x, L["ln_f2"]), L["f2a"], L["f2b"], c.hidden_act)
            x = self._ln(x, L["ln_out"])
        if self.inter is not None:
            x = x + 0.5 * self._ffn(x, self.inter[0], self.inter[1], "relu")
        return x

    @torch.no_grad()
    def logits(self, features: torch.Tensor) -> torch.Tensor:
        return self._lin(self.hidden(features), self.head)

    @torch.no_grad()
    def transcribe_ids(self, features: torch.Tensor) -> list[int]:
        """Greedy CTC: argmax per frame, repeats merged, blanks (pad id) dropped."""
        best = self.logits(features).argmax(-1).tolist()
        out, prev = [], None
        for t in best:
            if t != prev and t != self.cfg.pad_token_id:
                out.append(t)
            prev = t
        return out


class W2vBertTranscriber:
    """``transcribe(audio, sample_rate)``: mono 16 kHz, filterbank features,
    greedy CTC, tokenizer decode (token ids when there is no tokenizer)."""

    def __init__(self, model: W2vBertCTC, tokenizer=None):
        self.model, self.tokenizer = model, tokenizer

    def transcribe(self, audio, sample_rate: int = 16000):
        a = torch.as_tensor(audio, dtype=torch.float32)
        if a.dim() > 1:
            a = a.mean(-1)
        if sample_rate != 16000:
            a = F.interpolate(a[None, None], scale_factor=16000 / sample_rate, mode="linear",
                              align_corners=False)[0, 0]
        ids = self.model.transcribe_ids(fbank_features(a))
        return self.tokenizer.decode(ids) if self.tokenizer is not None else ids
