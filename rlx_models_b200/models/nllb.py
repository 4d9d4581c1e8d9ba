"""NLLB-200 / M2M-100 many-to-many translation: a pre-norm Transformer
encoder-decoder over a shared multilingual vocabulary.

    embed    token embedding x sqrt(d_model) + sinusoidal positions (fairseq
             layout: [sin | cos], positions counted from padding_idx + 1 over the
             non-pad tokens; the pad row is zero)
    encoder  x += attn(LN(x)); x += fc2(act(fc1(LN(x)))); final LN
    decoder  the same with causal self-attention and cross-attention on the
             encoder output (pre-norm), final LN, tied output projection
    decoding the decoder starts from </s> then the target-language token
             (``forced_bos``) and runs greedily to </s> or the length limit; the
             self-attention K / V of earlier steps are kept and the cross K / V
             are projected once per source

Linear layers run on the package's tcgen05 GEMM in bf16 on the GPU (fp32 on
CPU); attention is torch SDPA.

Checkpoint names: transformers' M2M100ForConditionalGeneration (NLLB-200 uses
the same architecture and names).

Reference: crates/rlx-nllb (NLLB-200 translation); transformers'
M2M100ForConditionalGeneration is the CPU oracle.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .flux_text import _linear


@dataclass
class NllbConfig:
    d_model: int = 1024
    encoder_layers: int = 24
    decoder_layers: int = 24
    encoder_attention_heads: int = 16
    decoder_attention_heads: int = 16
    encoder_ffn_dim: int = 8192
    decoder_ffn_dim: int = 8192
    activation_function: str = "relu"
    vocab_size: int = 256206
    max_position_embeddings: int = 1024
    pad_token_id: int = 1
    eos_token_id: int = 2
    decoder_start_token_id: int = 2
    scale_embedding: bool = True

    @classmethod
    def from_dict(cls, d: dict) -> "NllbConfig":
        names = set(cls.__dataclass_fields__)
        return cls(**{k: v for k, v in d.items() if k in names and v is not None})


def sinusoidal_table(n: int, dim: int, padding_idx: int | None) -> torch.Tensor:
    """[n, dim] table: row p = [sin(p w_i) | cos(p w_i)], w_i = 10000^(-i / (dim/2 - 1))."""
    half = dim // 2
    freq = torch.exp(torch.arange(half, dtype=torch.float32) * -(math.log(10000.0) / (half - 1)))
    ang = torch.arange(n, dtype=torch.float32)[:, None] * freq[None]
    t = torch.cat([torch.sin(ang), torch.cos(ang)], 1)
    if dim % 2:
        t = F.pad(t, (0, 1))
    if padding_idx is not None:
        t[padding_idx] = 0
    return t


def _act(name, x):
    return {"relu": F.relu, "gelu": F.gelu, "silu": F.silu}[name](x)


class NllbTranslator:
    def __init__(self, cfg: NllbConfig, weights, device="cpu"):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dt = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])
        names = set(weights.keys())
        dev, dt = self.device, self.dt
        lw = lambda n: get(n).to(dev, dt).contiguous()  # noqa: E731
        f32 = lambda n: get(n).to(dev, torch.float32).contiguous()  # noqa: E731
        emb = "model.shared.weight" if "model.shared.weight" in names else "model.encoder.embed_tokens.weight"
        self.embed = f32(emb)
        self.head = lw("lm_head.weight") if "lm_head.weight" in names else self.embed.to(dt)
        self.scale = math.sqrt(cfg.d_model) if cfg.scale_embedding else 1.0
        n_pos = cfg.max_position_embeddings + cfg.pad_token_id + 1
        self.pos = sinusoidal_table(n_pos, cfg.d_model, cfg.pad_token_id).to(dev)

        def attn(p):
            return dict(qkv=(torch.cat([get(p + f"{n}_proj.weight") for n in "qkv"]).to(dev, dt).contiguous(),
                             torch.cat([get(p + f"{n}_proj.bias") for n in "qkv"]).to(dev, dt).contiguous()),
                        q=(lw(p + "q_proj.weight"), lw(p + "q_proj.bias")),
                        kv=(torch.cat([get(p + f"{n}_proj.weight") for n in "kv"]).to(dev, dt).contiguous(),
                            torch.cat([get(p + f"{n}_proj.bias") for n in "kv"]).to(dev, dt).contiguous()),
                        o=(lw(p + "out_proj.weight"), lw(p + "out_proj.bias")))

        def ln(n):
            return f32(n + ".weight"), f32(n + ".bias")

        self.enc = []
        for i in range(cfg.encoder_layers):
            p = f"model.encoder.layers.{i}."
            self.enc.append(dict(sa=attn(p + "self_attn."), ln1=ln(p + "self_attn_layer_norm"),
                                 fc1=(lw(p + "fc1.weight"), lw(p + "fc1.bias")),
                                 fc2=(lw(p + "fc2.weight"), lw(p + "fc2.bias")), ln2=ln(p + "final_layer_norm")))
        self.enc_ln = ln("model.encoder.layer_norm")
        self.dec = []
        for i in range(cfg.decoder_layers):
            p = f"model.decoder.layers.{i}."
            self.dec.append(dict(sa=attn(p + "self_attn."), ln1=ln(p + "self_attn_layer_norm"),
                                 ca=attn(p + "encoder_attn."), ln_c=ln(p + "encoder_attn_layer_norm"),
                                 fc1=(lw(p + "fc1.weight"), lw(p + "fc1.bias")),
                                 fc2=(lw(p + "fc2.weight"), lw(p + "fc2.bias")), ln2=ln(p + "final_layer_norm")))
        self.dec_ln = ln("model.decoder.layer_norm")

    # -- pieces ------------------------------------------------------------
    def _lin(self, x, wb):
        shp = x.shape
        return _linear(x.reshape(-1, shp[-1]).to(self.dt).contiguous(), *wb).float().view(*shp[:-1], -1)

    def _embed(self, ids, positions):
        return self.embed[ids] * self.scale + self.pos[positions]

    @staticmethod
    def _ln(x, wb):
        return F.layer_norm(x, (x.shape[-1],), wb[0], wb[1], 1e-5)

    def _heads(self, x, nh):
        B, T, D = x.shape
        return x.view(B, T, nh, D // nh).transpose(1, 2).to(self.dt)

    def _ffn(self, x, L):
        return self._lin(_act(self.cfg.activation_function, self._lin(self._ln(x, L["ln2"]), L["fc1"])), L["fc2"])

    # -- encoder -----------------------------------------------------------
    @torch.no_grad()
    def encode(self, ids: torch.Tensor):
        """ids [B, S] (right-padded with pad_token_id) -> (encoder states [B, S, d] fp32,
        key mask [B, 1, 1, S] or None)."""
        c = self.cfg
        ids = ids.to(self.device)
        valid = ids.ne(c.pad_token_id)
        positions = torch.cumsum(valid.int(), 1) * valid + c.pad_token_id
        x = self._embed(ids, positions)
        mask = valid[:, None, None, :] if not bool(valid.all()) else None
        nh = c.encoder_attention_heads
        for L in self.enc:
            h = self._ln(x, L["ln1"])
            q, k, v = self._lin(h, L["sa"]["qkv"]).split(c.d_model, -1)
            o = F.scaled_dot_product_attention(self._heads(q, nh), self._heads(k, nh), self._heads(v, nh),
                                               attn_mask=mask)
            x = x + self._lin(o.transpose(1, 2).reshape(x.shape).float(), L["sa"]["o"])
            x = x + self._ffn(x, L)
        return self._ln(x, self.enc_ln), mask

    def cross_kv(self, enc: torch.Tensor) -> list:
        nh = self.cfg.decoder_attention_heads
        out = []
        for L in self.dec:
            k, v = self._lin(enc, L["ca"]["kv"]).split(self.cfg.d_model, -1)
            out.append((self._heads(k, nh), self._heads(v, nh)))
        return out

    # -- decoder -----------------------------------------------------------
    @torch.no_grad()
    def decode_step(self, ids: torch.Tensor, start: int, cache: list, cross: list, enc_mask=None) -> torch.Tensor:
        """New decoder tokens ids [B, T] at positions start .. start + T - 1
        (``cache`` holds the self-attention K / V of earlier positions, extended
        in place) -> logits [B, T, V] fp32."""
        c = self.cfg
        ids = ids.to(self.device)
        B, T = ids.shape
        positions = torch.arange(start, start + T, device=self.device)[None].expand(B, T) + c.pad_token_id + 1
        x = self._embed(ids, positions)
        nh = c.decoder_attention_heads
        if T > 1 and start > 0:
            raise NotImplementedError("multi-token decoder steps after the first")
        for i, L in enumerate(self.dec):
            h = self._ln(x, L["ln1"])
            q, k, v = self._lin(h, L["sa"]["qkv"]).split(c.d_model, -1)
            k, v = self._heads(k, nh), self._heads(v, nh)
            if len(cache) > i:
                k = torch.cat([cache[i][0], k], 2)
                v = torch.cat([cache[i][1], v], 2)
                cache[i] = (k, v)
            else:
                cache.append((k, v))
            o = F.scaled_dot_product_attention(self._heads(q, nh), k, v, is_causal=T > 1)
            x = x + self._lin(o.transpose(1, 2).reshape(B, T, -1).float(), L["sa"]["o"])
            h = self._ln(x, L["ln_c"])
            q = self._lin(h, L["ca"]["q"])
            o = F.scaled_dot_product_attention(self._heads(q, nh), cross[i][0], cross[i][1], attn_mask=enc_mask)
            x = x + self._lin(o.transpose(1, 2).reshape(B, T, -1).float(), L["ca"]["o"])
            x = x + self._ffn(x, L)
        x = self._ln(x, self.dec_ln)
        return _linear(x.reshape(B * T, -1).to(self.dt).contiguous(), self.head).float().view(B, T, -1)

    @torch.no_grad()
    def generate(self, src_ids: torch.Tensor, forced_bos: int | None = None, max_new_tokens: int = 64) -> list:
        """Greedy translation of src_ids [B, S] -> per input the generated ids
        (after the start token; the forced language token first, </s> last when reached)."""
        c = self.cfg
        enc, mask = self.encode(src_ids)
        cross = self.cross_kv(enc)
        B = enc.shape[0]
        cache: list = []
        tok = torch.full((B, 1), c.decoder_start_token_id, dtype=torch.long, device=self.device)
        out = [[] for _ in range(B)]
        done = torch.zeros(B, dtype=torch.bool, device=self.device)
        for step in range(max_new_tokens):
            lg = self.decode_step(tok, step, cache, cross, mask)[:, -1]
            if step == 0 and forced_bos is not None:
                nxt = torch.full((B,), forced_bos, dtype=torch.long, device=self.device)
            else:
                nxt = lg.argmax(-1)
            nxt = torch.where(done, torch.full_like(nxt, c.pad_token_id), nxt)
            for b in range(B):
                if not bool(done[b]):
                    out[b].append(int(nxt[b]))
            done = done | nxt.eq(c.eos_token_id)
            if bool(done.all()):
                break
            tok = nxt[:, None]
        return out
