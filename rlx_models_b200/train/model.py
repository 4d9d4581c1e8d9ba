"""Trainable decoder (Qwen3 / Llama family) on FSDP parameter groups.

Groups: one per transformer layer (q|k|v fused rows, o, gate|up fused rows,
down, the norms) plus an outer group (embedding, final norm, untied lm_head).
Forward gathers a group right before it is used; with activation
checkpointing each layer is recomputed in backward (gathering again), so the
live parameter footprint is one layer plus the outer group.

Tensor names and layouts are the HF ones the reference's loaders read
(rlx-qwen3 src/lib.rs:140-245; rlx-models-core src/weight_map.rs), so
checkpoints round-trip through :mod:`rlx_models_b200.weights`.
"""
from __future__ import annotations


import torch
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint

from ..config import DecoderConfig
from ..ops import rope_inv_freq
from . import functional as TF
from .fsdp import FlatGroup, gather_params


def _layer_tensors(cfg: DecoderConfig, i: int, get) -> list[tuple[str, torch.Tensor]]:
    p = f"model.layers.{i}."
    out = [(p + "input_layernorm.weight", get(p + "input_layernorm.weight")),
           (p + "self_attn.qkv_proj.weight", torch.cat([get(p + "self_attn.q_proj.weight"),
                                                        get(p + "self_attn.k_proj.weight"),
                                                        get(p + "self_attn.v_proj.weight")], 0))]
    if cfg.qk_norm:
        out += [(p + "self_attn.q_norm.weight", get(p + "self_attn.q_norm.weight")),
                (p + "self_attn.k_norm.weight", get(p + "self_attn.k_norm.weight"))]
    out += [(p + "self_attn.o_proj.weight", get(p + "self_attn.o_proj.weight")),
            (p + "post_attention_layernorm.weight", get(p + "post_attention_layernorm.weight")),
            (p + "mlp.gate_up_proj.weight", torch.cat([get(p + "mlp.gate_proj.weight"),
                                                       get(p + "mlp.up_proj.weight")], 0)),
            (p + "mlp.down_proj.weight", get(p + "mlp.down_proj.weight"))]
    return out


def split_fused(named: dict[str, torch.Tensor], cfg: DecoderConfig) -> dict[str, torch.Tensor]:
    """Fused training tensors -> HF names (q/k/v and gate/up split back)."""
    out = {}
    q, kv = cfg.q_size, cfg.kv_size
    for n, t in named.items():
        if n.endswith("self_attn.qkv_proj.weight"):
            b = n[:-len("qkv_proj.weight")]
            out[b + "q_proj.weight"], out[b + "k_proj.weight"], out[b + "v_proj.weight"] = torch.split(t, [q, kv, kv])
        elif n.endswith("mlp.gate_up_proj.weight"):
            b = n[:-len("gate_up_proj.weight")]
            out[b + "gate_proj.weight"], out[b + "up_proj.weight"] = torch.split(t, [t.shape[0] // 2] * 2)
        else:
            out[n] = t
    return out


class TrainableDecoder:
    def __init__(self, cfg: DecoderConfig, weights, rank: int = 0, world: int = 1, device="cuda", group=None,
                 activation_checkpointing: bool = True, max_seq: int = 8192,
                 param_dtype: torch.dtype = torch.bfloat16):
        assert not cfg.is_moe, "dense decoders only"
        self.cfg = cfg
        self.device = torch.device(device)
        self.ckpt = activation_checkpointing

        def get(name):
            t = weights.take(name) if hasattr(weights, "take") else weights[name]
            return t.to(self.device)

        outer = [("model.embed_tokens.weight", get("model.embed_tokens.weight")),
                 ("model.norm.weight", get("model.norm.weight"))]
        if not cfg.tie_word_embeddings:
            outer.append(("lm_head.weight", get("lm_head.weight")))
        self.outer = FlatGroup("outer", outer, rank, world, self.device, group, param_dtype)
        del outer
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            self.layers.append(FlatGroup(f"layer{i}", _layer_tensors(cfg, i, get), rank, world, self.device, group,
                                         param_dtype))
        inv, mult = rope_inv_freq(cfg.rotary_dim, cfg.rope_theta, cfg.rope_scaling, cfg.max_position_embeddings)
        t = torch.arange(max_seq, dtype=torch.float32)
        freqs = torch.outer(t, inv)
        emb = torch.cat([freqs, freqs], -1)
        self.cos = (emb.cos() * mult).to(self.device, torch.bfloat16)
        self.sin = (emb.sin() * mult).to(self.device, torch.bfloat16)
        self.lora = None  # train.lora.LoraAdapters when fine-tuning with adapters

    @property
    def groups(self) -> list[FlatGroup]:
        return [self.outer] + self.layers

    def num_params(self) -> int:
        return sum(g.numel for g in self.groups)

    def _prefetch_next(self, i: int):
        """Overlap the next layer's parameter all-gather with this layer: i + 1
        in forward order, i - 1 in the backward recompute (descending order)."""
        last, self._last_layer = getattr(self, "_last_layer", None), i
        nxt = i - 1 if (last is not None and last == i + 1) else i + 1
        if 0 <= nxt < len(self.layers) and not self.layers[nxt].frozen:
            self.layers[nxt].prefetch()

    def _layer(self, h: torch.Tensor, i: int) -> torch.Tensor:
        c = self.cfg
        w = gather_params(self.layers[i])
        self._prefetch_next(i)
        if c.qk_norm:
            ln1, wqkv, qn, kn, wo, ln2, wgu, wd = w
        else:
            ln1, wqkv, wo, ln2, wgu, wd = w
            qn = kn = None
        B, S, H = h.shape
        if getattr(self, "qat", None):  # quantisation-aware training: fake-quantised weights, STE gradients
            from ..quant.dwq import fake_quant
            wqkv, wo, wgu, wd = (fake_quant(t, self.qat) for t in (wqkv, wo, wgu, wd))
        if self.lora is not None:
            lp = self.lora.params()
            lin = lambda t, x, w: self.lora.linear(lp, i, t, x, w)
            lin_res = lambda t, x, w, r: r + lin(t, x, w)
        else:
            lin = lambda t, x, w: TF.linear(x, w)
            lin_res = lambda t, x, w, r: TF.linear_residual(x, w, r)  # residual add in the GEMM epilogue
        a = TF.rmsnorm(h, ln1, c.rms_norm_eps)
        qkv = lin("qkv", a, wqkv)
        cos, sin = self.cos[:S], self.sin[:S]
        q, k, v = TF.qk_norm_rope(qkv, qn, kn, cos, sin, c.num_attention_heads, c.num_key_value_heads, c.head_dim,
                                  c.rms_norm_eps)
        o = TF.attention(q, k, v, causal=True).reshape(B, S, c.q_size)
        h = lin_res("o", o, wo, h)
        m = TF.rmsnorm(h, ln2, c.rms_norm_eps)
        gu = lin("gate_up", m, wgu)
        return lin_res("down", TF.swiglu(gu), wd, h)

    def loss(self, ids: torch.Tensor, targets: torch.Tensor, denom: float | None = None) -> torch.Tensor:
        """Summed CE over valid targets divided by ``denom`` (default: this
        batch's valid-target count)."""
        c = self.cfg
        ow = gather_params(self.outer)
        embed, norm = ow[0], ow[1]
        head = embed if c.tie_word_embeddings else ow[2]
        h = F.embedding(ids, embed)
        for i in range(len(self.layers)):
            if self.ckpt and torch.is_grad_enabled():
                h = checkpoint(self._layer, h, i, use_reentrant=False)
            else:
                h = self._layer(h, i)
        x = TF.rmsnorm(h, norm, c.rms_norm_eps)
        return TF.lm_head_ce(x.reshape(-1, c.hidden_size), head, targets.reshape(-1), 2048, denom)

    def hf_state_dict(self) -> dict[str, torch.Tensor]:
        named = {}
        for g in self.groups:
            named.update(g.named_full())
        return split_fused(named, self.cfg)
