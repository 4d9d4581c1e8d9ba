"""fp32 CPU oracle for the decoder families (the numerical spec).

A direct PyTorch restatement of the HF modules for Qwen3 (dense), Llama /
Qwen2 (no QK-norm, optional qkv bias) and gpt-oss (q/k/v/o biases, learned
sinks, alternating sliding/full attention, YaRN RoPE, top-k-then-softmax
router, MXFP4 experts with biases, clamped SwiGLU). Used as the reference for
the GPU model and as the CPU execution path of config 1 (Qwen3-0.6B shape,
fp32, prefill + greedy decode).

Reference behaviour: rlx-models-core src/standard_decoder.rs (`DecoderSpec`
:172-312, `build_gpt_oss_moe_ffn` :1040-1205, gpt-oss attention :11946-12079,
prefill :12081); rlx-qwen3 src/generator.rs (`prefill_get_last_logits` :4303,
`decode_get_logits` :4391). Unlike the reference gpt-oss builder (prefill
only, all layers treated as full attention), this oracle applies the sliding
window for sequences longer than the window and supports decode.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from ..config import DecoderConfig
from ..ops import reference as R
from ..ops import rope_inv_freq
from ..quant.mxfp4 import dequantize_mxfp4


class OracleKV:
    def __init__(self, n_layers: int):
        self.k = [None] * n_layers
        self.v = [None] * n_layers

    @property
    def length(self) -> int:
        return 0 if self.k[0] is None else self.k[0].shape[0]


class DecoderOracle:
    """fp32 decoder over a ``{hf_name: tensor}`` dict."""

    def __init__(self, cfg: DecoderConfig, weights: dict[str, torch.Tensor], device="cpu"):
        self.cfg = cfg
        self.device = torch.device(device)
        from ..weights.aliases import FusedSplitView, Llama4View, canonical_name
        if cfg.model_type == "llama4_text":  # feed_forward.* names, fused expert banks
            weights = Llama4View(weights).as_dict()
        if FusedSplitView.needed(weights):  # Phi-3 fused qkv / gate_up
            v = FusedSplitView(weights, cfg.q_size, cfg.kv_size, cfg.intermediate_size)
            weights = {k: v[k] for k in v.keys()}
        self.w = {canonical_name(cfg.model_type, k): v.to(self.device) for k, v in weights.items()}
        self.inv_freq, self.rope_mult = rope_inv_freq(cfg.rotary_dim, cfg.rope_theta, cfg.rope_scaling,
                                                      cfg.max_position_embeddings)
        # sliding-window layers with their own RoPE base (Gemma-3)
        self.local_rope = (rope_inv_freq(cfg.rotary_dim, cfg.rope_local_theta, None, cfg.max_position_embeddings)
                           if cfg.rope_local_theta else None)
        self._experts: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}

    def W(self, name: str) -> torch.Tensor:
        return self.w[name].float()

    def N(self, name: str) -> torch.Tensor:
        """RMSNorm weight (Gemma stores w with the norm computing x * (1 + w))."""
        return self.W(name) + 1.0 if self.cfg.norm_unit_offset else self.W(name)

    def _mm(self, x: torch.Tensor, name: str) -> torch.Tensor:
        """x @ W^T; with ``self.taps`` set, records the input rows per weight
        name (calibration activations for quant.calib)."""
        taps = getattr(self, "taps", None)
        if taps is not None:
            taps.setdefault(name, []).append(x.detach().reshape(-1, x.shape[-1]).cpu())
        return x @ self.W(name).T

    def _experts_fp32(self, i: int):
        if i not in self._experts:
            p = f"model.layers.{i}.mlp.experts."
            if self.cfg.expert_quant == "mxfp4":
                gu = dequantize_mxfp4(self.w[p + "gate_up_proj_blocks"], self.w[p + "gate_up_proj_scales"])
                dn = dequantize_mxfp4(self.w[p + "down_proj_blocks"], self.w[p + "down_proj_scales"])
                # stored [E, out, in]; HF bf16 layout is [E, in, out]
                self._experts[i] = (gu.transpose(1, 2).contiguous(), dn.transpose(1, 2).contiguous())
            else:
                self._experts[i] = (self.W(p + "gate_up_proj"), self.W(p + "down_proj"))
        return self._experts[i]

    def _attn(self, i: int, x: torch.Tensor, pos: torch.Tensor, kv: OracleKV) -> torch.Tensor:
        c = self.cfg
        p = f"model.layers.{i}.self_attn."
        T = x.shape[0]

        def proj(n):
            y = self._mm(x, p + n + ".weight")
            if (p + n + ".bias") in self.w:
                y = y + self.W(p + n + ".bias")
            return y

        q = proj("q_proj").view(T, c.num_attention_heads, c.head_dim)
        k = proj("k_proj").view(T, c.num_key_value_heads, c.head_dim)
        v = proj("v_proj").view(T, c.num_key_value_heads, c.head_dim)
        if c.qk_norm_full:  # one norm over all heads of the token
            q = R.rmsnorm(q.reshape(T, -1), self.N(p + "q_norm.weight"), c.rms_norm_eps).view_as(q)
            k = R.rmsnorm(k.reshape(T, -1), self.N(p + "k_norm.weight"), c.rms_norm_eps).view_as(k)
        elif c.qk_norm:
            q = R.rmsnorm(q, self.N(p + "q_norm.weight"), c.rms_norm_eps)
            k = R.rmsnorm(k, self.N(p + "k_norm.weight"), c.rms_norm_eps)
        inv, mult = (self.local_rope if self.local_rope is not None and c.layer_window(i) > 0
                     else (self.inv_freq, self.rope_mult))
        chunk = 0
        if c.rope_layers is not None and not c.uses_rope(i):  # Llama-4 NoPE layer
            if c.attn_temperature_tuning:  # query temperature grows with log(position / floor_scale)
                q = q * (torch.log1p(torch.floor((pos.float() + 1.0) / c.floor_scale)) * c.attn_scale + 1.0)[:, None, None]
        elif c.rope_interleaved:
            q = R.rope_interleaved(q, pos, inv, mult)
            k = R.rope_interleaved(k, pos, inv, mult)
            chunk = c.attention_chunk_size
        else:
            q = R.rope(q, pos, inv, mult)
            k = R.rope(k, pos, inv, mult)
        if c.qk_l2_norm and c.uses_rope(i):  # weightless RMS norm after RoPE (Llama-4)
            q = q * torch.rsqrt(q.pow(2).mean(-1, keepdim=True) + c.rms_norm_eps)
            k = k * torch.rsqrt(k.pow(2).mean(-1, keepdim=True) + c.rms_norm_eps)
        if kv.k[i] is None:
            kv.k[i], kv.v[i] = k, v
        else:
            kv.k[i] = torch.cat([kv.k[i], k])
            kv.v[i] = torch.cat([kv.v[i], v])
        kpos = torch.arange(kv.k[i].shape[0], device=x.device)
        sinks = self.W(p + "sinks") if c.attn_sinks else None
        o = R.attention(q, kv.k[i], kv.v[i], pos, kpos, c.attention_multiplier or 1.0 / math.sqrt(c.head_dim),
                        causal=c.causal, window=c.layer_window(i), sinks=sinks, softcap=c.attn_softcap, chunk=chunk)
        y = self._mm(o.reshape(T, -1), p + "o_proj.weight")
        if (p + "o_proj.bias") in self.w:
            y = y + self.W(p + "o_proj.bias")
        return y

    def _mlp(self, i: int, x: torch.Tensor) -> torch.Tensor:
        c = self.cfg
        p = f"model.layers.{i}.mlp."
        if not c.is_moe_layer(i):
            g = self._mm(x, p + "gate_proj.weight")
            u = self._mm(x, p + "up_proj.weight")
            act = F.gelu(g, approximate="tanh") if c.mlp_act == "gelu_tanh" else F.silu(g)
            return self._mm(act * u, p + "down_proj.weight")
        if c.model_type == "gpt_oss":
            logits = x @ self.W(p + "router.weight").T + self.W(p + "router.bias")
            topv, topi = logits.topk(c.num_experts_per_tok, dim=-1)
            probs = torch.softmax(topv, dim=-1)
            gu_w, dn_w = self._experts_fp32(i)
            gu_b = self.W(p + "experts.gate_up_proj_bias")
            dn_b = self.W(p + "experts.down_proj_bias")
            out = torch.zeros_like(x)
            for slot in range(c.num_experts_per_tok):
                e = topi[:, slot]
                gu = torch.einsum("th,thn->tn", x, gu_w[e]) + gu_b[e]
                gate, up = gu[:, ::2], gu[:, 1::2]
                gate = gate.clamp(max=c.swiglu_limit)
                up = up.clamp(-c.swiglu_limit, c.swiglu_limit)
                act = (up + 1) * gate * torch.sigmoid(gate * c.swiglu_alpha)
                y = torch.einsum("tn,tnh->th", act, dn_w[e]) + dn_b[e]
                out += probs[:, slot:slot + 1] * y
            return out
        logits = x @ self.W(p + "gate.weight").T
        if c.router_scoring == "llama4":  # top-k on logits; each expert sees x * sigmoid(its logit)
            topv, topi = logits.topk(c.num_experts_per_tok, dim=-1)
            sc = torch.sigmoid(topv)
            out = torch.zeros_like(x)
            for t in range(x.shape[0]):
                for s in range(c.num_experts_per_tok):
                    pe = p + f"experts.{int(topi[t, s])}."
                    xs = x[t] * sc[t, s]
                    g = xs @ self.W(pe + "gate_proj.weight").T
                    u = xs @ self.W(pe + "up_proj.weight").T
                    out[t] += (F.silu(g) * u) @ self.W(pe + "down_proj.weight").T
            ps = p + "shared_experts."
            return out + (F.silu(x @ self.W(ps + "gate_proj.weight").T) * (x @ self.W(ps + "up_proj.weight").T)) \
                @ self.W(ps + "down_proj.weight").T
        if c.router_scoring == "sigmoid":  # glm4_moe: DeepSeek's group-limited sigmoid routing
            from types import SimpleNamespace
            from .deepseek import route
            spec = SimpleNamespace(scoring_func="sigmoid", topk_method="noaux_tc", n_group=c.n_group,
                                   topk_group=c.topk_group, num_experts_per_tok=c.num_experts_per_tok,
                                   norm_topk_prob=c.norm_topk_prob, routed_scaling_factor=c.routed_scaling_factor)
            topi, topv = route(spec, logits, self.W(p + "gate.e_score_correction_bias"))
        else:  # qwen3-moe style (softmax over all experts, top-k, optional renorm)
            probs = torch.softmax(logits, dim=-1)
            topv, topi = probs.topk(c.num_experts_per_tok, dim=-1)
            if c.norm_topk_prob:
                topv = topv / topv.sum(-1, keepdim=True)
        out = torch.zeros_like(x)
        for t in range(x.shape[0]):
            for s in range(c.num_experts_per_tok):
                e = int(topi[t, s])
                pe = p + f"experts.{e}."
                g = x[t] @ self.W(pe + "gate_proj.weight").T
                u = x[t] @ self.W(pe + "up_proj.weight").T
                out[t] += topv[t, s] * ((F.silu(g) * u) @ self.W(pe + "down_proj.weight").T)
        if c.n_shared_experts:  # glm4_moe: ungated shared experts
            ps = p + "shared_experts."
            out = out + (F.silu(x @ self.W(ps + "gate_proj.weight").T) * (x @ self.W(ps + "up_proj.weight").T)) \
                @ self.W(ps + "down_proj.weight").T
        elif c.shared_expert_intermediate_size:  # qwen2-moe: sigmoid-gated shared SwiGLU expert
            ps = p + "shared_expert."
            sh = (F.silu(x @ self.W(ps + "gate_proj.weight").T) * (x @ self.W(ps + "up_proj.weight").T)) \
                @ self.W(ps + "down_proj.weight").T
            out = out + torch.sigmoid(x @ self.W(p + "shared_expert_gate.weight").T) * sh
        return out

    @torch.no_grad()
    def forward(self, ids: torch.Tensor, kv: OracleKV | None = None, mm=None) -> tuple[torch.Tensor, OracleKV]:
        """ids: [T] new tokens continuing ``kv``; ``mm`` = (rows, embeds) replaces the
        input embeddings of those rows (image tokens). Returns fp32 logits [T, V]."""
        h, kv = self.forward_hidden(ids, kv, mm)
        c = self.cfg
        head = self.W("model.embed_tokens.weight") if c.tie_word_embeddings else self.W("lm_head.weight")
        logits = h @ head.T / c.logits_scaling
        if c.final_softcap > 0:
            logits = torch.tanh(logits / c.final_softcap) * c.final_softcap
        return logits, kv

    @torch.no_grad()
    def forward_hidden(self, ids: torch.Tensor, kv: OracleKV | None = None, mm=None) -> tuple[torch.Tensor, OracleKV]:
        """Final-normed hidden states [T, H] (the embedding models' last_hidden_state)."""
        c = self.cfg
        if kv is None:
            kv = OracleKV(c.num_hidden_layers)
        start = kv.length
        pos = torch.arange(start, start + ids.shape[0], device=self.device)
        h = self.W("model.embed_tokens.weight")[ids.to(self.device).long()] * c.embedding_multiplier
        if mm is not None:
            rows, emb = mm
            h = h.index_copy(0, rows.to(self.device).long(), emb.to(self.device, h.dtype))
        rm = c.residual_multiplier
        eps = c.rms_norm_eps
        for i in range(c.num_hidden_layers):
            p = f"model.layers.{i}."
            a = self._attn(i, R.rmsnorm(h, self.N(p + "input_layernorm.weight"), eps), pos, kv)
            if c.sandwich_norm:  # Gemma-2/3: norms on both sides of each sublayer
                h = h + R.rmsnorm(a, self.N(p + "post_attention_layernorm.weight"), eps)
                m = self._mlp(i, R.rmsnorm(h, self.N(p + "pre_feedforward_layernorm.weight"), eps))
                h = h + R.rmsnorm(m, self.N(p + "post_feedforward_layernorm.weight"), eps)
                continue
            h = h + rm * a
            h = h + rm * self._mlp(i, R.rmsnorm(h, self.N(p + "post_attention_layernorm.weight"), eps))
        return R.rmsnorm(h, self.N("model.norm.weight"), eps), kv

    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, max_new_tokens: int) -> tuple[list[int], list[torch.Tensor]]:
        """Greedy decode. Returns new token ids and the logits at each step."""
        logits, kv = self.forward(prompt)
        out, all_logits = [], [logits[-1]]
        nxt = int(logits[-1].argmax())
        for _ in range(max_new_tokens):
            out.append(nxt)
            if len(out) == max_new_tokens:
                break
            logits, kv = self.forward(torch.tensor([nxt]), kv)
            all_logits.append(logits[-1])
            nxt = int(logits[-1].argmax())
        return out, all_logits
