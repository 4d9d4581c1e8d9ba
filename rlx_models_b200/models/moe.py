"""GPU mixture-of-experts decoder (gpt-oss, Qwen3-MoE, Mixtral, Qwen2-MoE,
GLM-4.5 / glm4_moe) on the sm_100a kernels.

Attention is the dense decoder's (q/k/v/o biases, learned sinks, alternating
128-token sliding window / full attention, YaRN RoPE); the MLP is a routed
expert block with MXFP4 expert weights kept packed in HBM:

    router GEMM (f32 logits, bias) -> top-k, softmax over the k
    -> moe_align (device counts / offsets / permutation / tile list)
    -> gather rows -> grouped MXFP4 GEMM gate|up (bias, clamped SwiGLU)
    -> grouped MXFP4 GEMM down (bias, x router weight) -> combine

Expert parallelism: rank r holds experts [r E/ep, (r+1) E/ep). Every rank
routes all tokens of the step (attention is replicated), so dispatch is a
local gather, and runs only its own experts. Combine: for decode-sized steps
one kernel reads each token's k expert rows from the owning ranks' HBM over
NVLink and fuses the residual add and the next RMSNorm (parallel/ep.py);
larger steps sum per-rank partials with an NCCL all-reduce.

Reference: rlx-models-core src/standard_decoder.rs:1040-1205
(`build_gpt_oss_moe_ffn`), :11873-12208 (`GptOssSpec`, sinks attention,
prefill); crates/rlx-gpt-oss/src/gpt_oss_ops.rs (clamped SwiGLU, alpha 1.702,
limit 7). The reference has no decode path and treats every layer as full
attention; both are implemented here.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from ..config import DecoderConfig
from ..ops._ext import ext, scratch
from ..quant.mxfp4 import quantize_mxfp4, tile_mxfp4
from .decoder import DecoderLM, LayerWeights

GROUP = 64  # gate/up rows interleaved in groups of 64 for the fused epilogue


def hf_interleaved_to_grouped(t: torch.Tensor, dim: int = 1) -> torch.Tensor:
    """HF gpt-oss gate_up rows alternate (gate, up, gate, up, ...); the grouped
    GEMM wants [64 gate rows][64 up rows] per 128-row tile."""
    n = t.shape[dim]
    idx = torch.arange(n, device=t.device).view(n // (2 * GROUP), GROUP, 2)  # [g, j, (gate, up)]
    order = idx.permute(0, 2, 1).reshape(-1)  # g: gate_j..., up_j...
    return t.index_select(dim, order)


def token_tile(n_assign: int, num_experts: int) -> int:
    """Token-tile width of the grouped GEMM from the mean rows per expert."""
    avg = n_assign / max(1, num_experts)
    for bt in (32, 64):
        if avg <= bt:
            return bt
    return 128


def pack_experts(gates, ups, downs):
    """Per-expert gate / up [I, H] and down [H, I] fp32 -> tiled MXFP4 banks
    (gu_w, gu_exp, dn_w, dn_exp) for the grouped GEMM, gate / up rows in
    [64 gate][64 up] groups for its fused SwiGLU epilogue."""
    I = gates[0].shape[0]
    gu = torch.stack([torch.stack([g.reshape(I // GROUP, GROUP, -1), u.reshape(I // GROUP, GROUP, -1)], 1)
                      .reshape(2 * I, -1) for g, u in zip(gates, ups)])
    gu_w, gu_exp = tile_mxfp4(*quantize_mxfp4(gu))
    del gu
    dn_w, dn_exp = tile_mxfp4(*quantize_mxfp4(torch.stack(list(downs))))
    return gu_w, gu_exp, dn_w, dn_exp


def routed_experts(x: torch.Tensor, experts: torch.Tensor, weights: torch.Tensor, gu_w, gu_exp, dn_w, dn_exp,
                   num_experts: int, inter: int, alpha: float = 1.0) -> torch.Tensor:
    """sum_s weights[t, s] * expert_{experts[t, s]}(x[t]) on the grouped MXFP4
    GEMM (no biases, every expert local): align -> gather -> gate/up GEMM with
    the u * g * sigmoid(alpha g) epilogue (SwiGLU at alpha = 1; relu(u)^2 for
    experts packed with gate = up and a huge alpha) -> down GEMM scaled by the
    router weight -> combine."""
    T, H = x.shape
    k = experts.shape[1]
    E = num_experts
    dev = x.device
    n = T * k
    bt = token_tile(n, E)
    meta = torch.empty(2 * E + 2, dtype=torch.int32, device=dev)
    tiles = torch.empty(4 * (n // bt + E + 1), dtype=torch.int32, device=dev)
    perm = torch.empty(n, dtype=torch.int32, device=dev)
    inv = torch.empty(n, dtype=torch.int32, device=dev)
    cursor = torch.empty(E, dtype=torch.int32, device=dev)
    ext().moe_align(experts, E, 0, E, bt, meta, tiles, perm, inv, cursor)
    xa = torch.empty(n, H, dtype=torch.float16, device=dev)
    ext().moe_gather(x, perm, meta, E, k, xa)
    s = scratch(dev)
    gu = torch.empty(n, inter, dtype=torch.float16, device=dev)
    ext().moe_gemm(xa, gu_w, gu_exp, 2 * inter, None, None, perm, meta, tiles, gu, True, 1e30, float(alpha), bt,
                   s.status, 0.0)
    dn = torch.empty(n, H, dtype=torch.bfloat16, device=dev)
    ext().moe_gemm(gu, dn_w, dn_exp, H, None, weights.reshape(-1), perm, meta, tiles, dn, False, 0.0, 0.0, bt,
                   s.status)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    ext().moe_combine(dn, inv, k, out, False)
    ops._count(5)
    return out


def softmax_topk(logits: torch.Tensor, k: int, renorm: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """(expert ids int32 [T, k], weights fp32 [T, k]) of softmax-then-top-k
    routing on the device (optionally renormalised over the k)."""
    T = logits.shape[0]
    experts = torch.empty(T, k, dtype=torch.int32, device=logits.device)
    weights = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    ext().moe_route(logits, k, True, renorm, experts, weights)
    ops._count(1)
    return experts, weights


class MoELayer:
    __slots__ = ("router_w", "router_b", "router_corr", "gu_w", "gu_exp", "gu_bias", "dn_w", "dn_exp", "dn_bias",
                 "sh_gu", "sh_dn", "sh_gate")


class MoEDecoderLM(DecoderLM):
    def __init__(self, cfg: DecoderConfig, weights, device="cuda", ep_rank: int = 0, ep_size: int = 1, comm=None,
                 ep_combine: str = "fused", combine_max_tokens: int = 512):
        """``ep_combine``: "fused" gathers each token's expert rows from the
        owning ranks over NVLink and fuses the residual add and RMSNorm into the
        same kernel (parallel/ep.py) for steps of up to ``combine_max_tokens``
        tokens; larger steps, and "nccl", sum per-rank partials with an NCCL
        all-reduce."""
        assert cfg.is_moe
        if cfg.router_scoring == "llama4" and cfg.num_experts_per_tok != 1:
            raise NotImplementedError("Llama-4 routing scales the expert input: top-1 only on the GPU path")
        self.ep_rank, self.ep_size = ep_rank, ep_size
        assert cfg.num_experts % ep_size == 0
        self.e_local = cfg.num_experts // ep_size
        self.e_lo = ep_rank * self.e_local
        # attention / embeddings are replicated: build the dense parts with tp_size=1
        self._moe_comm = comm
        super().__init__(cfg, weights, device=device, tp_rank=0, tp_size=1, comm=None)
        self.combiner = None
        if ep_size > 1 and not (dist.is_available() and dist.is_initialized()):
            # one rank of an EP model built without a process group (single-GPU timing of a
            # rank's share: bench/decode_step.py --tp-emulate): only its own experts contribute
            ep_combine = "local"
        self._ep_local_only = ep_combine == "local"
        if ep_combine == "fused":
            from ..parallel.ep import EPCombiner
            n_moe = sum(cfg.is_moe_layer(i) for i in range(cfg.num_hidden_layers))
            self.combiner = EPCombiner(ep_rank, ep_size, self.device, hidden=cfg.hidden_size,
                                       top_k=cfg.num_experts_per_tok, e_local=self.e_local,
                                       max_tokens=combine_max_tokens, num_layers=n_moe,
                                       eps=cfg.rms_norm_eps)
        if cfg.rope_layers is not None:
            # Llama-4: chunked attention on the RoPE layers and the NoPE layers' query
            # temperature both start at position min(chunk, floor_scale); below it the
            # layers are plain causal attention, which is what the kernels here run
            lim = [v for v in (cfg.attention_chunk_size, int(cfg.floor_scale) if cfg.attn_temperature_tuning else 0)
                   if v > 0]
            self.max_context = min(lim) if lim else None
        self._route_spec = None
        if cfg.router_scoring == "sigmoid":  # DeepSeek-style group-limited routing (glm4_moe)
            from types import SimpleNamespace
            self._route_spec = SimpleNamespace(
                scoring_func="sigmoid", topk_method="noaux_tc", n_group=cfg.n_group, topk_group=cfg.topk_group,
                num_experts_per_tok=cfg.num_experts_per_tok, norm_topk_prob=cfg.norm_topk_prob,
                routed_scaling_factor=cfg.routed_scaling_factor)

    # -- weights ----------------------------------------------------------------
    def _load(self, w):
        c, dev, bf = self.cfg, self.device, torch.bfloat16
        if c.model_type in ("mixtral", "minimax_m2"):  # block_sparse_moe.* names -> the canonical MoE names
            from ..weights.aliases import CanonicalView
            w = CanonicalView(w, c.model_type)
        elif c.model_type == "llama4_text":  # feed_forward.* names, fused expert banks
            from ..weights.aliases import Llama4View
            w = Llama4View(w)

        def g(name):
            return self._get(w, name)

        def dv(t):
            return t.to(device=dev, dtype=bf).contiguous()

        self.embed = dv(g("model.embed_tokens.weight"))
        self.norm = dv(g("model.norm.weight"))
        self.lm_head = self.embed if c.tie_word_embeddings else dv(g("lm_head.weight"))
        D = c.head_dim
        self.layers, self.moe = [], []
        lo, hi = self.e_lo, self.e_lo + self.e_local
        for i in range(c.num_hidden_layers):
            p = f"model.layers.{i}."
            L = LayerWeights()
            L.ln1 = dv(g(p + "input_layernorm.weight"))
            L.ln2 = dv(g(p + "post_attention_layernorm.weight"))
            L.wqkv = dv(torch.cat([g(p + f"self_attn.{n}_proj.weight").to(dev) for n in "qkv"], 0))
            if c.rope_interleaved:
                # RoPE on interleaved pairs (2j, 2j+1) == half-split RoPE on q / k rows reordered
                # [0, 2, .., D-2, 1, 3, .., D-1] per head (attention scores are unchanged)
                perm = torch.cat([torch.arange(0, D, 2), torch.arange(1, D, 2)]).to(dev)
                nq, nk = c.num_attention_heads, c.num_key_value_heads
                rows = torch.cat([(h * D + perm) for h in range(nq + nk)] +
                                 [torch.arange((nq + nk) * D, L.wqkv.shape[0], device=dev)])
                L.wqkv = L.wqkv.index_select(0, rows).contiguous()
            L.bqkv = dv(torch.cat([g(p + f"self_attn.{n}_proj.bias").to(dev) for n in "qkv"])) \
                if c.attention_bias else None
            if c.qk_norm:
                L.q_norm = dv(g(p + "self_attn.q_norm.weight"))
                L.k_norm = dv(g(p + "self_attn.k_norm.weight"))
            elif c.qk_l2_norm and c.uses_rope(i):  # weightless RMS norm (it commutes with the rotation)
                L.q_norm = L.k_norm = torch.ones(D, dtype=bf, device=dev)
            else:
                L.q_norm = L.k_norm = None
            L.wo = dv(g(p + "self_attn.o_proj.weight"))
            ob = p + "self_attn.o_proj.bias"
            L.bo = dv(g(ob)) if (ob in w) else None
            L.bqkv = L.bqkv if c.attention_bias else None
            L.w_gu = L.wd = None
            L.sinks = g(p + "self_attn.sinks").to(dev, torch.float32).contiguous() if c.attn_sinks else None
            L.window = c.layer_window(i)
            L.inv_freq, L.rope_mult = self.inv_freq, self.rope_mult
            if not c.uses_rope(i):  # Llama-4 NoPE layer: zero frequencies rotate nothing
                L.inv_freq = torch.zeros_like(self.inv_freq)
            L.ln_post_attn = L.ln_post_ffn = None
            self.layers.append(L)
            if not c.is_moe_layer(i):  # dense layer of a mostly-MoE model (glm4_moe's first layers)
                L.w_gu = dv(ops.interleave_gate_up(g(p + "mlp.gate_proj.weight").to(dev),
                                                   g(p + "mlp.up_proj.weight").to(dev)))
                L.wd = dv(g(p + "mlp.down_proj.weight"))
                self.moe.append(None)
                continue
            M = MoELayer()
            M.router_corr = None
            pe = p + "mlp.experts."
            E_l = hi - lo
            if c.model_type != "gpt_oss":
                # qwen3-moe: router "mlp.gate", per-expert gate/up/down, no biases; experts are
                # packed to MXFP4 at load (the grouped GEMM streams 4-bit weights)
                M.router_w = dv(g(p + "mlp.gate.weight"))
                M.router_b = None
                if c.router_scoring == "sigmoid":  # fp32 router (as HF) + the choice-only correction bias
                    M.router_w = g(p + "mlp.gate.weight").to(dev, torch.float32).contiguous()
                    M.router_corr = g(p + "mlp.gate.e_score_correction_bias").to(dev, torch.float32)
                I = c.moe_intermediate_size
                gu_l, dn_l = [], []
                for e in range(lo, hi):
                    gt = g(pe + f"{e}.gate_proj.weight").to(dev).float()
                    up = g(pe + f"{e}.up_proj.weight").to(dev).float()
                    # [64 gate rows][64 up rows] per 128-row tile, like hf_interleaved_to_grouped's output
                    gu_l.append(torch.stack([gt.view(I // GROUP, GROUP, -1), up.view(I // GROUP, GROUP, -1)], 1)
                                .reshape(2 * I, -1))
                    dn_l.append(g(pe + f"{e}.down_proj.weight").to(dev).float())
                gub, gus = quantize_mxfp4(torch.stack(gu_l))
                dnb, dns = quantize_mxfp4(torch.stack(dn_l))
                M.gu_w, M.gu_exp = tile_mxfp4(gub, gus)
                M.dn_w, M.dn_exp = tile_mxfp4(dnb, dns)
                M.gu_bias = M.dn_bias = None
                M.sh_gu = M.sh_dn = M.sh_gate = None
                if c.n_shared_experts:  # glm4_moe / DeepSeek shared experts: dense, ungated, every token
                    ps = p + "mlp.shared_experts."
                    M.sh_gu = dv(ops.interleave_gate_up(g(ps + "gate_proj.weight"), g(ps + "up_proj.weight")))
                    M.sh_dn = dv(g(ps + "down_proj.weight"))
                elif c.shared_expert_intermediate_size:  # qwen2-moe shared expert (dense, sigmoid-gated)
                    ps = p + "mlp.shared_expert."
                    M.sh_gu = dv(ops.interleave_gate_up(g(ps + "gate_proj.weight"), g(ps + "up_proj.weight")))
                    M.sh_dn = dv(g(ps + "down_proj.weight"))
                    M.sh_gate = g(p + "mlp.shared_expert_gate.weight").to(dev, torch.float32)
                self.moe.append(M)
                continue
            M.router_w = dv(g(p + "mlp.router.weight"))
            M.router_b = dv(g(p + "mlp.router.bias"))
            if (pe + "gate_up_proj_blocks") in w:
                gub = g(pe + "gate_up_proj_blocks")[lo:hi]
                gus = g(pe + "gate_up_proj_scales")[lo:hi]
                dnb = g(pe + "down_proj_blocks")[lo:hi]
                dns = g(pe + "down_proj_scales")[lo:hi]
            else:  # bf16 checkpoint: quantize to MXFP4 at load ([E, in, out] -> [E, out, in])
                gub, gus = quantize_mxfp4(g(pe + "gate_up_proj")[lo:hi].to(dev).float().transpose(1, 2))
                dnb, dns = quantize_mxfp4(g(pe + "down_proj")[lo:hi].to(dev).float().transpose(1, 2))
            M.gu_w, M.gu_exp = tile_mxfp4(hf_interleaved_to_grouped(gub.to(dev).reshape(E_l, gub.shape[1], -1)),
                                hf_interleaved_to_grouped(gus.to(dev).reshape(E_l, gus.shape[1], -1)))
            M.gu_bias = hf_interleaved_to_grouped(dv(g(pe + "gate_up_proj_bias")[lo:hi]))
            M.dn_w, M.dn_exp = tile_mxfp4(dnb.to(dev), dns.to(dev).reshape(E_l, dns.shape[1], -1))
            M.dn_bias = dv(g(pe + "down_proj_bias")[lo:hi])  # each expert (and its bias) lives on one rank
            M.sh_gu = M.sh_dn = M.sh_gate = None
            self.moe.append(M)

    # -- forward ---------------------------------------------------------------
    def _moe(self, i: int, x: torch.Tensor, h: torch.Tensor, norm_w: torch.Tensor) -> torch.Tensor:
        """Routed expert block on the normalised input ``x``: ``h += moe(x)``;
        returns ``rmsnorm(h) * norm_w`` for the next layer."""
        c = self.cfg
        M = self.moe[i]
        T, H = x.shape
        k = c.num_experts_per_tok
        E_l = self.e_local
        dev = x.device
        x_in = x
        if self._route_spec is not None:
            from .deepseek import route
            idx, wts = route(self._route_spec, x.float() @ M.router_w.t(), M.router_corr)
            experts, weights = idx.to(torch.int32).contiguous(), wts.contiguous()
        elif c.router_scoring == "llama4":  # top-1 on the logits; the expert sees x * sigmoid(logit)
            logits = ops.linear(x, M.router_w, out_dtype=torch.float32)
            topv, topi = logits.topk(k, -1)
            experts = topi.to(torch.int32).contiguous()
            weights = torch.ones_like(topv)
            x_in = (x.float() * torch.sigmoid(topv)).to(x.dtype)
        else:
            logits = ops.linear(x, M.router_w, bias=M.router_b, out_dtype=torch.float32)
            experts = torch.empty(T, k, dtype=torch.int32, device=dev)
            weights = torch.empty(T, k, dtype=torch.float32, device=dev)
            ext().moe_route(logits, k, not c.softmax_after_topk, c.norm_topk_prob, experts, weights)
        n = T * k
        bt = token_tile(n, c.num_experts)
        meta = torch.empty(2 * E_l + 2, dtype=torch.int32, device=dev)
        max_tiles = n // bt + E_l + 1
        tiles = torch.empty(4 * max_tiles, dtype=torch.int32, device=dev)
        perm = torch.empty(n, dtype=torch.int32, device=dev)
        inv = torch.empty(n, dtype=torch.int32, device=dev)
        cursor = torch.empty(E_l, dtype=torch.int32, device=dev)
        fused = self.combiner is not None and self.combiner.fits(T)
        if fused:
            dn, inv = self.combiner.slots(n)  # symmetric slots the peers read
        ext().moe_align(experts, E_l, self.e_lo, E_l, bt, meta, tiles, perm, inv, cursor)
        a = torch.empty(n, H, dtype=torch.float16, device=dev)  # grouped GEMM operands are f16
        ext().moe_gather(x_in, perm, meta, E_l, k, a)
        I = c.moe_intermediate_size
        s = scratch(dev)
        gu = torch.empty(n, I, dtype=torch.float16, device=dev)
        gpt_oss = c.model_type == "gpt_oss"
        ext().moe_gemm(a, M.gu_w, M.gu_exp, 2 * I, M.gu_bias, None, perm, meta, tiles, gu, True,
                       float(c.swiglu_limit or 1e30), float(c.swiglu_alpha) if gpt_oss else 1.0, bt, s.status,
                       1.0 if gpt_oss else 0.0)
        if not fused:
            dn = torch.empty(n, H, dtype=torch.bfloat16, device=dev)
        ext().moe_gemm(gu, M.dn_w, M.dn_exp, H, M.dn_bias, weights.view(-1), perm, meta, tiles, dn, False,
                       0.0, 0.0, bt, s.status)
        ops._count(6)
        if M.sh_gu is not None and M.sh_gate is None:  # ungated shared experts: h += shared(x)
            ops.linear(ops.linear_swiglu(x, M.sh_gu), M.sh_dn, residual=h, out=h)
        elif M.sh_gu is not None:  # shared expert: every token; each rank adds it to its replicated residual
            sh = ops.linear(ops.linear_swiglu(x, M.sh_gu), M.sh_dn)
            gate = torch.sigmoid(x.float() @ M.sh_gate.t())
            h.add_((sh.float() * gate).to(h.dtype))
        if fused:
            return self.combiner.combine_norm(experts, h, norm_w)
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        ext().moe_combine(dn, inv, k, out, False)
        ops._count(1)
        if self.ep_size > 1 and not self._ep_local_only:
            dist.all_reduce(out)
        return ops.rmsnorm(out, norm_w, c.rms_norm_eps, residual=h, residual_out=h)  # h += moe; norm

    def forward_hidden(self, fb, kv) -> torch.Tensor:
        c = self.cfg
        h = ops.embedding(fb.input_ids, self.embed)
        x = ops.rmsnorm(h, self.layers[0].ln1, c.rms_norm_eps)
        n = len(self.layers)
        for i, L in enumerate(self.layers):
            a = self._attention(i, L, x, fb, kv)
            if a.shape[0] <= ops.ACC_MAX_M:  # decode: accumulate-only GEMM, bias + residual + norm in one kernel
                x = ops.add_rmsnorm_acc(ops.linear_acc(a, L.wo), h, L.ln2, c.rms_norm_eps, bias=L.bo)
            else:
                ops.linear(a, L.wo, bias=L.bo, residual=h, out=h)  # h += o_proj (+ bias)
                x = ops.rmsnorm(h, L.ln2, c.rms_norm_eps)
            nw = self.layers[i + 1].ln1 if i + 1 < n else self.norm
            if self.moe[i] is None:  # dense layer
                ops.linear(ops.linear_swiglu(x, L.w_gu), L.wd, residual=h, out=h)
                x = ops.rmsnorm(h, nw, c.rms_norm_eps)
            else:
                x = self._moe(i, x, h, nw)  # h += moe; x = rmsnorm(h) * nw
        return x
