"""GPU decoder (Qwen3 / Llama / Qwen2 dense families) on the sm_100a kernels.

One generic decoder driven by :class:`~rlx_models_b200.config.DecoderConfig`,
the B200 counterpart of the reference's `DecoderSpec` builder
(rlx-models-core src/standard_decoder.rs:172-312, `build_standard_decoder_packed`
:12210) and the Qwen3 flow (rlx-qwen3 src/flow.rs:310-434 prefill,
:558-690 decode). Weights are re-laid out once at load for the kernels:

* q/k/v fused into one [q + 2kv, H] matrix (one GEMM, one TMA stream),
* gate/up interleaved in groups of 64 rows so the GEMM epilogue applies SwiGLU,
* o_proj / down_proj GEMMs add the residual in their epilogue (in place).

A forward step works on a flat token batch: ``num_decode`` single-token decode
sequences first, then chunked-prefill segments, all sharing the GEMMs; the
attention kernels read/write the paged cache. Tensor parallelism shards heads
and the MLP intermediate dimension; the partial o/down outputs are combined by
the communicator (``comm``) — by the fused GEMM+reduce kernels over NVLink
peer memory, or NCCL as the baseline.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .. import ops
from ..utils.trace import inspect, inspecting, nvtx
from ..config import DecoderConfig
from ..ops import interleave_gate_up, rope_inv_freq
from ..runtime.kv_cache import PagedKVCache


@dataclass
class ForwardBatch:
    """Device tensors describing one engine step."""
    input_ids: torch.Tensor        # [T] int32
    positions: torch.Tensor        # [T] int32
    slots: torch.Tensor            # [T] int64 cache slot per token
    num_decode: int                # first num_decode tokens are decode tokens (1 per sequence)
    dec_block_tables: torch.Tensor | None = None  # [Bd, maxb] int32
    dec_ctx_lens: torch.Tensor | None = None      # [Bd] int32 (incl. the new token)
    pre_block_tables: torch.Tensor | None = None  # [Bp, maxb] int32
    pre_ctx_lens: torch.Tensor | None = None      # [Bp] int32
    pre_cu_q: torch.Tensor | None = None          # [Bp + 1] int32 offsets into the prefill tokens
    pre_max_q: int = 0
    logit_rows: torch.Tensor | None = None        # [R] int64 rows needing logits
    seq_slots: torch.Tensor | None = None         # [Bd + Bp] int32 state slot per sequence (stateful models)
    pre_cu_host: list | None = None               # host copy of pre_cu_q (lets a TP model split the step)
    mm_rows: torch.Tensor | None = None           # [n] int64 token rows whose input embedding is replaced
    mm_embeds: torch.Tensor | None = None         # [n, H] their embeddings (image tokens of a VLM)

    @property
    def num_tokens(self) -> int:
        return int(self.input_ids.shape[0])


class LayerWeights:
    __slots__ = ("ln1", "ln2", "wqkv", "bqkv", "q_norm", "k_norm", "wo", "bo", "w_gu", "wd", "sinks", "window",
                 "ln_post_attn", "ln_post_ffn", "inv_freq", "rope_mult")


class DecoderLM:
    def __init__(self, cfg: DecoderConfig, weights, device: torch.device | str = "cuda",
                 tp_rank: int = 0, tp_size: int = 1, comm=None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.tp_rank, self.tp_size, self.comm = tp_rank, tp_size, comm
        c = cfg
        assert c.num_attention_heads % tp_size == 0 and c.num_key_value_heads % tp_size == 0
        self.hq = c.num_attention_heads // tp_size
        self.hkv = c.num_key_value_heads // tp_size
        self.D = c.head_dim
        self.inter = c.intermediate_size // tp_size
        assert self.inter % ops.SWIGLU_GROUP == 0
        inv, mult = rope_inv_freq(c.rotary_dim, c.rope_theta, c.rope_scaling, c.max_position_embeddings)
        self.inv_freq = inv.to(self.device)
        self.rope_mult = mult
        self.scale = c.attention_multiplier or 1.0 / math.sqrt(c.head_dim)
        self.glu_act = 1 if c.mlp_act == "gelu_tanh" else 0  # GeGLU (Gemma) in the gated GEMM epilogue
        self.local_rope = None
        if c.rope_local_theta:  # sliding-window layers with their own RoPE base (Gemma-3)
            li, lm = rope_inv_freq(c.rotary_dim, c.rope_local_theta, None, c.max_position_embeddings)
            self.local_rope = (li.to(self.device), lm)
        if c.sandwich_norm and tp_size > 1:
            raise NotImplementedError("sandwich-norm (Gemma-2/3) decoders run with tp_size 1")
        if c.qk_norm_full and tp_size > 1:
            raise NotImplementedError("full-width QK-norm (MiniMax-M2) needs every head of a token: tp_size 1")
        self._load(weights)

    # -- weights ---------------------------------------------------------------
    def _get(self, w, name):
        t = w.take(name) if hasattr(w, "take") else w[name]
        return t

    def _rows(self, t: torch.Tensor, per_rank: int, rank_parts: int = 1) -> torch.Tensor:
        """Rank slice of dim 0 (column-parallel)."""
        return t.narrow(0, self.tp_rank * per_rank, per_rank)

    def _cols(self, t: torch.Tensor, per_rank: int) -> torch.Tensor:
        """Rank slice of dim 1 (row-parallel)."""
        return t.narrow(1, self.tp_rank * per_rank, per_rank)

    def _load(self, w):
        c, dev, bf = self.cfg, self.device, torch.bfloat16
        D = self.D

        def g(name):
            return self._get(w, name)

        def dv(t):
            return t.to(device=dev, dtype=bf).contiguous()

        from ..weights.aliases import FusedSplitView
        if FusedSplitView.needed(w):  # Phi-3: fused qkv_proj / gate_up_proj
            w = FusedSplitView(w, c.q_size, c.kv_size, c.intermediate_size)
        rm = c.residual_multiplier

        def dv_res(t):  # Granite: the residual multiplier folds into o_proj / down_proj
            return dv(t.to(dev).float() * rm) if rm != 1.0 else dv(t)

        def dv_norm(t):  # Gemma norms compute x * (1 + w): fold the offset at load
            return dv(t.to(dev).float() + 1.0) if c.norm_unit_offset else dv(t)

        self.embed = dv(g("model.embed_tokens.weight"))
        self.norm = dv_norm(g("model.norm.weight"))
        if c.tie_word_embeddings:
            head = self.embed
        else:
            head = dv(g("lm_head.weight"))
        V = c.vocab_size
        if self.tp_size > 1:
            assert V % self.tp_size == 0
            self.lm_head = head.narrow(0, self.tp_rank * (V // self.tp_size), V // self.tp_size).contiguous()
        else:
            self.lm_head = head
        self.layers: list[LayerWeights] = []
        for i in range(c.num_hidden_layers):
            p = f"model.layers.{i}."
            L = LayerWeights()
            L.ln1 = dv_norm(g(p + "input_layernorm.weight"))
            L.ln_post_attn = L.ln_post_ffn = None
            if c.sandwich_norm:  # pre-MLP norm is pre_feedforward_layernorm; post_attention_layernorm follows attention
                L.ln2 = dv_norm(g(p + "pre_feedforward_layernorm.weight"))
                L.ln_post_attn = dv_norm(g(p + "post_attention_layernorm.weight"))
                L.ln_post_ffn = dv_norm(g(p + "post_feedforward_layernorm.weight"))
            else:
                L.ln2 = dv_norm(g(p + "post_attention_layernorm.weight"))
            q = self._rows(g(p + "self_attn.q_proj.weight"), self.hq * D)
            k = self._rows(g(p + "self_attn.k_proj.weight"), self.hkv * D)
            v = self._rows(g(p + "self_attn.v_proj.weight"), self.hkv * D)
            L.wqkv = dv(torch.cat([q.to(dev), k.to(dev), v.to(dev)], 0))
            L.bqkv = None
            if c.attention_bias:
                qb = self._rows(g(p + "self_attn.q_proj.bias"), self.hq * D)
                kb = self._rows(g(p + "self_attn.k_proj.bias"), self.hkv * D)
                vb = self._rows(g(p + "self_attn.v_proj.bias"), self.hkv * D)
                L.bqkv = dv(torch.cat([qb.to(dev), kb.to(dev), vb.to(dev)]))
            L.q_norm = dv_norm(g(p + "self_attn.q_norm.weight")) if c.qk_norm else None
            L.k_norm = dv_norm(g(p + "self_attn.k_norm.weight")) if c.qk_norm else None
            L.wo = dv_res(self._cols(g(p + "self_attn.o_proj.weight"), self.hq * D))
            L.bo = None
            gt = self._rows(g(p + "mlp.gate_proj.weight"), self.inter)
            up = self._rows(g(p + "mlp.up_proj.weight"), self.inter)
            L.w_gu = interleave_gate_up(gt.to(dev, bf), up.to(dev, bf))
            L.wd = dv_res(self._cols(g(p + "mlp.down_proj.weight"), self.inter))
            L.sinks = None
            L.window = c.layer_window(i)
            L.inv_freq, L.rope_mult = (self.local_rope if self.local_rope is not None and L.window > 0
                                       else (self.inv_freq, self.rope_mult))
            self.layers.append(L)

    def enable_kv_retrieval(self, num_blocks: int, **kw):
        """Long-context decode over a bounded set of retrieved KV blocks
        (runtime/kv_retrieval.py); kw: topk_blocks, window_blocks, sink_blocks."""
        from ..runtime.kv_retrieval import KVRetrieval
        if any(L.window for L in self.layers) or any(L.sinks is not None for L in self.layers):
            raise NotImplementedError("KV retrieval is for full-attention layers without sinks")
        self.retrieval = KVRetrieval(self.cfg.num_hidden_layers, num_blocks, self.hkv, self.D, self.device, **kw)

    kv_dtype = torch.bfloat16       # or torch.float8_e4m3fn (set_kv_cache_dtype)
    kv_scales = (1.0, 1.0)

    def set_kv_cache_dtype(self, dtype: str, scales: tuple = (1.0, 1.0)) -> None:
        """"bf16" or "fp8" (e4m3 pages holding value / scale; scales (k, v))."""
        if dtype not in ("bf16", "fp8"):
            raise ValueError(f"kv cache dtype {dtype!r}: 'bf16' or 'fp8'")
        if dtype == "fp8" and getattr(self, "retrieval", None) is not None:
            raise NotImplementedError("KV retrieval reads bf16 pages")
        self.kv_dtype = torch.float8_e4m3fn if dtype == "fp8" else torch.bfloat16
        self.kv_scales = (float(scales[0]), float(scales[1]))

    def kv_bytes_per_block(self) -> int:
        return PagedKVCache.bytes_per_block(self.cfg.num_hidden_layers, self.hkv, self.D,
                                            1 if self.kv_dtype == torch.float8_e4m3fn else 2)

    def make_kv_cache(self, num_blocks: int) -> PagedKVCache:
        return PagedKVCache(self.cfg.num_hidden_layers, num_blocks, self.hkv, self.D, self.device,
                            dtype=self.kv_dtype, scales=self.kv_scales)

    # -- forward ---------------------------------------------------------------
    def _attention(self, i: int, L: LayerWeights, x: torch.Tensor, fb: ForwardBatch, kv: PagedKVCache):
        T = x.shape[0]
        kc, vc = kv.layer(i)
        full = self.cfg.qk_norm_full
        acc = T <= ops.ACC_MAX_M and not full
        if acc:
            qkv = ops.linear_acc(x, L.wqkv)  # fp32 sums, consumed (and zeroed) by qkv_rope, which adds the bias
        else:
            qkv = ops.linear(x, L.wqkv, bias=L.bqkv)
        if full:  # MiniMax-M2: one RMSNorm over all q heads (and all k heads) of a token, in place
            qd, kd = self.hq * self.D, self.hkv * self.D
            ops.rmsnorm(qkv[:, :qd], L.q_norm, self.cfg.rms_norm_eps, out=qkv[:, :qd])
            ops.rmsnorm(qkv[:, qd:qd + kd], L.k_norm, self.cfg.rms_norm_eps, out=qkv[:, qd:qd + kd])
        f8 = kc.dtype == torch.float8_e4m3fn
        sc = kv.scales if f8 else (1.0, 1.0)
        q = ops.qkv_rope(qkv, num_q_heads=self.hq, num_kv_heads=self.hkv, head_dim=self.D,
                         positions=fb.positions, inv_freq=L.inv_freq, rope_scale=L.rope_mult,
                         rot_dim=self.cfg.rotary_dim,
                         q_norm=None if full else L.q_norm, k_norm=None if full else L.k_norm,
                         eps=self.cfg.rms_norm_eps, slots=fb.slots,
                         k_cache=kc, v_cache=vc, bias=L.bqkv if acc else None, kv_scales=sc)
        o = torch.empty_like(q)
        nd = fb.num_decode
        retrieval = getattr(self, "retrieval", None)
        if retrieval is not None:
            retrieval.update(i, kc, fb.slots)
        if nd > 0:
            tables, ctx = fb.dec_block_tables, fb.dec_ctx_lens
            if retrieval is not None:
                tables, ctx = retrieval.select(i, q[:nd], tables, ctx)
            ops.decode_attention(q[:nd], kc, vc, tables, ctx, scale=self.scale,
                                 sinks=L.sinks, window=L.window, out=o[:nd], softcap=self.cfg.attn_softcap,
                                 kv_scales=sc)
        if T > nd:
            pk, pv, ptab = kc, vc, fb.pre_block_tables
            if f8:  # prefill reads bf16 copies of its sequences' pages (after this step's writes)
                pk, pv, ptab = ops.kv_dequant_pages(kc, vc, fb.pre_block_tables, fb.pre_ctx_lens, sc)
            ops.prefill_attention(q[nd:], pk, pv, ptab, fb.pre_ctx_lens, fb.pre_cu_q,
                                  fb.pre_max_q, scale=self.scale, sinks=L.sinks, window=L.window, out=o[nd:],
                                  softcap=self.cfg.attn_softcap, causal=self.cfg.causal)
        return o.view(T, self.hq * self.D)

    def _layer(self, i: int, L: LayerWeights, x: torch.Tensor, h: torch.Tensor, fb: ForwardBatch, kv, comm,
               nw: torch.Tensor) -> torch.Tensor:
        """One decoder layer on the normed input ``x``; updates the residual
        ``h`` in place and returns rmsnorm(h) * nw for the next layer."""
        eps = self.cfg.rms_norm_eps
        a = self._attention(i, L, x, fb, kv)
        if L.ln_post_attn is not None:  # sandwich norms: h += norm(o_proj(a)); h += norm(mlp(norm(h)))
            y = ops.rmsnorm(ops.linear(a, L.wo), L.ln_post_attn, eps)
            x = ops.rmsnorm(y, L.ln2, eps, residual=h, residual_out=h)
            m = ops.linear(ops.linear_swiglu(x, L.w_gu, act=self.glu_act), L.wd)
            return ops.rmsnorm(ops.rmsnorm(m, L.ln_post_ffn, eps), nw, eps, residual=h, residual_out=h)
        x = comm.rowpar_add_norm(a, L.wo, h, L.ln2, bias=L.bo)
        if x.shape[0] <= ops.ACC_MAX_M:
            gu = ops.swiglu_acc(ops.linear_acc(x, L.w_gu), act=self.glu_act)
        else:
            gu = ops.linear_swiglu(x, L.w_gu, act=self.glu_act)
        return comm.rowpar_add_norm(gu, L.wd, h, nw)

    MB_MIN_TOKENS = 1024  # smallest step split into two overlapped micro-batches under TP

    def _microbatches(self, fb: ForwardBatch):
        """Split a prefill-heavy step into two sequence-disjoint micro-batches of
        about equal token counts (decode rows go with the first), or None."""
        cu = fb.pre_cu_host
        if (cu is None or len(cu) < 3 or fb.seq_slots is not None or fb.num_tokens < self.MB_MIN_TOKENS
                or getattr(self, "retrieval", None) is not None):
            return None
        nd, npf = fb.num_decode, len(cu) - 1
        half = (nd + cu[-1]) / 2
        k = min(range(1, npf), key=lambda j: abs(nd + cu[j] - half))
        tA = nd + cu[k]
        if tA <= ops.ACC_MAX_M or fb.num_tokens - tA <= ops.ACC_MAX_M:
            return None  # both halves must stay on the prefill (non-accumulating) paths
        qA = max(cu[j + 1] - cu[j] for j in range(k))
        qB = max(cu[j + 1] - cu[j] for j in range(k, npf))
        a = ForwardBatch(input_ids=fb.input_ids[:tA], positions=fb.positions[:tA], slots=fb.slots[:tA],
                         num_decode=nd, dec_block_tables=fb.dec_block_tables, dec_ctx_lens=fb.dec_ctx_lens,
                         pre_block_tables=fb.pre_block_tables[:k], pre_ctx_lens=fb.pre_ctx_lens[:k],
                         pre_cu_q=fb.pre_cu_q[:k + 1], pre_max_q=qA)
        b = ForwardBatch(input_ids=fb.input_ids[tA:], positions=fb.positions[tA:], slots=fb.slots[tA:],
                         num_decode=0, pre_block_tables=fb.pre_block_tables[k:], pre_ctx_lens=fb.pre_ctx_lens[k:],
                         pre_cu_q=fb.pre_cu_q[k:] - cu[k], pre_max_q=qB)
        return a, b

    def _forward_overlapped(self, a: ForwardBatch, b: ForwardBatch, kv, comm, comm_b) -> torch.Tensor:
        """Tensor-parallel prefill as two micro-batches on two streams with one
        communicator (process group) each: while one micro-batch's row-parallel
        all-reduce crosses NVLink, the other's GEMMs and attention run, layer by
        layer. The halves touch disjoint sequences (KV pages), so they need no
        ordering between them; each stream uses its own scratch set."""
        from ..ops._ext import scratch_slot
        main = torch.cuda.current_stream(self.device)
        side = getattr(self, "_side_stream", None)
        if side is None:
            side = self._side_stream = torch.cuda.Stream(self.device)
        side.wait_stream(main)
        n = len(self.layers)
        ha = comm.embed(a.input_ids, self.embed)
        xa = comm.norm_in(ha, self.layers[0].ln1)
        with torch.cuda.stream(side), scratch_slot(1):
            hb = comm_b.embed(b.input_ids, self.embed)
            xb = comm_b.norm_in(hb, self.layers[0].ln1)
        for i, L in enumerate(self.layers):
            nw = self.layers[i + 1].ln1 if i + 1 < n else self.norm
            with nvtx(f"layer{i}.mb0"):
                xa = self._layer(i, L, xa, ha, a, kv, comm, nw)
            with torch.cuda.stream(side), scratch_slot(1), nvtx(f"layer{i}.mb1"):
                xb = self._layer(i, L, xb, hb, b, kv, comm_b, nw)
        main.wait_stream(side)
        xb.record_stream(main)
        return torch.cat([xa, xb])

    def forward_hidden(self, fb: ForwardBatch, kv: PagedKVCache) -> torch.Tensor:
        """Returns the final-normed hidden states of every token ([T, H])."""
        comm = self.comm or LocalComm(self.cfg.rms_norm_eps)
        comm_b = getattr(comm, "microbatch_comm", None)
        if comm_b is not None and not inspecting() and fb.mm_rows is None:
            mbs = self._microbatches(fb)
            if mbs is not None:
                return self._forward_overlapped(mbs[0], mbs[1], kv, comm, comm_b)
        h = comm.embed(fb.input_ids, self.embed)
        if self.cfg.embedding_multiplier != 1.0:
            h.mul_(self.cfg.embedding_multiplier)
        if fb.mm_rows is not None:
            h.index_copy_(0, fb.mm_rows, fb.mm_embeds.to(h.dtype))
        x = comm.norm_in(h, self.layers[0].ln1)
        n = len(self.layers)
        for i, L in enumerate(self.layers):
            with nvtx(f"layer{i}"):
                x = self._layer(i, L, x, h, fb, kv, comm, self.layers[i + 1].ln1 if i + 1 < n else self.norm)
            if inspecting():
                inspect(f"layer{i}.residual", h)
        if inspecting():
            inspect("final_hidden", x)
        return x

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        """lm_head on final-normed rows (fp32; vocab-sharded under TP)."""
        logits = ops.linear(x, self.lm_head, out_dtype=torch.float32, alpha=1.0 / self.cfg.logits_scaling)
        cap = self.cfg.final_softcap
        if cap > 0:  # Gemma-2 final logit softcapping
            logits.div_(cap).tanh_().mul_(cap)
        return logits

    def forward(self, fb: ForwardBatch, kv: PagedKVCache) -> torch.Tensor:
        x = self.forward_hidden(fb, kv)
        if fb.logit_rows is not None:
            x = x.index_select(0, fb.logit_rows)
        return self.logits(x)


class LocalComm:
    """Single-GPU residual-stream ops (no communication)."""

    def __init__(self, eps: float):
        self.eps = eps

    def embed(self, ids, table):
        return ops.embedding(ids, table)

    def norm_in(self, h, w):
        return ops.rmsnorm(h, w, self.eps)

    def rowpar_add_norm(self, x, w, h, norm_w, bias=None):
        """h += x @ w.T (+ bias); returns rmsnorm(h) * norm_w.

        Decode-sized batches: accumulate-only GEMM + one add+RMSNorm kernel that
        consumes the fp32 sums; larger batches: residual add in the GEMM epilogue."""
        if x.shape[0] <= ops.ACC_MAX_M:
            return ops.add_rmsnorm_acc(ops.linear_acc(x, w), h, norm_w, self.eps, bias=bias)
        ops.linear(x, w, bias=bias, residual=h, out=h)
        return ops.rmsnorm(h, norm_w, self.eps)
