"""Functional wrappers over the sm_100a kernels.

Every function here launches one of this package's own CUDA kernels on the
current stream; none falls back to a torch/cuBLAS implementation. The fp32
CPU restatements used as test oracles live in :mod:`rlx_models_b200.ops.reference`.
"""
from __future__ import annotations

import math

import torch

from ._ext import KernelError, available, check_errors, ext, launch_count, scratch
from ._ext import count_launches as _count

__all__ = [
    "linear", "linear_swiglu", "rmsnorm", "qkv_rope", "embedding", "decode_attention",
    "prefill_attention", "argmax", "sample", "interleave_gate_up", "rope_inv_freq",
    "check_errors", "KernelError", "available",
]

SWIGLU_GROUP = 64  # gate/up rows interleaved in groups of 64 for the fused epilogue


def linear(x: torch.Tensor, w: torch.Tensor, *, out: torch.Tensor | None = None,
           residual: torch.Tensor | None = None, bias: torch.Tensor | None = None,
           alpha: float = 1.0, out_dtype: torch.dtype = torch.bfloat16,
           swap: int = -1, bn: int = 0, splits: int = 0, gelu_from: int = -1, relu: bool = False,
           gate: torch.Tensor | None = None, gate_rows: tuple = (0, 1, 1)) -> torch.Tensor:
    """``out = alpha * x @ w.T (+ bias) (+ residual)`` on the tcgen05 GEMM.

    x: [M, K] bf16, w: [N, K] bf16 (nn.Linear layout). ``out_dtype`` bf16 or f32.
    DiT epilogues: ``gelu_from`` >= 0 applies GELU (tanh) to output columns
    >= gelu_from; ``gate`` [batches, N] multiplies the (biased) product before
    the residual add, row i using gate row ``i // r1`` below ``split`` and
    ``(i - split) // r2`` above, with ``gate_rows = (split, r1, r2[, row offset added to i])``.
    """
    M, N = x.shape[0], w.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype, device=x.device)
    s = scratch(x.device)
    mode = 1 if out.dtype == torch.float32 else 0
    _count(1)
    act_from = (1 << 30) if relu else int(gelu_from)
    ext().linear(x, w, out, mode, residual, bias, float(alpha), s.gemm_ws, s.gemm_sem, s.status,
                 swap, bn, splits, None, act_from, gate, int(gate_rows[0]), int(gate_rows[1]),
                 int(gate_rows[2]), int(gate_rows[3]) if len(gate_rows) > 3 else 0)
    return out


_DENSE_Q_CACHE: dict = {}


def linear_mxfp4(x: torch.Tensor, w_tiled: torch.Tensor, row_exp: torch.Tensor, n_out: int,
                 bias: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ dequant(W).T (+ bias)`` with W stored as MXFP4 in the grouped-GEMM
    tile layout (``quant.mxfp4.tile_mxfp4`` of one expert, [1, NT, KT, 4352]):
    the dense weight-only 4-bit linear runs on the grouped kernel with a single
    expert (f16 operands, E2M1 expanded into TMEM). x [T, K] bf16 -> [T, N] bf16."""
    T, K = x.shape
    dev = x.device
    bt = 32 if T <= 32 else (64 if T <= 64 else 128)
    key = (dev, T, bt)
    st = _DENSE_Q_CACHE.get(key)
    if st is None:
        ntile = (T + bt - 1) // bt
        meta = torch.tensor([ntile, T, 0, T], dtype=torch.int32, device=dev)  # tiles, count[0], offs[0..1]
        info = torch.tensor([[0, m, m * bt, min(bt, T - m * bt)] for m in range(ntile)], dtype=torch.int32,
                            device=dev).reshape(-1)
        perm = torch.arange(T, dtype=torch.int32, device=dev)
        st = _DENSE_Q_CACHE[key] = (meta, info, perm)
    meta, info, perm = st
    a = torch.empty(T, K, dtype=torch.float16, device=dev)
    ext().moe_gather(x, perm, meta, 1, 1, a)
    if out is None:
        out = torch.empty(T, n_out, dtype=torch.bfloat16, device=dev)
    _count(2)
    ext().moe_gemm(a, w_tiled, row_exp, n_out, bias, None, perm, meta, info, out, False, 0.0, 0.0, bt,
                   scratch(dev).status)
    return out


def linear_swiglu(x: torch.Tensor, w_gu: torch.Tensor, *, out: torch.Tensor | None = None,
                  swap: int = -1, bn: int = 0, splits: int = 0, act: int = 0) -> torch.Tensor:
    """``silu(x @ Wg.T) * (x @ Wu.T)`` with ``w_gu = interleave_gate_up(Wg, Wu)``;
    ``act=1``: GELU (tanh form) on the gate instead (GeGLU)."""
    M, N = x.shape[0], w_gu.shape[0]
    if out is None:
        out = torch.empty(M, N // 2, dtype=torch.bfloat16, device=x.device)
    s = scratch(x.device)
    _count(1)
    ext().linear(x, w_gu, out, 2, None, None, 1.0, s.gemm_ws, s.gemm_sem, s.status, swap, bn, splits,
                 glu_act=int(act))
    return out


def matmul(a: torch.Tensor, b: torch.Tensor, *, out: torch.Tensor | None = None, out_dtype=torch.bfloat16,
           accumulate: bool = False, alpha: float = 1.0, residual: torch.Tensor | None = None,
           bias: torch.Tensor | None = None, static_b: bool = False) -> torch.Tensor:
    """``out (+)= alpha * a @ b`` on the tcgen05 GEMM; ``a`` [M, K] and ``b`` [K, N]
    may each be row-major or a transposed view (training: dX = dY @ W uses a
    row-major ``b``; dW = dY.T @ X a transposed ``a``). ``static_b`` lets the
    kernel prefetch ``b`` before the previous kernel finishes (weights only)."""
    if out is None:
        out = torch.empty(a.shape[0], b.shape[1], dtype=out_dtype, device=a.device)
    s = scratch(a.device)
    _count(1)
    ext().gemm(a, b, out, accumulate, float(alpha), residual, bias, static_b, s.gemm_ws, s.gemm_sem, s.status)
    return out


ACC_MAX_M = 128  # accumulate-only GEMM mode applies to decode-sized batches


def linear_acc(x: torch.Tensor, w: torch.Tensor, acc: torch.Tensor | None = None) -> torch.Tensor:
    """Accumulate-only GEMM: ``acc += x @ w.T`` in fp32 (split-K partials are
    added with red.add, no reduction tail). ``acc`` must be zero on entry
    unless a running sum is intended; consumers zero it after reading."""
    s = scratch(x.device)
    if acc is None:
        acc = s.acc_view(x.shape[0], w.shape[0])
    _count(1)
    ext().linear(x, w, acc, 3, None, None, 1.0, s.gemm_ws, s.gemm_sem, s.status, -1, 0, 0)
    return acc


def add_rmsnorm_acc(acc: torch.Tensor, h: torch.Tensor, w: torch.Tensor, eps: float,
                    out: torch.Tensor | None = None, bias: torch.Tensor | None = None) -> torch.Tensor:
    """h = bf16(h + bf16(acc (+ bias))); returns rmsnorm(h) * w; zeroes acc."""
    if out is None:
        out = torch.empty_like(h)
    _count(1)
    ext().add_rmsnorm_acc(acc, h, w, out, float(eps), bias)
    return out


def swiglu_acc(acc: torch.Tensor, out: torch.Tensor | None = None, act: int = 0) -> torch.Tensor:
    """SwiGLU (``act=1``: GeGLU) of interleaved gate/up fp32 sums [M, 2I] -> bf16 [M, I]; zeroes acc."""
    if out is None:
        out = torch.empty(acc.shape[0], acc.shape[1] // 2, dtype=torch.bfloat16, device=acc.device)
    _count(1)
    ext().swiglu_acc(acc, out, int(act))
    return out


def interleave_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor, group: int = SWIGLU_GROUP) -> torch.Tensor:
    """[I, K] x2 -> [2I, K] with rows [g*2G, g*2G+G) = gate, [g*2G+G, (g+1)*2G) = up."""
    I, K = w_gate.shape
    assert I % group == 0, "intermediate size must be a multiple of the SwiGLU group"
    g = w_gate.reshape(I // group, group, K)
    u = w_up.reshape(I // group, group, K)
    return torch.stack([g, u], dim=1).reshape(2 * I, K).contiguous()


def deinterleave_gate_up(w_gu: torch.Tensor, group: int = SWIGLU_GROUP):
    two_i, K = w_gu.shape
    v = w_gu.reshape(two_i // (2 * group), 2, group, K)
    return v[:, 0].reshape(-1, K), v[:, 1].reshape(-1, K)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, *, out: torch.Tensor | None = None,
            residual: torch.Tensor | None = None, residual_out: torch.Tensor | None = None) -> torch.Tensor:
    """``rmsnorm(x (+ residual)) * w``; with ``residual_out`` the sum is also stored."""
    if out is None:
        out = torch.empty_like(x)
    _count(1)
    ext().rmsnorm(x, w, out, float(eps), residual, residual_out)
    return out


def embedding(ids: torch.Tensor, table: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device)
    _count(1)
    ext().embedding(ids, table, out)
    return out


def rope_inv_freq(head_dim: int, theta: float, scaling: dict | None = None,
                  max_position: int | None = None) -> tuple[torch.Tensor, float]:
    """fp32 inverse frequencies (HF formula) and the cos/sin multiplier.

    Supports no scaling, ``linear``, ``llama3``, ``longrope`` / ``su`` and
    ``yarn`` (the last two return their attention factor).
    """
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    mult = 1.0
    if scaling:
        kind = scaling.get("rope_type", scaling.get("type", "default"))
        if kind == "linear":
            inv = inv / float(scaling["factor"])
        elif kind == "llama3":
            factor = float(scaling["factor"])
            lo = float(scaling.get("low_freq_factor", 1.0))
            hi = float(scaling.get("high_freq_factor", 4.0))
            old = float(scaling.get("original_max_position_embeddings", 8192))
            lo_wl, hi_wl = old / lo, old / hi
            wl = 2 * math.pi / inv
            smooth = (old / wl - lo) / (hi - lo)
            scaled = torch.where(wl > lo_wl, inv / factor, inv)
            mid = (1 - smooth) * scaled / factor + smooth * scaled
            is_mid = (wl >= hi_wl) & (wl <= lo_wl)
            inv = torch.where(is_mid, mid, scaled)
        elif kind in ("longrope", "su"):
            # per-dimension extension factors (Phi-3): the short factors; the long ones
            # replace them when ``scaling["use_long_factor"]`` is set
            old = float(scaling.get("original_max_position_embeddings", max_position or 4096))
            ext = scaling["long_factor"] if scaling.get("use_long_factor") else scaling["short_factor"]
            inv = inv / torch.tensor(ext, dtype=torch.float32)
            factor = float(scaling.get("factor") or (max_position or old) / old)
            if scaling.get("attention_factor") is not None:
                mult = float(scaling["attention_factor"])
            elif factor > 1.0:
                mult = math.sqrt(1 + math.log(factor) / math.log(old))
        elif kind == "yarn":
            factor = float(scaling["factor"])
            old = float(scaling.get("original_max_position_embeddings", max_position or 4096))
            beta_fast = float(scaling.get("beta_fast", 32.0))
            beta_slow = float(scaling.get("beta_slow", 1.0))

            def corr_dim(n_rot):
                return (head_dim * math.log(old / (n_rot * 2 * math.pi))) / (2 * math.log(theta))

            low = max(math.floor(corr_dim(beta_fast)), 0)
            high = min(math.ceil(corr_dim(beta_slow)), head_dim - 1)
            if scaling.get("truncate", True) is False:
                low, high = corr_dim(beta_fast), corr_dim(beta_slow)
            if low == high:
                high += 0.001
            ramp = (torch.arange(head_dim // 2, dtype=torch.float32) - low) / (high - low)
            ramp = ramp.clamp(0, 1)
            extrap = 1 - ramp
            inv = (inv / factor) * (1 - extrap) + inv * extrap
            def get_mscale(m=1.0):
                return 0.1 * m * math.log(factor) + 1.0 if factor > 1 else 1.0

            ms, ms_all = scaling.get("mscale"), scaling.get("mscale_all_dim")
            if scaling.get("attention_factor") is not None:
                mult = float(scaling["attention_factor"])
            elif ms and ms_all:  # DeepSeek: ratio of the two magnitudes (1 when they are equal)
                mult = get_mscale(float(ms)) / get_mscale(float(ms_all))
            else:
                mult = get_mscale()
    return inv.float(), mult


def qkv_rope(qkv: torch.Tensor, *, num_q_heads: int, num_kv_heads: int, head_dim: int,
             positions: torch.Tensor, inv_freq: torch.Tensor, rope_scale: float = 1.0,
             q_norm: torch.Tensor | None = None, k_norm: torch.Tensor | None = None, eps: float = 1e-6,
             slots: torch.Tensor | None = None, k_cache: torch.Tensor | None = None,
             v_cache: torch.Tensor | None = None, q_out: torch.Tensor | None = None,
             k_out: torch.Tensor | None = None, v_out: torch.Tensor | None = None,
             rot_dim: int = 0, bias: torch.Tensor | None = None, kv_scales: tuple = (1.0, 1.0)) -> torch.Tensor:
    """QK RMSNorm + RoPE on the fused qkv projection; K/V written to the paged cache.
    ``rot_dim`` (0 = head_dim): rotate only the first rot_dim dims of each head.
    ``bias`` (bf16) is added to an fp32 accumulate-mode ``qkv`` before rounding.
    float8_e4m3fn caches store saturate(value / scale) with ``kv_scales`` = (k, v)."""
    T = qkv.shape[0]
    if q_out is None:
        q_out = torch.empty(T, num_q_heads, head_dim, dtype=torch.bfloat16, device=qkv.device)
    _count(1)
    ext().qkv_rope(qkv, q_norm, k_norm, positions, slots, inv_freq, float(rope_scale), q_out, k_cache,
                   v_cache, k_out, v_out, num_q_heads, num_kv_heads, head_dim, float(eps), int(rot_dim), bias,
                   float(kv_scales[0]), float(kv_scales[1]))
    return q_out


def decode_attention(q, k_cache, v_cache, block_tables, ctx_lens, *, scale, sinks=None, window=0,
                     splits=0, out=None, softcap=0.0, kv_scales=(1.0, 1.0)):
    """Paged decode attention (one query per sequence); ``softcap`` > 0 caps
    the scaled scores at softcap * tanh(s / softcap)."""
    if out is None:
        out = torch.empty_like(q)
    s = scratch(q.device)
    _count(ext().decode_attention(q, k_cache, v_cache, block_tables, ctx_lens, out, sinks, int(window), float(scale),
                           int(splits), s.attn_ws, s.status, float(softcap), float(kv_scales[0]),
                           float(kv_scales[1])))
    return out


_DEQ_CACHE: dict = {}


def kv_dequant_pages(k_cache, v_cache, block_tables, ctx_lens, kv_scales=(1.0, 1.0)):
    """bf16 copies of the float8_e4m3fn pages a prefill batch reads: page p of
    sequence b goes to block b * max_blocks + p of the returned [B * max_blocks,
    Hkv, 16, D] caches, whose block table is returned with them (an arange).
    The buffers are reused across calls on a device (grown as needed)."""
    B, mb = block_tables.shape
    _, Hkv, _, D = k_cache.shape
    key = (k_cache.device, Hkv, D)
    st = _DEQ_CACHE.get(key)
    n = B * mb
    if st is None or st[0].shape[0] < n:
        cap = max(n, 2 * st[0].shape[0]) if st is not None else n
        st = _DEQ_CACHE[key] = (torch.empty(cap, Hkv, 16, D, dtype=torch.bfloat16, device=k_cache.device),
                                torch.empty(cap, Hkv, 16, D, dtype=torch.bfloat16, device=k_cache.device),
                                torch.arange(cap, dtype=torch.int32, device=k_cache.device))
    kb, vb, ar = st
    _count(1)
    ext().kv_dequant_pages(k_cache, v_cache, block_tables, ctx_lens, float(kv_scales[0]), float(kv_scales[1]),
                           kb, vb)
    return kb, vb, ar[:n].view(B, mb)


def prefill_attention(q, k_cache, v_cache, block_tables, ctx_lens, cu_q, max_q_len, *, scale, sinks=None,
                      window=0, out=None, causal=True, q_paged=False, softcap=0.0):
    """Causal prefill over paged K/V; ``causal=False`` lets every query see the
    whole context (DiT joint attention) and ``q_paged`` places query/output rows
    through the same block table as the keys (row = table[t // 16] * 16 + t % 16)."""
    if out is None:
        out = torch.empty_like(q)
    s = scratch(q.device)
    _count(1)
    ext().prefill_attention(q, k_cache, v_cache, block_tables, ctx_lens, cu_q, out, sinks, int(window),
                            float(scale), int(max_q_len), s.status, bool(causal), bool(q_paged), float(softcap))
    return out


def argmax(logits: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    _count(1)
    ext().argmax(logits, out)
    return out


def forward_tokens(ids: torch.Tensor, src: torch.Tensor, prev: torch.Tensor) -> torch.Tensor:
    """In place: ``ids[t] = prev[src[t]]`` where ``src[t] >= 0`` (int32). Decode
    rows scheduled before the previous step's tokens reached the host take
    their input token from that step's sampler output on the device."""
    _count(1)
    ext().forward_tokens(ids, src, prev)
    return ids


def instance_norm(x: torch.Tensor, gamma: torch.Tensor | None = None, beta: torch.Tensor | None = None, *,
                  active: int = 0, eps: float = 1e-5) -> torch.Tensor:
    """Instance norm of x [N, C, T] (fp32 / bf16) over time: statistics of the
    first ``active`` steps (all when 0), applied to every step, then per-channel
    affine ``gamma`` / ``beta`` (fp32 [C])."""
    y = torch.empty_like(x)
    _count(1)
    ext().instance_norm(x.contiguous(), gamma, beta, y, int(active), float(eps))
    return y


_ACTS = {None: 0, "snake": 1, "elu": 2, "gelu": 3}


def act_im2col(x: torch.Tensor, k: int, *, stride: int = 1, pad: int = 0, pad_right: int | None = None,
               dil: int = 1, act: str | None = None, alpha: torch.Tensor | None = None,
               reflect: bool = False) -> torch.Tensor:
    """Channels-last im2col with the preceding activation fused in: x [B, T, C]
    bf16 -> [B * T_out, round_up(k * C, 8)] bf16, column ``j * C + c`` of row
    ``(b, t)`` = act(x[b, t * stride - pad + j * dil, c]); positions outside the
    signal read zero, or the reflected sample when ``reflect``. ``act``: None,
    "snake" (``alpha`` fp32 [C]), "elu" or "gelu" (erf); padding columns are zero."""
    B, T, C = x.shape
    pr = pad if pad_right is None else pad_right
    T_out = (T + pad + pr - dil * (k - 1) - 1) // stride + 1
    cols = torch.empty(B * T_out, (k * C + 7) // 8 * 8, dtype=torch.bfloat16, device=x.device)
    _count(1)
    ext().act_im2col(x.contiguous(), alpha, cols, int(k), int(stride), int(pad), int(pr), int(dil), _ACTS[act],
                     bool(reflect))
    return cols


def convt_fold(Y: torch.Tensor, bias: torch.Tensor | None, c_out: int, *, stride: int, pad: int,
               pad_right: int | None = None) -> torch.Tensor:
    """Overlap-add of a transposed convolution computed as a GEMM: Y [B, T_in,
    k * C_out] fp32 (column ``j * C_out + o`` = tap j of output channel o) ->
    y [B, (T_in - 1) * stride + k - pad - pad_right, C_out] bf16 (the full
    output with ``pad`` samples cut on the left and ``pad_right`` on the right),
    plus ``bias`` fp32 [C_out]."""
    B, T_in, kc = Y.shape
    k = kc // c_out
    pr = pad if pad_right is None else pad_right
    y = torch.empty(B, (T_in - 1) * stride + k - pad - pr, c_out, dtype=torch.bfloat16, device=Y.device)
    _count(1)
    ext().convt_fold(Y.contiguous(), bias, y, int(stride), int(pad), int(pr))
    return y


def lstm_cell(G: torch.Tensor, c: torch.Tensor, h: torch.Tensor, y: torch.Tensor) -> None:
    """One LSTM step from accumulated gate pre-activations G [B, 4H] fp32
    (order i, f, g, o): updates c [B, H] fp32 in place and writes
    h = sig(o) tanh(c) in bf16 to ``h`` and ``y``."""
    _count(1)
    ext().lstm_cell(G, c, h, y)


def sample(logits, temperature, top_k, top_p, min_p, seeds, offsets, *, out=None, logprob=None):
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    _count(1)
    ext().sample(logits, temperature, top_k, top_p, min_p, seeds, offsets, out, logprob)
    return out


def gguf_dequant(raw: torch.Tensor, kind: str, shape, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """GGUF blocks (device uint8) -> dequantised tensor of ``shape`` (bf16 or
    fp32); F16 / BF16 payloads are converted with a cast."""
    from ..weights.gguf import GGML_TYPES, TYPE_ID
    tid = TYPE_ID[kind]
    _, be, bb = GGML_TYPES[tid]
    if kind in ("F16", "BF16"):
        src = raw.view(torch.float16 if kind == "F16" else torch.bfloat16)
        return src.to(dtype).view(*shape)
    n = 1
    for d in shape:
        n *= int(d)
    assert raw.numel() == n // be * bb, "gguf_dequant: byte count does not match the shape"
    out = torch.empty(*shape, dtype=dtype, device=raw.device)
    _count(1)
    ext().gguf_dequant(raw.contiguous(), tid, out)
    return out


def apply_penalties(logits: torch.Tensor, rows: list) -> torch.Tensor:
    """In place on fp32 ``logits`` [B, V]: per row ``(counts: dict[token, n],
    repetition, frequency, presence, bias: dict[token, value] | None)`` or
    None for an untouched row. Repetition scales x by 1/rep (x > 0) or rep
    for every listed token; frequency subtracts freq * n and presence pres
    for tokens with n > 0; bias adds."""
    B = logits.shape[0]
    off, ids, cnt, boff, bids, bval = [0], [], [], [0], [], []
    rep, freq, pres = [1.0] * B, [0.0] * B, [0.0] * B
    for r in range(B):
        row = rows[r] if r < len(rows) else None
        if row is not None:
            counts, rep[r], freq[r], pres[r], bias = row
            for t, n in counts.items():
                ids.append(int(t))
                cnt.append(int(n))
            for t, v in (bias or {}).items():
                bids.append(int(t))
                bval.append(float(v))
        off.append(len(ids))
        boff.append(len(bids))
    dev = logits.device

    def up(v, dt):
        return torch.tensor(v if v else [0], dtype=dt).pin_memory().to(dev, non_blocking=True)

    i32, f32 = torch.int32, torch.float32
    _count(1)
    ext().apply_penalties(logits, up(off, i32), up(ids, i32)[:len(ids)], up(cnt, i32)[:len(cnt)], up(rep, f32),
                          up(freq, f32), up(pres, f32), up(boff, i32), up(bids, i32)[:len(bids)],
                          up(bval, f32)[:len(bval)])
    return logits
