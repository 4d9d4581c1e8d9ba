"""Differentiable building blocks of the training path.

On CUDA every matmul (forward, dgrad, wgrad) runs on the tcgen05 GEMM and the
loss runs on the fused chunked lm_head + cross-entropy kernels; on CPU the same
functions fall back to plain fp32 torch so the host-side logic (FSDP sharding,
checkpointing, schedules) is testable on gloo ranks without a GPU.

Reference: the rlx-tune loss graph appends next-token CE to the LM graph
(rlx-tune src/lm.rs:77-115, src/loss.rs:20) and differentiates it with the
external autodiff crate; here autograd drives our kernels.
"""
from __future__ import annotations

import math

import torch

from .. import ops


def _cuda(t: torch.Tensor) -> bool:
    return t.is_cuda


class LinearFn(torch.autograd.Function):
    """y = x @ w.T with bf16 operands; dW in fp32."""

    @staticmethod
    def forward(ctx, x, w):
        ctx.save_for_backward(x, w)
        x2 = x.reshape(-1, x.shape[-1])
        if _cuda(x):
            y = ops.matmul(x2, w.t(), static_b=False)
        else:
            y = (x2.float() @ w.float().t()).to(x.dtype)
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x, w = ctx.saved_tensors
        x2 = x.reshape(-1, x.shape[-1])
        g2 = gy.reshape(-1, gy.shape[-1]).contiguous()
        dx = dw = None
        if _cuda(x):
            if ctx.needs_input_grad[0]:
                dx = ops.matmul(g2, w).view(x.shape)
            if ctx.needs_input_grad[1]:
                from .fsdp import push_target
                tgt = push_target(w)
                if tgt is not None:  # FSDP push: the GEMM adds dW into the owners' shards
                    fg, base = tgt
                    s = ops.scratch(w.device)
                    ops._count(1)
                    ops.ext().gemm_push_shards(g2.t(), x2, fg.push_table, base, fg.shard_n, 1.0, s.gemm_ws,
                                               s.gemm_sem, s.status)
                else:
                    dw = torch.empty(w.shape, dtype=torch.float32, device=w.device)
                    ops.matmul(g2.t(), x2, out=dw)
        else:
            if ctx.needs_input_grad[0]:
                dx = (g2.float() @ w.float()).to(x.dtype).view(x.shape)
            if ctx.needs_input_grad[1]:
                dw = g2.float().t() @ x2.float()
        return dx, dw


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return LinearFn.apply(x, w)


class LinearResidualFn(torch.autograd.Function):
    """y = residual + x @ w.T with the residual add in the GEMM epilogue; the
    residual's gradient is the output gradient itself."""

    @staticmethod
    def forward(ctx, x, w, residual):
        ctx.save_for_backward(x, w)
        x2 = x.reshape(-1, x.shape[-1])
        y = ops.matmul(x2, w.t(), static_b=False, residual=residual.reshape(-1, w.shape[0]).contiguous())
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, gy):
        dx, dw = LinearFn.backward(ctx, gy)
        return dx, dw, gy


def linear_residual(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
    """``residual + x @ w.T`` (one GEMM with the add fused on CUDA)."""
    if _cuda(x):
        return LinearResidualFn.apply(x, w, residual)
    return residual + LinearFn.apply(x, w)


class LMHeadCE(torch.autograd.Function):
    """Mean next-token cross-entropy of ``x @ w.T`` without materialising all
    logits: per chunk of rows, fp32 logits on the GEMM, one kernel for loss +
    dlogits, then dX and dW from dlogits. Gradients are computed in forward
    (the loss is the end of the graph) and scaled by grad_output in backward."""

    @staticmethod
    def forward(ctx, x, w, targets, chunk: int = 2048, denom: float | None = None):
        T, H = x.shape
        V = w.shape[0]
        # the trainer passes the global valid-target count as ``denom``; counting here
        # (a device read) only happens for direct calls without it
        n_valid = int((targets >= 0).sum()) if denom is None else None
        scale = 1.0 / (denom if denom is not None else max(1, n_valid))
        total = torch.zeros((), dtype=torch.float32, device=x.device)
        dx = torch.empty_like(x)
        dw = torch.zeros(V, H, dtype=torch.float32, device=x.device)
        for s in range(0, T, chunk):
            e = min(T, s + chunk)
            xc, tc = x[s:e], targets[s:e]
            if _cuda(x):
                logits = ops.matmul(xc, w.t(), out_dtype=torch.float32, static_b=False)
                loss = torch.empty(e - s, dtype=torch.float32, device=x.device)
                dlog = torch.empty(e - s, V, dtype=torch.bfloat16, device=x.device)
                ops.ext().ce_fwd_bwd(logits, tc, loss, dlog, float(scale))
                ops._count(1)
                del logits
                ops.matmul(dlog, w, out=dx[s:e])
                ops.matmul(dlog.t(), xc, out=dw, accumulate=True)
            else:
                logits = xc.float() @ w.float().t()
                valid = tc >= 0
                lse = torch.logsumexp(logits, -1)
                tgt = tc.clamp(min=0)
                loss = torch.where(valid, lse - logits.gather(1, tgt[:, None]).squeeze(1), torch.zeros_like(lse))
                p = torch.softmax(logits, -1)
                p[torch.arange(e - s), tgt] -= 1.0
                dlog = (p * valid[:, None].float() * scale).to(x.dtype)
                dx[s:e] = (dlog.float() @ w.float()).to(x.dtype)
                dw += dlog.float().t() @ xc.float()
            total += loss.sum()
        ctx.save_for_backward(dx, dw)
        return total * scale

    @staticmethod
    def backward(ctx, g):
        dx, dw = ctx.saved_tensors
        if _cuda(dx):
            # gradients were formed in forward: scale them in place by the incoming
            # loss gradient, read on the device (the kernels return at once when it is 1)
            gf = g.detach().float().reshape(1).contiguous()
            ops._count(2)
            ops.ext().scale_by(dx, gf)
            ops.ext().scale_by(dw, gf)
            return dx, dw, None, None, None
        return dx * g.to(dx.dtype), dw * g, None, None, None


def lm_head_ce(x, w, targets, chunk: int = 2048, denom: float | None = None):
    return LMHeadCE.apply(x, w, targets, chunk, denom)


def _rmsnorm_ref(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return w * y.to(x.dtype)


class RMSNormFn(torch.autograd.Function):
    """RMSNorm on the training kernels (``csrc/train/train_fused.cu``): forward
    saves the per-row rstd; backward gives dx and the fp32 weight gradient."""

    @staticmethod
    def forward(ctx, x, w, eps: float):
        xc = x.contiguous()
        y = torch.empty_like(xc)
        rows = xc.numel() // xc.shape[-1]
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        ops._count(1)
        ops.ext().rmsnorm_train_fwd(xc, w.contiguous(), y, rstd, float(eps))
        ctx.save_for_backward(xc, w, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        dx = torch.empty_like(x)
        dw = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        ops._count(1)
        ops.ext().rmsnorm_train_bwd(dy.contiguous(), x, w.contiguous(), rstd, dx, dw)
        return dx, dw, None


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """HF RMSNorm semantics (normalise in fp32, cast, scale); this package's
    kernels on CUDA for bf16 hidden sizes that are multiples of 2048."""
    if _cuda(x) and x.dtype == torch.bfloat16 and x.shape[-1] % 2048 == 0 and x.shape[-1] <= 8192:
        return RMSNormFn.apply(x, w, eps)
    return _rmsnorm_ref(x, w, eps)


class QKNormRopeFn(torch.autograd.Function):
    """q|k|v GEMM output [B, S, (Hq + 2 Hkv) * D] -> per-head RMSNorm of q and k
    (when norm weights are given) and rotary embedding, as q [B, S, Hq, D],
    k / v [B, S, Hkv, D]; one kernel each way (``csrc/train/train_fused.cu``)."""

    @staticmethod
    def forward(ctx, qkv, qn, kn, cos, sin, Hq: int, Hkv: int, eps: float):
        B, S, _ = qkv.shape
        D = 128
        qkv = qkv.contiguous()
        dev = qkv.device
        q = torch.empty(B, S, Hq, D, dtype=qkv.dtype, device=dev)
        k = torch.empty(B, S, Hkv, D, dtype=qkv.dtype, device=dev)
        v = torch.empty(B, S, Hkv, D, dtype=qkv.dtype, device=dev)
        rq = torch.empty(B * S * Hq, dtype=torch.float32, device=dev)
        rk = torch.empty(B * S * Hkv, dtype=torch.float32, device=dev)
        ops._count(1)
        ops.ext().qk_norm_rope_fwd(qkv, qn, kn, cos, sin, S, Hq, Hkv, float(eps), q, k, v, rq, rk)
        empty = torch.empty(0, device=dev)
        ctx.save_for_backward(qkv, qn if qn is not None else empty, kn if kn is not None else empty, cos, sin, rq, rk)
        ctx.meta = (S, Hq, Hkv, qn is not None)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        qkv, qn, kn, cos, sin, rq, rk = ctx.saved_tensors
        S, Hq, Hkv, normed = ctx.meta
        dqkv = torch.empty_like(qkv)
        dwq = torch.zeros(128, dtype=torch.float32, device=qkv.device) if normed else None
        dwk = torch.zeros(128, dtype=torch.float32, device=qkv.device) if normed else None
        ops._count(1)
        ops.ext().qk_norm_rope_bwd(qkv, qn if normed else None, kn if normed else None, cos, sin, S, Hq, Hkv, rq, rk,
                                   dq.contiguous(), dk.contiguous(), dv.contiguous(), dqkv, dwq, dwk)
        return dqkv, dwq, dwk, None, None, None, None, None


def qk_norm_rope(qkv, qn, kn, cos, sin, Hq: int, Hkv: int, D: int, eps: float):
    """Split the fused q|k|v projection, QK-norm (if ``qn``) and rotate; returns q, k, v [B, S, H, D]."""
    B, S, _ = qkv.shape
    if _cuda(qkv) and qkv.dtype == torch.bfloat16 and D == 128 and cos.shape[-1] == D:
        return QKNormRopeFn.apply(qkv, qn, kn, cos.contiguous(), sin.contiguous(), Hq, Hkv, eps)
    q, k, v = torch.split(qkv, [Hq * D, Hkv * D, Hkv * D], -1)
    q = q.reshape(B, S, Hq, D)
    k = k.reshape(B, S, Hkv, D)
    v = v.reshape(B, S, Hkv, D)
    if qn is not None:
        q = _rmsnorm_ref(q, qn, eps)
        k = _rmsnorm_ref(k, kn, eps)
    return rope(q, cos, sin), rope(k, cos, sin), v


class SwiGLUFn(torch.autograd.Function):
    """[..., 2I] = [gate | up] -> silu(gate) * up, one kernel each way."""

    @staticmethod
    def forward(ctx, gu):
        gu = gu.contiguous()
        h = torch.empty(*gu.shape[:-1], gu.shape[-1] // 2, dtype=gu.dtype, device=gu.device)
        ops._count(1)
        ops.ext().swiglu_train_fwd(gu, h)
        ctx.save_for_backward(gu)
        return h

    @staticmethod
    def backward(ctx, dh):
        (gu,) = ctx.saved_tensors
        dgu = torch.empty_like(gu)
        ops._count(1)
        ops.ext().swiglu_train_bwd(dh.contiguous(), gu, dgu)
        return dgu


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up over the [gate | up] halves of the last dimension."""
    if _cuda(gu) and gu.dtype == torch.bfloat16 and (gu.shape[-1] // 2) % 8 == 0:
        return SwiGLUFn.apply(gu)
    g, u = gu.chunk(2, dim=-1)
    return torch.nn.functional.silu(g) * u


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Half-split rotary embedding; x [B, S, H, D], cos/sin [S, R] (R < D:
    only the first R dims rotate)."""
    R = cos.shape[-1]
    if R < x.shape[-1]:
        return torch.cat([rope(x[..., :R], cos, sin), x[..., R:]], -1)
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos[None, :, None, :] + rot * sin[None, :, None, :]


_ATTN_META: dict = {}


def _attn_meta(B: int, S: int, dev):
    """Block tables / lengths / query offsets that view dense [B * S, H, D] K/V
    rows as 16-row pages of B sequences, for the tcgen05 attention kernel."""
    key = (B, S, dev)
    m = _ATTN_META.get(key)
    if m is None:
        nb = S // 16
        tables = (torch.arange(B, dtype=torch.int32)[:, None] * nb + torch.arange(nb, dtype=torch.int32)[None, :])
        m = _ATTN_META[key] = (tables.to(dev).contiguous(), torch.full((B,), S, dtype=torch.int32, device=dev),
                               (torch.arange(B + 1, dtype=torch.int32) * S).to(dev))
    return m


class AttentionFn(torch.autograd.Function):
    """Causal GQA attention on this package's kernels: the tcgen05 forward (it
    also saves each row's log-sum-exp) and the flash-style backward
    (``csrc/train/attn_bwd.cu``). q [B, S, Hq, 128], k / v [B, S, Hkv, 128]."""

    @staticmethod
    def forward(ctx, q, k, v):
        B, S, Hq, D = q.shape
        Hkv = k.shape[2]
        q3 = q.reshape(B * S, Hq, D).contiguous()
        k3 = k.reshape(B * S, Hkv, D).contiguous()
        v3 = v.reshape(B * S, Hkv, D).contiguous()
        out = torch.empty_like(q3)
        lse = torch.empty(B * S, Hq, dtype=torch.float32, device=q.device)
        tables, lens, cu = _attn_meta(B, S, q.device)
        scale = 1.0 / math.sqrt(D)
        s = ops.scratch(q.device)
        ops._count(1)
        ops.ext().attn_train_fwd(q3, k3, v3, tables, lens, cu, S, scale, out, lse, s.status)
        ctx.save_for_backward(q3, k3, v3, out, lse)
        ctx.meta = (B, S, scale)
        return out.view(B, S, Hq, D)

    @staticmethod
    def backward(ctx, do):
        q3, k3, v3, out, lse = ctx.saved_tensors
        B, S, scale = ctx.meta
        dq = torch.empty_like(q3)
        dk = torch.empty_like(k3)
        dv = torch.empty_like(v3)
        delta = torch.empty_like(lse)
        dq_acc = torch.empty(q3.shape, dtype=torch.float32, device=q3.device)
        ops._count(3)
        ops.ext().attn_train_bwd(q3, k3, v3, out, do.reshape(q3.shape).contiguous(), lse, delta, dq_acc, dq, dk, dv,
                                 B, S, scale)
        shp_q, shp_k = (B, S) + tuple(q3.shape[1:]), (B, S) + tuple(k3.shape[1:])
        return dq.view(shp_q), dk.view(shp_k), dv.view(shp_k)


def _kernel_attention_ok(q, k) -> bool:
    B, S, Hq, D = q.shape
    G = Hq // k.shape[2]
    return (q.is_cuda and q.dtype == torch.bfloat16 and D == 128 and S % 64 == 0 and Hq % k.shape[2] == 0
            and G <= 8 and (G & (G - 1)) == 0)


def attention(q, k, v, causal: bool = True):
    """q [B, S, Hq, D], k/v [B, S, Hkv, D] -> [B, S, Hq, D] (GQA). On CUDA,
    causal attention with head_dim 128 and S a multiple of 64 runs on this
    package's forward / backward kernels."""
    if causal and _kernel_attention_ok(q, k):
        return AttentionFn.apply(q, k, v)
    qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    if not q.is_cuda:
        g = q.shape[2] // k.shape[2]
        kt = kt.repeat_interleave(g, dim=1)
        vt = vt.repeat_interleave(g, dim=1)
        o = torch.nn.functional.scaled_dot_product_attention(qt.float(), kt.float(), vt.float(), is_causal=causal)
        return o.to(q.dtype).transpose(1, 2)
    o = torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, is_causal=causal,
                                                         enable_gqa=q.shape[2] != k.shape[2])
    return o.transpose(1, 2)
