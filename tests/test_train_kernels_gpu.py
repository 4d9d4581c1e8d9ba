"""Training-path kernels (csrc/train/train_fused.cu) forward and backward
against fp32 torch autograd of the same ops: RMSNorm, per-head QK-norm +
rotary embedding on the fused q|k|v output, SwiGLU, the residual-fused
linear and the loss-gradient scaling of the fused lm_head + CE."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def test_rmsnorm_fwd_bwd(cuda):
    from rlx_models_b200.train import functional as TF
    g = torch.Generator(device=cuda).manual_seed(0)
    x = torch.randn(37, 2048, device=cuda, generator=g).bfloat16().requires_grad_()
    w = (1 + 0.1 * torch.randn(2048, device=cuda, generator=g)).bfloat16().requires_grad_()
    dy = torch.randn(37, 2048, device=cuda, generator=g).bfloat16()
    y = TF.rmsnorm(x, w, 1e-6)
    y.backward(dy)
    xr = x.detach().float().requires_grad_()
    wr = w.detach().float().requires_grad_()
    yr = wr * (xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-6))
    yr.backward(dy.float())
    assert _rel(y, yr) < 1e-2
    assert _rel(x.grad, xr.grad) < 2e-2
    assert _rel(w.grad, wr.grad) < 2e-2


@pytest.mark.parametrize("qk_norm", [True, False])
def test_qk_norm_rope_fwd_bwd(cuda, qk_norm):
    from rlx_models_b200.train import functional as TF
    B, S, Hq, Hkv, D = 2, 40, 4, 2, 128
    g = torch.Generator(device=cuda).manual_seed(1)
    qkv = torch.randn(B, S, (Hq + 2 * Hkv) * D, device=cuda, generator=g).bfloat16().requires_grad_()
    qn = (1 + 0.1 * torch.randn(D, device=cuda, generator=g)).bfloat16().requires_grad_() if qk_norm else None
    kn = (1 + 0.1 * torch.randn(D, device=cuda, generator=g)).bfloat16().requires_grad_() if qk_norm else None
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, device=cuda).float() / D))
    fr = torch.outer(torch.arange(S, device=cuda).float(), inv)
    emb = torch.cat([fr, fr], -1)
    cos, sin = emb.cos().bfloat16(), emb.sin().bfloat16()
    q, k, v = TF.qk_norm_rope(qkv, qn, kn, cos, sin, Hq, Hkv, D, 1e-6)
    dq, dk, dv = (torch.randn_like(t) for t in (q, k, v))
    torch.autograd.backward([q, k, v], [dq, dk, dv])

    # fp32 reference of the same math
    xr = qkv.detach().float().requires_grad_()
    qnr = qn.detach().float().requires_grad_() if qk_norm else None
    knr = kn.detach().float().requires_grad_() if qk_norm else None
    qr, kr, vr = torch.split(xr, [Hq * D, Hkv * D, Hkv * D], -1)
    qr, kr, vr = qr.reshape(B, S, Hq, D), kr.reshape(B, S, Hkv, D), vr.reshape(B, S, Hkv, D)

    def norm(t, w):
        return w * (t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6))

    def rot(t):
        c, s = cos.float()[None, :, None], sin.float()[None, :, None]
        return t * c + torch.cat([-t[..., D // 2:], t[..., :D // 2]], -1) * s

    if qk_norm:
        qr, kr = norm(qr, qnr), norm(kr, knr)
    qr, kr = rot(qr), rot(kr)
    torch.autograd.backward([qr, kr, vr], [dq.float(), dk.float(), dv.float()])
    assert _rel(q, qr) < 2e-2 and _rel(k, kr) < 2e-2 and _rel(v, vr) < 1e-3
    assert _rel(qkv.grad, xr.grad) < 3e-2
    if qk_norm:
        assert _rel(qn.grad, qnr.grad) < 3e-2 and _rel(kn.grad, knr.grad) < 3e-2


def test_swiglu_fwd_bwd(cuda):
    from rlx_models_b200.train import functional as TF
    g = torch.Generator(device=cuda).manual_seed(2)
    gu = torch.randn(3, 50, 2 * 96, device=cuda, generator=g).bfloat16().requires_grad_()
    h = TF.swiglu(gu)
    dh = torch.randn_like(h)
    h.backward(dh)
    gr = gu.detach().float().requires_grad_()
    a, b = gr.chunk(2, -1)
    hr = torch.nn.functional.silu(a) * b
    hr.backward(dh.float())
    assert _rel(h, hr) < 1e-2
    assert _rel(gu.grad, gr.grad) < 2e-2


def test_linear_residual_and_ce_scale(cuda):
    from rlx_models_b200.train import functional as TF
    g = torch.Generator(device=cuda).manual_seed(3)
    x = torch.randn(64, 256, device=cuda, generator=g).bfloat16().requires_grad_()
    w = (0.05 * torch.randn(512, 256, device=cuda, generator=g)).bfloat16().requires_grad_()
    r = torch.randn(64, 512, device=cuda, generator=g).bfloat16().requires_grad_()
    y = TF.linear_residual(x, w, r)
    dy = torch.randn_like(y)
    y.backward(dy)
    xr, wr, rr = (t.detach().float().requires_grad_() for t in (x, w, r))
    yr = rr + xr @ wr.t()
    yr.backward(dy.float())
    assert _rel(y, yr) < 1e-2
    assert _rel(x.grad, xr.grad) < 2e-2 and _rel(w.grad, wr.grad) < 2e-2 and _rel(r.grad, rr.grad) < 1e-6
    # fused lm_head + CE: a loss scaled by 3 must give 3x the gradients
    xh = torch.randn(40, 256, device=cuda, generator=g).bfloat16().requires_grad_()
    wh = (0.05 * torch.randn(1000, 256, device=cuda, generator=g)).bfloat16().requires_grad_()
    tg = torch.randint(0, 1000, (40,), device=cuda, generator=g)
    (TF.lm_head_ce(xh, wh, tg, 16) * 3.0).backward()
    xr2, wr2 = xh.detach().float().requires_grad_(), wh.detach().float().requires_grad_()
    (torch.nn.functional.cross_entropy(xr2 @ wr2.t(), tg) * 3.0).backward()
    assert _rel(xh.grad, xr2.grad) < 3e-2 and _rel(wh.grad, wr2.grad) < 3e-2


@pytest.mark.parametrize("B,S,Hq,Hkv", [(2, 128, 4, 2), (1, 320, 2, 2), (1, 192, 8, 1)])
def test_attention_fwd_bwd(cuda, B, S, Hq, Hkv):
    """tcgen05 forward (with saved log-sum-exp) + flash-style backward vs fp32 causal GQA attention."""
    from rlx_models_b200.train import functional as TF
    D = 128
    g = torch.Generator(device=cuda).manual_seed(4)
    q = torch.randn(B, S, Hq, D, device=cuda, generator=g).bfloat16().requires_grad_()
    k = torch.randn(B, S, Hkv, D, device=cuda, generator=g).bfloat16().requires_grad_()
    v = torch.randn(B, S, Hkv, D, device=cuda, generator=g).bfloat16().requires_grad_()
    o = TF.attention(q, k, v, causal=True)
    do = torch.randn_like(o)
    o.backward(do)
    qr, kr, vr = (t.detach().float().requires_grad_() for t in (q, k, v))
    G = Hq // Hkv
    kk, vv = kr.repeat_interleave(G, 2), vr.repeat_interleave(G, 2)
    s = torch.einsum("bqhd,bkhd->bhqk", qr, kk) / D ** 0.5
    mask = torch.ones(S, S, dtype=torch.bool, device=cuda).tril()
    p = torch.softmax(s.masked_fill(~mask, float("-inf")), -1)
    orf = torch.einsum("bhqk,bkhd->bqhd", p, vv)
    orf.backward(do.float())
    assert _rel(o, orf) < 2e-2
    assert _rel(q.grad, qr.grad) < 3e-2
    assert _rel(k.grad, kr.grad) < 3e-2
    assert _rel(v.grad, vr.grad) < 3e-2
