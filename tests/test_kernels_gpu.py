"""Numerics of every sm_100a kernel against the fp32 PyTorch oracle.

Small and odd shapes (M, N, K not multiples of the tile) exercise the TMA
out-of-bounds fill and the epilogue masks; split-K and both GEMM orientations
are forced explicitly.
"""
import math

import pytest
import torch

from rlx_models_b200 import ops
from rlx_models_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-6)).item()


def _mk(shape, dev, scale=1.0, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dev, torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (7, 384, 192), (64, 4096, 4096), (129, 512, 320),
                                   (300, 768, 1024), (512, 2048, 512), (1000, 1280, 2048)])
@pytest.mark.parametrize("swap", [-1, 0, 1])
def test_linear_bf16(cuda, M, N, K, swap):
    if swap == 1 and M > 256:
        pytest.skip("swap-AB only for skinny M")
    x, w = _mk((M, K), cuda, 1.0, 1), _mk((N, K), cuda, 0.05, 2)
    y = ops.linear(x, w, swap=swap)
    ops.check_errors(cuda)
    r = x.float() @ w.float().T
    assert rel_err(y, r) < 1e-2


@pytest.mark.parametrize("splits", [1, 2, 5])
@pytest.mark.parametrize("M", [16, 200])
def test_linear_splitk_residual_bias_f32(cuda, splits, M):
    N, K = 640, 1536
    x, w = _mk((M, K), cuda, 1.0, 3), _mk((N, K), cuda, 0.05, 4)
    res, b = _mk((M, N), cuda, 1.0, 5), _mk((N,), cuda, 1.0, 6)
    y = ops.linear(x, w, residual=res, bias=b, splits=splits)
    r = x.float() @ w.float().T + b.float() + res.float()
    assert rel_err(y, r) < 1e-2
    y32 = ops.linear(x, w, out_dtype=torch.float32, alpha=0.5, splits=splits)
    assert rel_err(y32, 0.5 * (x.float() @ w.float().T)) < 5e-3
    ops.check_errors(cuda)
    # split-K accumulators / semaphores must be self-resetting: a second call
    # matches (fp32 atomics make the summation order, hence the last bit, vary)
    y2 = ops.linear(x, w, residual=res, bias=b, splits=splits)
    assert rel_err(y2, y) < 2e-3


@pytest.mark.parametrize("M", [1, 33, 64, 128, 257, 1024])
def test_linear_swiglu(cuda, M):
    I, K = 768, 1024
    x = _mk((M, K), cuda, 1.0, 7)
    wg, wu = _mk((I, K), cuda, 0.05, 8), _mk((I, K), cuda, 0.05, 9)
    wgu = ops.interleave_gate_up(wg, wu)
    y = ops.linear_swiglu(x, wgu)
    r = ref.swiglu(x.float() @ wg.float().T, x.float() @ wu.float().T)
    assert rel_err(y, r) < 1.5e-2
    ops.check_errors(cuda)


def test_rmsnorm_residual(cuda):
    T, H = 37, 4096
    x, res, w = _mk((T, H), cuda, 1.0, 10), _mk((T, H), cuda, 1.0, 11), _mk((H,), cuda, 1.0, 12)
    res_out = torch.empty_like(res)
    y = ops.rmsnorm(x, w, 1e-6, residual=res, residual_out=res_out)
    s = (x.float() + res.float()).bfloat16()
    assert torch.equal(res_out, s)
    assert rel_err(y, ref.rmsnorm(s, w, 1e-6)) < 1e-2
    y2 = ops.rmsnorm(x, w, 1e-6)
    assert rel_err(y2, ref.rmsnorm(x, w, 1e-6)) < 1e-2


def test_embedding(cuda):
    V, H = 1000, 512
    tab = _mk((V, H), cuda, 1.0, 13)
    ids = torch.randint(0, V, (77,), dtype=torch.int32, device=cuda)
    assert torch.equal(ops.embedding(ids, tab), tab[ids.long()])


@pytest.mark.parametrize("D,Hq,Hkv,rot", [(128, 32, 8, 128), (64, 8, 1, 64), (128, 8, 2, 64), (64, 4, 2, 32),
                                           (128, 4, 1, 96), (256, 8, 4, 256)])
def test_qkv_rope_cache_write(cuda, D, Hq, Hkv, rot):
    """QK-norm + RoPE (full, or partial over the first ``rot`` dims) + paged cache write."""
    T = 40
    qkv = _mk((T, (Hq + 2 * Hkv) * D), cuda, 1.0, 14)
    qn, kn = _mk((D,), cuda, 1.0, 15), _mk((D,), cuda, 1.0, 16)
    pos = torch.randint(0, 3000, (T,), dtype=torch.int32, device=cuda)
    inv, _ = ops.rope_inv_freq(rot, 1e6)
    inv = inv.to(cuda)
    NB = 16
    kc = torch.zeros(NB, Hkv, 16, D, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(NB * 16, device=cuda)[:T].long()
    q = ops.qkv_rope(qkv, num_q_heads=Hq, num_kv_heads=Hkv, head_dim=D, positions=pos, inv_freq=inv,
                     q_norm=qn, k_norm=kn, eps=1e-6, slots=slots, k_cache=kc, v_cache=vc, rot_dim=rot)
    qr = qkv[:, :Hq * D].view(T, Hq, D)
    kr = qkv[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D)
    vr = qkv[:, (Hq + Hkv) * D:].view(T, Hkv, D)
    q_ref = ref.rope(ref.rmsnorm_hf_bf16(qr, qn, 1e-6), pos, inv)
    k_ref = ref.rope(ref.rmsnorm_hf_bf16(kr, kn, 1e-6), pos, inv)
    assert rel_err(q, q_ref) < 1e-2
    blk, off = slots // 16, slots % 16
    kg = kc[blk, :, off]  # [T, Hkv, D]
    vg = vc[blk, :, off]
    assert rel_err(kg, k_ref) < 1e-2
    assert torch.equal(vg, vr)


def _paged_setup(dev, B, Hkv, D, lens, seed=0):
    g = torch.Generator().manual_seed(seed)
    maxb = max((l + 15) // 16 for l in lens)
    NB = sum((l + 15) // 16 for l in lens) + 3
    perm = torch.randperm(NB, generator=g)
    tables = torch.zeros(B, maxb, dtype=torch.int32)
    c = 0
    for b, l in enumerate(lens):
        n = (l + 15) // 16
        tables[b, :n] = perm[c:c + n].int()
        c += n
    kc = (torch.randn(NB, Hkv, 16, D, generator=g)).to(dev, torch.bfloat16)
    vc = (torch.randn(NB, Hkv, 16, D, generator=g)).to(dev, torch.bfloat16)
    return tables.to(dev), kc, vc


@pytest.mark.parametrize("D,Hq,Hkv", [(128, 32, 8), (128, 4, 1), (64, 64, 8)])
@pytest.mark.parametrize("splits", [0, 1, 3])
@pytest.mark.parametrize("window,use_sinks", [(0, False), (128, True)])
def test_decode_attention(cuda, D, Hq, Hkv, splits, window, use_sinks):
    lens = [1, 15, 16, 17, 100, 513, 2047]
    B = len(lens)
    tables, kc, vc = _paged_setup(cuda, B, Hkv, D, lens)
    q = _mk((B, Hq, D), cuda, 1.0, 20)
    ctx = torch.tensor(lens, dtype=torch.int32, device=cuda)
    sinks = torch.randn(Hq, device=cuda) if use_sinks else None
    scale = 1 / math.sqrt(D)
    out = ops.decode_attention(q, kc, vc, tables, ctx, scale=scale, sinks=sinks, window=window, splits=splits)
    ops.check_errors(cuda)
    for b, l in enumerate(lens):
        k = ref.gather_paged(kc, tables[b], l)
        v = ref.gather_paged(vc, tables[b], l)
        pos = torch.arange(l, device=cuda)
        r = ref.attention(q[b:b + 1], k, v, pos[-1:], pos, scale, causal=True, window=window, sinks=sinks)
        assert rel_err(out[b:b + 1], r) < 2e-2, (b, l)


@pytest.mark.parametrize("D,Hq,Hkv", [(128, 32, 8), (128, 16, 8), (64, 64, 8), (128, 24, 24)])
@pytest.mark.parametrize("window,use_sinks", [(0, False), (128, True)])
def test_prefill_attention_chunked(cuda, D, Hq, Hkv, window, use_sinks):
    # (q_len, ctx_len): ctx > q_len means earlier tokens are already cached
    cfg = [(1, 1), (17, 17), (70, 300), (257, 257), (33, 1000)]
    B = len(cfg)
    lens = [c for _, c in cfg]
    tables, kc, vc = _paged_setup(cuda, B, Hkv, D, lens, seed=3)
    qlens = [q for q, _ in cfg]
    cu = torch.tensor([0] + list(torch.tensor(qlens).cumsum(0)), dtype=torch.int32, device=cuda)
    q = _mk((sum(qlens), Hq, D), cuda, 1.0, 21)
    ctx = torch.tensor(lens, dtype=torch.int32, device=cuda)
    sinks = torch.randn(Hq, device=cuda) if use_sinks else None
    scale = 1 / math.sqrt(D)
    out = ops.prefill_attention(q, kc, vc, tables, ctx, cu, max(qlens), scale=scale, sinks=sinks, window=window)
    ops.check_errors(cuda)
    for b, (ql, l) in enumerate(cfg):
        k = ref.gather_paged(kc, tables[b], l)
        v = ref.gather_paged(vc, tables[b], l)
        kpos = torch.arange(l, device=cuda)
        qpos = kpos[l - ql:]
        r = ref.attention(q[cu[b]:cu[b + 1]], k, v, qpos, kpos, scale, causal=True, window=window, sinks=sinks)
        assert rel_err(out[cu[b]:cu[b + 1]], r) < 2e-2, (b, ql, l)


def test_argmax_and_greedy_sample(cuda):
    B, V = 9, 151936
    logits = torch.randn(B, V, device=cuda)
    logits[3, 777] = 100.0
    am = ops.argmax(logits)
    assert torch.equal(am.long(), logits.argmax(-1))
    z = torch.zeros(B, device=cuda)
    one = torch.ones(B, device=cuda)
    k0 = torch.zeros(B, dtype=torch.int32, device=cuda)
    seeds = torch.arange(B, dtype=torch.int64, device=cuda)
    offs = torch.zeros(B, dtype=torch.int64, device=cuda)
    s = ops.sample(logits, z, k0, one, z, seeds, offs)
    assert torch.equal(s.long(), logits.argmax(-1))
    # top-k = 1 at any temperature is greedy
    s1 = ops.sample(logits, one, torch.ones(B, dtype=torch.int32, device=cuda), one, z, seeds, offs)
    assert torch.equal(s1.long(), logits.argmax(-1))


def test_sampling_distribution(cuda):
    V, N = 64, 4000
    base = torch.randn(V) * 2
    logits = base[None].repeat(N, 1).to(cuda)
    T = torch.full((N,), 0.7, device=cuda)
    k0 = torch.zeros(N, dtype=torch.int32, device=cuda)
    one = torch.ones(N, device=cuda)
    z = torch.zeros(N, device=cuda)
    seeds = torch.arange(N, dtype=torch.int64, device=cuda) * 7919
    offs = torch.zeros(N, dtype=torch.int64, device=cuda)
    s = ops.sample(logits, T, k0, one, z, seeds, offs).long().cpu()
    emp = torch.bincount(s, minlength=V).float() / N
    p = torch.softmax(base / 0.7, -1)
    assert (emp - p).abs().max() < 0.04
    # top-p: every draw must come from the nucleus
    tp = torch.full((N,), 0.5, device=cuda)
    s2 = ops.sample(logits, T, k0, tp, z, seeds, offs).long().cpu()
    srt, idx = p.sort(descending=True)
    n_keep = int((srt.cumsum(0) < 0.5).sum()) + 1
    assert set(s2.tolist()) <= set(idx[:n_keep].tolist())
    # top-k = 3
    s3 = ops.sample(logits, T, torch.full((N,), 3, dtype=torch.int32, device=cuda), one, z, seeds, offs)
    assert set(s3.long().cpu().tolist()) <= set(idx[:3].tolist())


@pytest.mark.parametrize("M", [1, 17, 64, 128])
def test_accumulate_gemm_and_consumers(cuda, M):
    """Accumulate-only GEMM (split-K partials via red.add) + the three
    consumers that read the fp32 sums and zero them."""
    H, I = 1024, 768
    x = _mk((M, H), cuda, 1.0, 31)
    w = _mk((H, H), cuda, 0.05, 32)
    acc = ops.linear_acc(x, w)
    assert rel_err(acc, x.float() @ w.float().T) < 5e-3
    h = _mk((M, H), cuda, 1.0, 33)
    nw = _mk((H,), cuda, 1.0, 34)
    h_ref = (h.float() + acc.bfloat16().float()).bfloat16()
    y = ops.add_rmsnorm_acc(acc, h, nw, 1e-6)
    assert torch.equal(h, h_ref)
    assert rel_err(y, ref.rmsnorm(h_ref, nw, 1e-6)) < 1e-2
    assert torch.count_nonzero(acc) == 0
    wg, wu = _mk((I, H), cuda, 0.05, 35), _mk((I, H), cuda, 0.05, 36)
    g = ops.swiglu_acc(ops.linear_acc(x, ops.interleave_gate_up(wg, wu)))
    assert rel_err(g, ref.swiglu(x.float() @ wg.float().T, x.float() @ wu.float().T)) < 1.5e-2
    assert torch.count_nonzero(ops.scratch(cuda).acc) == 0


@pytest.mark.parametrize("M,N,K", [(256, 384, 512), (1000, 2048, 640), (4096, 1024, 2048), (96, 1536, 4096)])
def test_matmul_training_majors(cuda, M, N, K):
    """Forward (x @ W.T), dgrad (dY @ W) and wgrad (dY.T @ X, f32 accumulate)."""
    x = _mk((M, K), cuda, 1.0, 40)
    w = _mk((N, K), cuda, 0.05, 41)
    dy = _mk((M, N), cuda, 1.0, 42)
    y = ops.matmul(x, w.t())
    assert rel_err(y, x.float() @ w.float().T) < 1e-2
    dx = ops.matmul(dy, w)
    assert rel_err(dx, dy.float() @ w.float()) < 1e-2
    dw = torch.zeros(N, K, dtype=torch.float32, device=cuda)
    ops.matmul(dy.t(), x, out=dw, accumulate=True)
    ops.matmul(dy.t(), x, out=dw, accumulate=True)
    assert rel_err(dw, 2 * (dy.float().T @ x.float())) < 5e-3
    ops.check_errors(cuda)


@pytest.mark.parametrize("qscale,causal", [(0.5, False), (3.0, False), (3.0, True)])
def test_attention_noncausal_paged_rescale(cuda, qscale, causal):
    """Joint (non-causal) attention with query rows through the page table, and
    score ranges large enough that the running max grows by > 2^8 mid-row
    (lazy O rescale in the tcgen05 kernel; rows of a warp disagree)."""
    B, L, H, D = 2, 640, 2, 128
    nb = B * L // 16
    g = torch.Generator(device=cuda).manual_seed(5)
    q = (torch.randn(B * L, H, D, device=cuda, generator=g) * qscale).bfloat16()
    k = (torch.randn(nb, H, 16, D, device=cuda, generator=g) * qscale).bfloat16()
    v = torch.randn(nb, H, 16, D, device=cuda, generator=g).bfloat16()
    # batch b's pages interleaved with the other batch's: a non-identity table
    bt = torch.arange(nb, dtype=torch.int32, device=cuda).view(L // 16, B).t().contiguous()
    ctx = torch.full((B,), L, dtype=torch.int32, device=cuda)
    cu = (torch.arange(B + 1, dtype=torch.int32) * L).to(cuda)
    out = ops.prefill_attention(q, k, v, bt, ctx, cu, L, scale=1 / math.sqrt(D), causal=causal, q_paged=True)
    ops.check_errors(cuda)
    for b in range(B):
        rows = (bt[b].long()[:, None] * 16 + torch.arange(16, device=cuda)[None]).reshape(-1)
        kk = ref.gather_paged(k, bt[b], L)
        vv = ref.gather_paged(v, bt[b], L)
        pos = torch.arange(L, device=cuda)
        r = ref.attention(q[rows], kk, vv, pos, pos, 1 / math.sqrt(D), causal=causal)
        assert rel_err(out[rows], r) < 2e-2, b


@pytest.mark.parametrize("M", [1, 40, 200])
def test_linear_mxfp4_dense_and_relu(cuda, M):
    from rlx_models_b200.quant.mxfp4 import dequantize_mxfp4, quantize_mxfp4, tile_mxfp4
    N, K = 320, 512
    w = torch.randn(N, K, device=cuda) * 0.05
    b = (torch.randn(N, device=cuda) * 0.1).bfloat16()
    blocks, scales = quantize_mxfp4(w.view(1, N, K))
    wt, rexp = tile_mxfp4(blocks, scales)
    x = torch.randn(M, K, device=cuda).bfloat16()
    y = ops.linear_mxfp4(x, wt, rexp, N, bias=b)
    ops.check_errors(cuda)
    wd = dequantize_mxfp4(blocks, scales)[0]
    ref = x.half().float() @ wd.T + b.float()
    assert rel_err(y, ref) < 1e-2
    wb = w.bfloat16()
    yr = ops.linear(x, wb, bias=b, relu=True)
    assert rel_err(yr, torch.relu(x.float() @ wb.float().T + b.float())) < 1e-2


@pytest.mark.parametrize("M", [3, 64])
def test_linear_small_m_epilogues(cuda, M):
    """Swap-AB (M <= 128) path: bias + ReLU / GELU and the adaLN gate with residual."""
    import torch.nn.functional as F
    N, K, B = 512, 256, 1
    x = torch.randn(M, K, device=cuda).bfloat16()
    w = (torch.randn(N, K, device=cuda) * 0.05).bfloat16()
    b = (torch.randn(N, device=cuda) * 0.1).bfloat16()
    lin = x.float() @ w.float().T + b.float()
    assert rel_err(ops.linear(x, w, bias=b, relu=True), torch.relu(lin)) < 1e-2
    g = ops.linear(x, w, bias=b, gelu_from=128)
    assert rel_err(g, torch.cat([lin[:, :128], F.gelu(lin[:, 128:], approximate="tanh")], 1)) < 1e-2
    res = torch.randn(M, N, device=cuda).bfloat16()
    gate = torch.randn(B, N, device=cuda).bfloat16()
    y = ops.linear(x, w, bias=b, residual=res, gate=gate, gate_rows=(0, 1, M))
    assert rel_err(y, res.float() + gate.float() * lin) < 1e-2


@pytest.mark.parametrize("D,Hq,Hkv,softcap", [(256, 8, 4, 0.0), (256, 16, 8, 30.0), (128, 16, 8, 20.0),
                                               (64, 8, 2, 10.0)])
def test_attention_head256_and_softcap(cuda, D, Hq, Hkv, softcap):
    """Decode (1 and 3 KV splits) and prefill at head_dim 256 and with logit
    softcapping (Gemma), against the fp32 reference."""
    lens = [1, 17, 300, 1029]
    B = len(lens)
    tables, kc, vc = _paged_setup(cuda, B, Hkv, D, lens, seed=5)
    scale = 1 / math.sqrt(D) * 4  # large scores so that the cap matters
    ctx = torch.tensor(lens, dtype=torch.int32, device=cuda)
    q = _mk((B, Hq, D), cuda, 1.0, 40)
    for splits in (1, 3):
        out = ops.decode_attention(q, kc, vc, tables, ctx, scale=scale, splits=splits, softcap=softcap)
        ops.check_errors(cuda)
        for b, l in enumerate(lens):
            k, v = ref.gather_paged(kc, tables[b], l), ref.gather_paged(vc, tables[b], l)
            pos = torch.arange(l, device=cuda)
            r = ref.attention(q[b:b + 1], k, v, pos[-1:], pos, scale, softcap=softcap)
            assert rel_err(out[b:b + 1], r) < 2e-2, (splits, b, l)
    qlens = [1, 17, 120, 29]
    cu = torch.tensor([0] + list(torch.tensor(qlens).cumsum(0)), dtype=torch.int32, device=cuda)
    qp = _mk((sum(qlens), Hq, D), cuda, 1.0, 41)
    out = ops.prefill_attention(qp, kc, vc, tables, ctx, cu, max(qlens), scale=scale, softcap=softcap)
    ops.check_errors(cuda)
    for b, (ql, l) in enumerate(zip(qlens, lens)):
        k, v = ref.gather_paged(kc, tables[b], l), ref.gather_paged(vc, tables[b], l)
        kpos = torch.arange(l, device=cuda)
        r = ref.attention(qp[cu[b]:cu[b + 1]], k, v, kpos[l - ql:], kpos, scale, softcap=softcap)
        assert rel_err(out[cu[b]:cu[b + 1]], r) < 2e-2, (b, ql, l)


def test_geglu_epilogues(cuda):
    """GeGLU (GELU tanh form on the gate) in the gated GEMM epilogue (normal and
    swap-AB) and in the accumulate-path consumer."""
    H, I = 512, 384
    wg, wu = _mk((I, H), cuda, 0.05, 42), _mk((I, H), cuda, 0.05, 43)
    w_gu = ops.interleave_gate_up(wg, wu)
    for M in (5, 300):
        x = _mk((M, H), cuda, 1.0, 44)
        r = torch.nn.functional.gelu(x.float() @ wg.float().t(), approximate="tanh") * (x.float() @ wu.float().t())
        assert rel_err(ops.linear_swiglu(x, w_gu, act=1), r) < 1e-2
        if M <= ops.ACC_MAX_M:
            assert rel_err(ops.swiglu_acc(ops.linear_acc(x, w_gu), act=1), r) < 1e-2


@pytest.mark.parametrize("dtype,active", [(torch.float32, 0), (torch.float32, 700), (torch.bfloat16, 333)])
def test_instance_norm_vs_fp32(cuda, dtype, active):
    from rlx_models_b200 import ops
    from rlx_models_b200.ops import reference as R
    g = torch.Generator(device=cuda).manual_seed(0)
    x = (torch.randn(3, 20, 1000, device=cuda, generator=g) * 3 + 1).to(dtype)
    gamma = torch.randn(20, device=cuda, generator=g)
    beta = torch.randn(20, device=cuda, generator=g)
    y = ops.instance_norm(x, gamma, beta, active=active)
    ref = R.instance_norm(x, gamma, beta, active=active)
    rel = ((y.float() - ref).norm() / ref.norm()).item()
    assert rel < (1e-5 if dtype == torch.float32 else 1e-2), rel
