"""float8 (e4m3) KV cache: the cache write in qkv_rope, the fp8-page decode
kernel (every head dim, split and unsplit, unit and non-unit scales) against
fp32 attention over the dequantised pages, the page dequantisation that
prefill reads through, and a tiny model served with fp8 KV against the fp32
oracle (teacher-forced greedy tokens and prefill logits)."""
import math

import pytest
import torch

from rlx_models_b200 import config as C
from rlx_models_b200 import ops
from rlx_models_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
F8 = torch.float8_e4m3fn


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-6)).item()


def _paged_fp8(dev, B, Hkv, D, lens, seed=0):
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
    kc = (2 * torch.randn(NB, Hkv, 16, D, generator=g)).to(F8).to(dev)
    vc = (2 * torch.randn(NB, Hkv, 16, D, generator=g)).to(F8).to(dev)
    return tables.to(dev), kc, vc


@pytest.mark.parametrize("D,Hq,Hkv", [(128, 32, 8), (64, 64, 8), (256, 16, 4), (128, 24, 24)])
@pytest.mark.parametrize("splits", [0, 1, 3])
@pytest.mark.parametrize("scales", [(1.0, 1.0), (0.5, 2.0)])
def test_decode_attention_fp8(cuda, D, Hq, Hkv, splits, scales):
    lens = [1, 15, 16, 17, 100, 513, 2047]
    B = len(lens)
    tables, kc, vc = _paged_fp8(cuda, B, Hkv, D, lens)
    g = torch.Generator().manual_seed(20)
    q = (torch.randn(B, Hq, D, generator=g) * 0.5).to(cuda, torch.bfloat16)
    ctx = torch.tensor(lens, dtype=torch.int32, device=cuda)
    scale = 1 / math.sqrt(D)
    out = ops.decode_attention(q, kc, vc, tables, ctx, scale=scale, splits=splits, kv_scales=scales)
    ops.check_errors(cuda)
    kf, vf = kc.float() * scales[0], vc.float() * scales[1]
    for b, l in enumerate(lens):
        k = ref.gather_paged(kf, tables[b], l)
        v = ref.gather_paged(vf, tables[b], l)
        pos = torch.arange(l, device=cuda)
        r = ref.attention(q[b:b + 1], k, v, pos[-1:], pos, scale, causal=True)
        assert rel_err(out[b:b + 1], r) < 2e-2, (b, l)


@pytest.mark.parametrize("D", [64, 128, 256])
def test_qkv_rope_fp8_cache_write(cuda, D):
    T, Hq, Hkv = 40, 8, 2
    g = torch.Generator().manual_seed(14)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g).to(cuda, torch.bfloat16)
    pos = torch.randint(0, 3000, (T,), dtype=torch.int32, device=cuda)
    inv, _ = ops.rope_inv_freq(D, 1e6)
    inv = inv.to(cuda)
    NB = 16
    slots = torch.randperm(NB * 16, device=cuda)[:T].long()
    kb = torch.zeros(NB, Hkv, 16, D, dtype=torch.bfloat16, device=cuda)
    vb = torch.zeros_like(kb)
    k8 = torch.zeros(NB, Hkv, 16, D, dtype=F8, device=cuda)
    v8 = torch.zeros_like(k8)
    kw = dict(num_q_heads=Hq, num_kv_heads=Hkv, head_dim=D, positions=pos, inv_freq=inv, slots=slots)
    q_b = ops.qkv_rope(qkv, k_cache=kb, v_cache=vb, **kw)
    q_8 = ops.qkv_rope(qkv, k_cache=k8, v_cache=v8, kv_scales=(0.5, 2.0), **kw)
    assert torch.equal(q_b, q_8)
    blk, off = slots // 16, slots % 16
    want_k = (kb[blk, :, off].float() / 0.5).to(F8)
    want_v = (vb[blk, :, off].float() / 2.0).to(F8)
    assert torch.equal(k8[blk, :, off].view(torch.uint8), want_k.view(torch.uint8))
    assert torch.equal(v8[blk, :, off].view(torch.uint8), want_v.view(torch.uint8))


def test_kv_dequant_pages_and_prefill(cuda):
    D, Hq, Hkv = 128, 16, 4
    cfg = [(17, 17), (70, 300), (33, 1000)]
    lens = [c for _, c in cfg]
    tables, kc, vc = _paged_fp8(cuda, len(cfg), Hkv, D, lens, seed=3)
    ctx = torch.tensor(lens, dtype=torch.int32, device=cuda)
    kb, vb, tb = ops.kv_dequant_pages(kc, vc, tables, ctx, (0.5, 2.0))
    ops.check_errors(cuda)
    mb = tables.shape[1]
    for b, l in enumerate(lens):
        for p in range((l + 15) // 16):
            src = int(tables[b, p])
            assert torch.equal(kb[b * mb + p], (kc[src].float() * 0.5).bfloat16())
            assert torch.equal(vb[b * mb + p], (vc[src].float() * 2.0).bfloat16())
    qlens = [q for q, _ in cfg]
    cu = torch.tensor([0] + list(torch.tensor(qlens).cumsum(0)), dtype=torch.int32, device=cuda)
    g = torch.Generator().manual_seed(21)
    q = (torch.randn(sum(qlens), Hq, D, generator=g) * 0.5).to(cuda, torch.bfloat16)
    scale = 1 / math.sqrt(D)
    out = ops.prefill_attention(q, kb, vb, tb, ctx, cu, max(qlens), scale=scale)
    ops.check_errors(cuda)
    for b, (ql, l) in enumerate(cfg):
        k = ref.gather_paged(kc.float() * 0.5, tables[b], l)
        v = ref.gather_paged(vc.float() * 2.0, tables[b], l)
        kpos = torch.arange(l, device=cuda)
        r = ref.attention(q[cu[b]:cu[b + 1]], k, v, kpos[l - ql:], kpos, scale, causal=True)
        assert rel_err(out[cu[b]:cu[b + 1]], r) < 2e-2, b


def test_engine_fp8_kv_against_oracle(cuda):
    from rlx_models_b200.models.decoder import DecoderLM, ForwardBatch
    from rlx_models_b200.models.oracle import DecoderOracle
    from rlx_models_b200.runtime.engine import EngineConfig, LLMEngine, SamplingParams
    from rlx_models_b200.weights.init import random_weights
    cfg = C.tiny(num_hidden_layers=3, hidden_size=512, intermediate_size=1024, num_attention_heads=8,
                 num_key_value_heads=2, head_dim=128, vocab_size=1024)
    w = random_weights(cfg, seed=11, dtype=torch.bfloat16)
    oracle = DecoderOracle(cfg, {k: v.float() for k, v in w.items()})
    model = DecoderLM(cfg, w, device=cuda)
    eng = LLMEngine(model, EngineConfig(max_num_seqs=8, max_batched_tokens=512, max_model_len=512, num_blocks=64,
                                        kv_cache_dtype="fp8"))
    assert eng.kv.k.dtype == F8
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg.vocab_size, (100,), generator=g)
    out = eng.generate([prompt.tolist()], SamplingParams(max_new_tokens=12, ignore_eos=True))[0]
    ref_logits, _ = oracle.forward(torch.tensor(prompt.tolist() + out.token_ids[:-1]))
    ref_tokens = ref_logits[len(prompt) - 1:].argmax(-1).tolist()
    agree = sum(int(a == b) for a, b in zip(ref_tokens, out.token_ids))
    assert agree >= len(out.token_ids) - 2, (ref_tokens, out.token_ids)
    kv = model.make_kv_cache(16)
    assert kv.k.dtype == F8
    T = len(prompt)
    nb = (T + 15) // 16
    fb = ForwardBatch(input_ids=prompt.int().cuda(), positions=torch.arange(T, dtype=torch.int32).cuda(),
                      slots=torch.arange(T, dtype=torch.int64).cuda(), num_decode=0,
                      pre_block_tables=torch.arange(nb, dtype=torch.int32).view(1, -1).cuda(),
                      pre_ctx_lens=torch.tensor([T], dtype=torch.int32).cuda(),
                      pre_cu_q=torch.tensor([0, T], dtype=torch.int32).cuda(), pre_max_q=T, logit_rows=None)
    lg = model.forward(fb, kv)
    ref_prefill, _ = oracle.forward(prompt)
    assert rel_err(lg.cpu(), ref_prefill) < 6e-2
    model.set_kv_cache_dtype("bf16")
