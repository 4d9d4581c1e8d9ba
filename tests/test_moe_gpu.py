"""MoE (gpt-oss family) on the GPU: routing/permutation kernels, the grouped
MXFP4 GEMM against a dequantized fp32 reference, and the full model against
the fp32 oracle (sinks, sliding window beyond its length, YaRN, biases)."""

import math

import pytest
import torch

from rlx_models_b200 import config as C
from rlx_models_b200.models.moe import MoEDecoderLM, hf_interleaved_to_grouped
from rlx_models_b200.models.oracle import DecoderOracle
from rlx_models_b200.ops import ext, scratch
from rlx_models_b200.quant.mxfp4 import dequantize_mxfp4, quantize_mxfp4, tile_mxfp4
from rlx_models_b200.weights.init import random_weights

pytestmark = pytest.mark.gpu


def rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-9)).item()


@pytest.mark.parametrize("T,E,k,bt,wscale", [(3, 8, 2, 32, 0.05), (200, 16, 4, 64, 0.05), (1, 128, 4, 32, 0.05),
                                             (300, 8, 4, 128, 0.05), (600, 8, 4, 128, 0.05),
                                             (40, 8, 2, 32, 300.0)])
def test_grouped_mxfp4_gemm(cuda, T, E, k, bt, wscale):
    """All four token-tile widths; wscale 300 puts E8M0 scales above 2^0."""
    H, I = 256, 384 if T != 600 else 320
    g = torch.Generator().manual_seed(0)
    x = (torch.randn(T, H, generator=g) / max(1.0, wscale)).to(cuda, torch.bfloat16)
    wgu = torch.randn(E, 2 * I, H, generator=g) * wscale
    wdn = torch.randn(E, H, I, generator=g) * 0.05
    gub, gus = quantize_mxfp4(wgu)
    dnb, dns = quantize_mxfp4(wdn)
    gu_bias = torch.randn(E, 2 * I, generator=g) * 0.1
    dn_bias = torch.randn(E, H, generator=g) * 0.1
    logits = torch.randn(T, E, generator=g).to(cuda)
    experts = torch.empty(T, k, dtype=torch.int32, device=cuda)
    weights = torch.empty(T, k, dtype=torch.float32, device=cuda)
    ext().moe_route(logits, k, False, True, experts, weights)
    tv, ti = logits.topk(k, -1)
    assert torch.equal(ti.int().sort(-1).values, experts.sort(-1).values)
    n = T * k
    meta = torch.empty(2 * E + 2, dtype=torch.int32, device=cuda)
    tiles = torch.empty(4 * (n // bt + E + 1), dtype=torch.int32, device=cuda)
    perm = torch.empty(n, dtype=torch.int32, device=cuda)
    inv = torch.empty(n, dtype=torch.int32, device=cuda)
    cur = torch.empty(E, dtype=torch.int32, device=cuda)
    ext().moe_align(experts, E, 0, E, bt, meta, tiles, perm, inv, cur)
    a = torch.empty(n, H, dtype=torch.float16, device=cuda)
    ext().moe_gather(x, perm, meta, E, k, a)
    assert int(meta[0]) > 0 and int(meta[1:E + 1].sum()) == n
    grouped = lambda t: hf_interleaved_to_grouped(t.reshape(E, 2 * I, -1).to(cuda)).contiguous()
    gu_t, gu_e = tile_mxfp4(grouped(gub), grouped(gus))
    dn_t, dn_e = tile_mxfp4(dnb.to(cuda), dns.to(cuda))
    gu = torch.empty(n, I, dtype=torch.float16, device=cuda)
    st = scratch(cuda).status
    limit = 7.0 * max(1.0, wscale)
    ext().moe_gemm(a, gu_t, gu_e, 2 * I, hf_interleaved_to_grouped(gu_bias.to(cuda).bfloat16()), None,
                   perm, meta, tiles, gu, True, limit, 1.702, bt, st)
    dn = torch.empty(n, H, dtype=torch.bfloat16, device=cuda)
    ext().moe_gemm(gu, dn_t, dn_e, H, dn_bias.to(cuda).bfloat16(), weights.view(-1), perm, meta, tiles, dn, False,
                   0.0, 0.0, bt, st)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=cuda)
    ext().moe_combine(dn, inv, k, out, False)
    torch.cuda.synchronize()
    assert int(st[0]) == 0
    # reference
    wgu_d, wdn_d = dequantize_mxfp4(gub, gus), dequantize_mxfp4(dnb, dns)
    xf = x.float().cpu()
    ref = torch.zeros(T, H)
    for t in range(T):
        for s in range(k):
            e = int(experts[t, s])
            h = xf[t] @ wgu_d[e].T + gu_bias[e].bfloat16().float()
            gt, up = h[::2].clamp(max=limit), h[1::2].clamp(-limit, limit)
            act = ((up + 1) * gt * torch.sigmoid(1.702 * gt)).half().float()
            ref[t] += float(weights[t, s]) * (act @ wdn_d[e].T + dn_bias[e].bfloat16().float())
    assert rel(out.cpu(), ref) < 3e-2


def test_gpt_oss_model_vs_oracle(cuda):
    cfg = C.tiny("gpt_oss", hidden_size=256, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                 num_experts=8, num_experts_per_tok=2, moe_intermediate_size=256, intermediate_size=256,
                 vocab_size=512, sliding_window=16)
    w = random_weights(cfg, seed=3, dtype=torch.bfloat16)
    for k, v in list(w.items()):
        if k.endswith("sinks"):
            w[k] = torch.randn_like(v)
    model = MoEDecoderLM(cfg, w, device=cuda)
    oracle = DecoderOracle(cfg, {k: (v.float() if v.dtype != torch.uint8 else v) for k, v in w.items()})
    from rlx_models_b200.models.decoder import ForwardBatch
    T = 40
    ids = torch.randint(0, cfg.vocab_size, (T,), generator=torch.Generator().manual_seed(1))
    nb = (T + 15) // 16
    fb = ForwardBatch(input_ids=ids.int().to(cuda), positions=torch.arange(T, dtype=torch.int32, device=cuda),
                      slots=torch.arange(T, dtype=torch.int64, device=cuda), num_decode=0,
                      pre_block_tables=torch.arange(nb, dtype=torch.int32, device=cuda).view(1, -1),
                      pre_ctx_lens=torch.tensor([T], dtype=torch.int32, device=cuda),
                      pre_cu_q=torch.tensor([0, T], dtype=torch.int32, device=cuda), pre_max_q=T)
    lg = model.forward(fb, model.make_kv_cache(nb))
    ref, _ = oracle.forward(ids)
    # bf16 router logits can flip a near-tied top-k choice against the fp32
    # oracle, which changes that token's row outright: judge rows, not the sum
    row = ((lg.cpu().float() - ref).norm(dim=-1) / ref.norm(dim=-1))
    assert row.median() < 2e-2, row
    assert (row > 0.1).float().mean() <= 0.1, row
    # engine decode (graphs) produces the oracle's greedy continuation's first token
    from rlx_models_b200.runtime.engine import EngineConfig, LLMEngine, SamplingParams
    eng = LLMEngine(model, EngineConfig(max_num_seqs=4, max_model_len=128, num_blocks=32))
    out = eng.generate([ids.tolist()], SamplingParams(max_new_tokens=6, ignore_eos=True))[0]
    assert out.token_ids[0] == int(lg[-1].argmax())


def test_qwen3_moe_model_vs_oracle(cuda):
    """Qwen3-MoE (softmax-first routing with renormalisation, plain SwiGLU,
    QK-norm, no biases) through the grouped MXFP4 GEMM; the oracle uses the
    same MXFP4-rounded expert weights."""
    from rlx_models_b200.quant.mxfp4 import mxfp4_roundtrip
    cfg = C.tiny("qwen3_moe", hidden_size=256, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                 num_experts=8, num_experts_per_tok=2, moe_intermediate_size=128, vocab_size=512)
    w = random_weights(cfg, seed=4, dtype=torch.bfloat16)
    for k in list(w):
        if ".mlp.experts." in k:
            w[k] = mxfp4_roundtrip(w[k].float()).bfloat16()
    model = MoEDecoderLM(cfg, w, device=cuda)
    oracle = DecoderOracle(cfg, {k: v.float() for k, v in w.items()})
    from rlx_models_b200.models.decoder import ForwardBatch
    T = 37
    ids = torch.randint(0, cfg.vocab_size, (T,), generator=torch.Generator().manual_seed(2))
    nb = (T + 15) // 16
    fb = ForwardBatch(input_ids=ids.int().to(cuda), positions=torch.arange(T, dtype=torch.int32, device=cuda),
                      slots=torch.arange(T, dtype=torch.int64, device=cuda), num_decode=0,
                      pre_block_tables=torch.arange(nb, dtype=torch.int32, device=cuda).view(1, -1),
                      pre_ctx_lens=torch.tensor([T], dtype=torch.int32, device=cuda),
                      pre_cu_q=torch.tensor([0, T], dtype=torch.int32, device=cuda), pre_max_q=T)
    lg = model.forward(fb, model.make_kv_cache(nb))
    ref, _ = oracle.forward(ids)
    row = ((lg.cpu().float() - ref).norm(dim=-1) / ref.norm(dim=-1))
    assert row.median() < 2e-2, row
    assert (row > 0.1).float().mean() <= 0.1, row


@pytest.mark.parametrize("family", ["mixtral", "qwen2_moe"])
def test_mixtral_qwen2_moe_vs_oracle(cuda, family):
    """Mixtral (block_sparse_moe checkpoint names) and Qwen2-MoE (q/k/v biases,
    sigmoid-gated shared expert) through the grouped MXFP4 GEMM; the oracle
    uses the same MXFP4-rounded expert weights."""
    from rlx_models_b200.quant.mxfp4 import mxfp4_roundtrip
    kw = dict(hidden_size=256, num_attention_heads=4, num_key_value_heads=2, head_dim=64, num_experts=8,
              num_experts_per_tok=2, moe_intermediate_size=128, vocab_size=512, qk_norm=False)
    if family == "qwen2_moe":
        kw.update(attention_bias=True, shared_expert_intermediate_size=256, norm_topk_prob=False)
    cfg = C.tiny(family, **kw)
    w = random_weights(cfg, seed=6, dtype=torch.bfloat16)
    for k in list(w):
        if ".mlp.experts." in k:
            w[k] = mxfp4_roundtrip(w[k].float()).bfloat16()
        if k.endswith(".bias"):
            w[k] = (torch.randn(w[k].shape, generator=torch.Generator().manual_seed(3)) * 0.1).bfloat16()
    if family == "mixtral":  # serve the checkpoint under Mixtral's own tensor names
        ren = {}
        for k, v in w.items():
            if ".mlp.gate." in k:
                k = k.replace(".mlp.gate.", ".block_sparse_moe.gate.")
            elif ".mlp.experts." in k:
                k = k.replace(".mlp.experts.", ".block_sparse_moe.experts.")
                k = k.replace(".gate_proj.", ".w1.").replace(".up_proj.", ".w3.").replace(".down_proj.", ".w2.")
            ren[k] = v
        w = ren
    model = MoEDecoderLM(cfg, w, device=cuda)
    oracle = DecoderOracle(cfg, {k: v.float() for k, v in w.items()})
    from rlx_models_b200.models.decoder import ForwardBatch
    T = 33
    ids = torch.randint(0, cfg.vocab_size, (T,), generator=torch.Generator().manual_seed(4))
    nb = (T + 15) // 16
    fb = ForwardBatch(input_ids=ids.int().to(cuda), positions=torch.arange(T, dtype=torch.int32, device=cuda),
                      slots=torch.arange(T, dtype=torch.int64, device=cuda), num_decode=0,
                      pre_block_tables=torch.arange(nb, dtype=torch.int32, device=cuda).view(1, -1),
                      pre_ctx_lens=torch.tensor([T], dtype=torch.int32, device=cuda),
                      pre_cu_q=torch.tensor([0, T], dtype=torch.int32, device=cuda), pre_max_q=T)
    lg = model.forward(fb, model.make_kv_cache(nb))
    ref, _ = oracle.forward(ids)
    row = ((lg.cpu().float() - ref).norm(dim=-1) / ref.norm(dim=-1))
    assert row.median() < 2e-2, row
    assert (row > 0.1).float().mean() <= 0.1, row


def test_minimax_m2_vs_oracle(cuda):
    """MiniMax-M2 on the GPU: full-width QK-norm (one RMSNorm over all heads of
    a token, in place on the bf16 q|k|v projection), partial RoPE, sigmoid
    routing with the correction bias; oracle on the same MXFP4-rounded experts."""
    from rlx_models_b200.config import DecoderConfig
    from rlx_models_b200.models.decoder import ForwardBatch
    from rlx_models_b200.quant.mxfp4 import mxfp4_roundtrip
    cfg = DecoderConfig.from_hf_dict(dict(model_type="minimax_m2", vocab_size=512, hidden_size=256,
                                          intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                                          num_key_value_heads=2, head_dim=64, num_local_experts=8,
                                          num_experts_per_tok=2, rotary_dim=32, rms_norm_eps=1e-6,
                                          max_position_embeddings=256))
    assert cfg.qk_norm_full and cfg.rotary_dim == 32
    w = random_weights(cfg, seed=8, dtype=torch.bfloat16)
    for k in list(w):
        if ".mlp.experts." in k:
            w[k] = mxfp4_roundtrip(w[k].float()).bfloat16()
        if k.endswith("e_score_correction_bias"):
            w[k] = torch.randn(w[k].shape, generator=torch.Generator().manual_seed(5)) * 0.5
    model = MoEDecoderLM(cfg, w, device=cuda)
    oracle = DecoderOracle(cfg, {k: v.float() for k, v in w.items()})
    for T in (37, 5):  # prefill-sized and decode-sized batches
        ids = torch.randint(0, cfg.vocab_size, (T,), generator=torch.Generator().manual_seed(T))
        nb = (T + 15) // 16
        fb = ForwardBatch(input_ids=ids.int().to(cuda), positions=torch.arange(T, dtype=torch.int32, device=cuda),
                          slots=torch.arange(T, dtype=torch.int64, device=cuda), num_decode=0,
                          pre_block_tables=torch.arange(nb, dtype=torch.int32, device=cuda).view(1, -1),
                          pre_ctx_lens=torch.tensor([T], dtype=torch.int32, device=cuda),
                          pre_cu_q=torch.tensor([0, T], dtype=torch.int32, device=cuda), pre_max_q=T)
        lg = model.forward(fb, model.make_kv_cache(nb))
        ref, _ = oracle.forward(ids)
        row = ((lg.cpu().float() - ref).norm(dim=-1) / ref.norm(dim=-1))
        assert row.median() < 2e-2, row
        assert (row > 0.1).float().mean() <= 0.2, row


def test_llama4_text_vs_oracle(cuda):
    """Llama-4 text on the GPU: q / k rows reordered so the half-split RoPE kernel
    rotates the interleaved pairs, weightless QK norm on the RoPE layers, zero
    frequencies on the NoPE layer, top-1 sigmoid routing that scales the expert
    input, shared expert, dense / MoE interleave, checkpoint names with fused
    expert banks; against the oracle (HF semantics) on MXFP4-rounded experts,
    below the context where chunking and the query temperature start."""
    from rlx_models_b200.config import DecoderConfig
    from rlx_models_b200.models.decoder import ForwardBatch
    from rlx_models_b200.quant.mxfp4 import mxfp4_roundtrip
    hf = dict(model_type="llama4_text", vocab_size=512, hidden_size=256, intermediate_size=128,
              intermediate_size_mlp=384, num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2,
              head_dim=64, num_local_experts=8, num_experts_per_tok=1, interleave_moe_layer_step=2,
              attention_chunk_size=128, floor_scale=128, rms_norm_eps=1e-5, max_position_embeddings=256)
    cfg = DecoderConfig.from_hf_dict(hf)
    g = torch.Generator().manual_seed(4)
    H, I, E = 256, 128, 8
    r = lambda *s, f=1.0: (torch.randn(*s, generator=g) * f / math.sqrt(s[-1])).bfloat16()  # noqa: E731
    w = {"model.embed_tokens.weight": torch.randn(512, H, generator=g).bfloat16(),
         "model.norm.weight": (1 + 0.1 * torch.randn(H, generator=g)).bfloat16(), "lm_head.weight": r(512, H)}
    for i in range(4):
        p = f"model.layers.{i}."
        w[p + "input_layernorm.weight"] = (1 + 0.1 * torch.randn(H, generator=g)).bfloat16()
        w[p + "post_attention_layernorm.weight"] = (1 + 0.1 * torch.randn(H, generator=g)).bfloat16()
        for n, o in (("q", 256), ("k", 128), ("v", 128)):
            w[p + f"self_attn.{n}_proj.weight"] = r(o, H)
        w[p + "self_attn.o_proj.weight"] = r(H, 256)
        f = p + "feed_forward."
        if i in cfg.moe_layers:
            w[f + "router.weight"] = r(E, H, f=4.0)
            gu = torch.randn(E, H, 2 * I, generator=g) / math.sqrt(H)
            dn = torch.randn(E, I, H, generator=g) / math.sqrt(I)
            # experts as the MXFP4 rounding the GPU path stores (per output row, along the input)
            gu = torch.stack([mxfp4_roundtrip(gu[e].t().contiguous()).t() for e in range(E)])
            dn = torch.stack([mxfp4_roundtrip(dn[e].t().contiguous()).t() for e in range(E)])
            w[f + "experts.gate_up_proj"], w[f + "experts.down_proj"] = gu.bfloat16(), dn.bfloat16()
            for n, (o, ii) in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
                w[f + f"shared_expert.{n}_proj.weight"] = r(o, ii)
        else:
            for n, (o, ii) in (("gate", (384, H)), ("up", (384, H)), ("down", (H, 384))):
                w[f + f"{n}_proj.weight"] = r(o, ii)
    model = MoEDecoderLM(cfg, w, device=cuda)
    assert model.max_context == 128
    oracle = DecoderOracle(cfg, {k: v.float() for k, v in w.items()})
    for T in (45, 6):
        ids = torch.randint(0, 512, (T,), generator=torch.Generator().manual_seed(T))
        nb = (T + 15) // 16
        fb = ForwardBatch(input_ids=ids.int().to(cuda), positions=torch.arange(T, dtype=torch.int32, device=cuda),
                          slots=torch.arange(T, dtype=torch.int64, device=cuda), num_decode=0,
                          pre_block_tables=torch.arange(nb, dtype=torch.int32, device=cuda).view(1, -1),
                          pre_ctx_lens=torch.tensor([T], dtype=torch.int32, device=cuda),
                          pre_cu_q=torch.tensor([0, T], dtype=torch.int32, device=cuda), pre_max_q=T)
        lg = model.forward(fb, model.make_kv_cache(nb))
        ref, _ = oracle.forward(ids)
        row = ((lg.cpu().float() - ref).norm(dim=-1) / ref.norm(dim=-1))
        assert row.median() < 2e-2, row
        assert (row > 0.1).float().mean() <= 0.2, row
