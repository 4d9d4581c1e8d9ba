"""KV-block retrieval on the GPU: attention over the retrieved blocks with the
paged decode kernel (needle test against full attention), and engine decode
with retrieval enabled (CUDA graphs) matching full attention while the
context fits the budget."""
import math

import pytest
import torch

from rlx_models_b200 import config as C
from rlx_models_b200 import ops
from rlx_models_b200.runtime.kv_retrieval import KVRetrieval

pytestmark = pytest.mark.gpu


def test_needle_decode_matches_full(cuda):
    g = torch.Generator().manual_seed(0)
    B, Hkv, G, D, nb = 2, 8, 4, 128, 300
    kc = (0.1 * torch.randn(nb, Hkv, 16, D, generator=g)).bfloat16().to(cuda)
    vc = torch.randn(nb, Hkv, 16, D, generator=g).bfloat16().to(cuda)
    base = torch.randn(B, Hkv, 1, D, generator=g)
    q = (base.expand(B, Hkv, G, D) + 0.05 * torch.randn(B, Hkv, G, D, generator=g)).reshape(B, Hkv * G, D)
    tables = torch.stack([torch.randperm(nb, generator=g)[:140] for _ in range(B)]).int()
    needles = [17, 90]
    for b in range(B):
        kc[tables[b, needles[b]]] = (base[b, :, 0][:, None, :] * 6).bfloat16().to(cuda)
    q, tables = q.bfloat16().to(cuda), tables.to(cuda)
    ctx = torch.tensor([140 * 16 - 7, 139 * 16 + 2], dtype=torch.int32, device=cuda)
    r = KVRetrieval(1, nb, Hkv, D, cuda, topk_blocks=8, window_blocks=8, sink_blocks=1)
    r.update(0, kc, torch.arange(nb * 16, device=cuda))
    sel, sctx = r.select(0, q, tables, ctx)
    for b in range(B):
        assert int(tables[b, needles[b]]) in sel[b].tolist()
    scale = 1 / math.sqrt(D)
    full = ops.decode_attention(q, kc, vc, tables, ctx, scale=scale)
    part = ops.decode_attention(q, kc, vc, sel, sctx, scale=scale)
    assert ((part.float() - full.float()).norm() / full.float().norm()) < 0.05


def test_engine_with_retrieval_matches_full_within_budget(cuda):
    from rlx_models_b200.api import LLM
    from rlx_models_b200.models.decoder import DecoderLM
    from rlx_models_b200.runtime.engine import EngineConfig, SamplingParams
    from rlx_models_b200.weights.init import random_weights
    cfg = C.tiny(num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=64, vocab_size=512)
    w = random_weights(cfg, 3, dtype=torch.bfloat16)
    prompts = [torch.randint(0, 512, (n,), generator=torch.Generator().manual_seed(n)).tolist() for n in (30, 75)]
    sp = SamplingParams(max_new_tokens=12, ignore_eos=True)
    outs = []
    for kvr in (None, {"topk_blocks": 4, "window_blocks": 2, "sink_blocks": 1}):
        llm = LLM(DecoderLM(cfg, w, device=cuda), EngineConfig(max_num_seqs=4, max_model_len=512, num_blocks=96,
                                                               kv_retrieval=kvr))
        llm.engine.capture_graphs()
        outs.append([o.token_ids for o in llm.generate(prompts, sp)])
        assert llm.engine.stats["graph_steps"] > 0
    assert outs[0] == outs[1]  # 7 blocks of budget cover these contexts (<= 6 blocks)


@pytest.mark.parametrize("Hkv,D,W,lens", [(8, 128, 700, [700 * 16 - 5, 3000, 40, 1]), (2, 64, 90, [90 * 16, 500])])
def test_select_kernel_matches_reference(cuda, Hkv, D, W, lens):
    g = torch.Generator().manual_seed(W)
    B, G, nb = len(lens), 4, W + 20
    r = KVRetrieval(1, nb, Hkv, D, cuda, topk_blocks=24, window_blocks=6, sink_blocks=2)
    r.summ[0] = torch.randn(nb, Hkv, D, generator=g).bfloat16().to(cuda)
    q = torch.randn(B, Hkv * G, D, generator=g).bfloat16().to(cuda)
    tables = torch.stack([torch.randperm(nb, generator=g)[:W] for _ in range(B)]).int().to(cuda)
    ctx = torch.tensor(lens, dtype=torch.int32, device=cuda)
    sel, sctx = r.select(0, q, tables, ctx)
    ref_sel, ref_ctx = r.select_reference(0, q, tables, ctx)
    torch.cuda.synchronize()
    assert torch.equal(sctx, ref_ctx)
    for b in range(B):
        n = (int(sctx[b]) + 15) // 16
        assert sel[b, :n].tolist() == ref_sel[b, :n].tolist(), b
