"""LFM2 on the GPU: the short-conv decode kernel, the model against the fp32
oracle, engine serving (graph decode with per-sequence conv windows, chunked
prefill continuing a window, batching)."""
import pytest
import torch

from rlx_models_b200.models.lfm2 import Lfm2Config, Lfm2LM, Lfm2Oracle, random_weights, short_conv

pytestmark = pytest.mark.gpu


def test_shortconv_decode_kernel(cuda):
    from rlx_models_b200.ops._ext import ext
    g = torch.Generator().manual_seed(0)
    B, H, K, S = 4, 256, 3, 6
    proj = torch.randn(B, 3 * H, generator=g).bfloat16().to(cuda)
    w = torch.randn(H, K, generator=g).to(cuda)
    bias = torch.randn(H, generator=g).to(cuda)
    conv = torch.randn(S, 2, H, K - 1, generator=g).bfloat16().to(cuda)
    slots = torch.tensor([2, -1, 0, 5], dtype=torch.int32, device=cuda)
    pos = torch.tensor([4, 0, 9, 1], dtype=torch.int32, device=cuda)
    conv0 = conv.clone()
    out = torch.empty(B, H, dtype=torch.bfloat16, device=cuda)
    ext().shortconv_decode(proj, w, bias, conv, slots, pos, out)
    torch.cuda.synchronize()
    for b in range(B):
        s, p = int(slots[b]), int(pos[b])
        if s < 0:
            assert out[b].abs().max() == 0
            continue
        bx = (proj[b, :H].float() * proj[b, 2 * H:].float()).bfloat16()
        y, win = short_conv(bx[:, None], w, bias, conv0[s, p & 1])
        assert torch.equal(conv[s, (p + 1) & 1], win)
        r = proj[b, H:2 * H].float() * y[:, 0].float()
        assert ((out[b].float() - r).norm() / r.norm()) < 1e-2


def test_lfm2_model_and_engine_vs_oracle(cuda):
    from rlx_models_b200.api import LLM
    from rlx_models_b200.runtime.engine import EngineConfig, SamplingParams
    cfg = Lfm2Config(vocab_size=512, hidden_size=256, intermediate_size=768, num_hidden_layers=4, num_attention_heads=4,
                     num_key_value_heads=2, block_multiple_of=128, layer_types=["conv", "full_attention", "conv",
                                                                                 "full_attention"])
    w = random_weights(cfg, seed=2)
    llm = LLM(Lfm2LM(cfg, w, device=cuda), EngineConfig(max_num_seqs=4, max_model_len=256, num_blocks=64,
                                                        chunk_size=40))
    oracle = Lfm2Oracle(cfg, {k: v.float() for k, v in w.items()})
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, 512, (57,), generator=g).tolist()
    lg = llm.logits(ids).float().cpu()
    ref = oracle.logits(ids)
    row = (lg - ref).norm(dim=-1) / ref.norm(dim=-1)
    assert row.median() < 3e-2 and (row > 0.1).float().mean() <= 0.1, row
    llm.engine.capture_graphs()
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (5, 90, 23)]
    sp = SamplingParams(max_new_tokens=8, ignore_eos=True)
    singles = [llm.generate(p, sp)[0].token_ids for p in prompts]
    for p, toks in zip(prompts, singles):
        for t, r in zip(toks, oracle.logits(p + toks[:-1])[len(p) - 1:]):
            assert r[t] >= r.max() - 0.05 * (r.max() - r.min())
    assert [o.token_ids for o in llm.generate(prompts, sp)] == singles
    assert llm.engine.stats["graph_steps"] > 0
