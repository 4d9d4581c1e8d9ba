"""Mamba-1 on the GPU: the conv and selective-scan kernels against the torch
recurrence (a mixed step of continuing decode rows and fresh / continuing
prefill rows), and Mamba / Falcon-Mamba / Jamba models against the fp32
oracle through the engine (graph decode, chunked prefill continuing a state)."""
import pytest
import torch
import torch.nn.functional as F

from rlx_models_b200.models.mamba1 import Mamba1Config, Mamba1LM, Mamba1Oracle, random_weights, selective_scan

pytestmark = pytest.mark.gpu


def test_conv_and_scan_kernels(cuda):
    from rlx_models_b200.ops._ext import ext
    g = torch.Generator().manual_seed(0)
    Di, N, K, S = 256, 16, 4, 6
    lens, starts, slots = [1, 1, 9, 5], [7, 0, 0, 12], [2, 4, 0, 5]  # two decode rows, a fresh and a continuing prefill
    T = sum(lens)
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32)
    pos = torch.cat([torch.arange(s, s + n) for s, n in zip(starts, lens)]).int()
    xz = torch.randn(T, 2 * Di, generator=g).bfloat16()
    conv_w, conv_b = torch.randn(Di, K, generator=g) * 0.5, torch.randn(Di, generator=g) * 0.1
    win = torch.randn(S, Di, K - 1, generator=g).bfloat16()
    ssm = torch.randn(S, Di, N, generator=g) * 0.1
    dt = torch.randn(T, Di, generator=g).bfloat16()
    dt_bias = torch.randn(Di, generator=g) - 1
    bc = torch.randn(T, 2 * N, generator=g).bfloat16()
    A_log = torch.rand(Di, N, generator=g)
    Dp = torch.randn(Di, generator=g)
    d = lambda t: t.to(cuda)  # noqa: E731
    win_d, ssm_d = d(win.clone()), d(ssm.clone())
    xs = torch.empty(T, Di, dtype=torch.bfloat16, device=cuda)
    y = torch.empty(T, Di, dtype=torch.bfloat16, device=cuda)
    sl = torch.tensor(slots, dtype=torch.int64, device=cuda)
    ext().mamba_conv(d(cu), sl, d(pos), d(xz), d(conv_w), d(conv_b), win_d, xs)
    ext().mamba_scan(d(cu), sl, d(pos), xs, d(dt), d(dt_bias), d(bc), N, d(A_log), d(Dp), d(xz)[:, Di:], ssm_d, y)
    torch.cuda.synchronize()
    for s, (a, b) in enumerate(zip(cu[:-1].tolist(), cu[1:].tolist())):
        fresh = starts[s] == 0
        w0 = torch.zeros(Di, K - 1) if fresh else win[slots[s]].float()
        full = torch.cat([w0, xz[a:b, :Di].float().t()], 1)
        xr = F.silu(F.conv1d(full[None], conv_w[:, None, :], conv_b, groups=Di)[0]).t()
        assert torch.allclose(xs[a:b].float().cpu(), xr, atol=2e-2, rtol=2e-2)
        assert torch.equal(win_d[slots[s]].cpu(), full[:, -(K - 1):].bfloat16())
        yr, hr = selective_scan(xs[a:b].float().cpu(), F.softplus(dt[a:b].float() + dt_bias), -A_log.exp(),
                                bc[a:b, :N].float(), bc[a:b, N:].float(), Dp, xz[a:b, Di:].float(),
                                None if fresh else ssm[slots[s]])
        assert ((y[a:b].float().cpu() - yr).norm() / yr.norm()) < 1e-2
        assert torch.allclose(ssm_d[slots[s]].cpu(), hr, atol=1e-3, rtol=1e-3)


@pytest.mark.parametrize("family", ["mamba", "falcon_mamba", "jamba"])
def test_model_and_engine_vs_oracle(cuda, family):
    from rlx_models_b200.api import LLM
    from rlx_models_b200.quant.mxfp4 import mxfp4_roundtrip
    from rlx_models_b200.runtime.engine import EngineConfig, SamplingParams
    kw = dict(model_type=family, vocab_size=512, hidden_size=256, num_hidden_layers=4, state_size=16,
              time_step_rank=16)
    if family == "jamba":
        kw.update(num_attention_heads=4, num_key_value_heads=2, intermediate_size=256, num_experts=8,
                  attn_layer_period=4, attn_layer_offset=2, tie_word_embeddings=False)
    cfg = Mamba1Config(**kw)
    w = random_weights(cfg, seed=3)
    for k in list(w):
        if ".experts." in k:
            w[k] = mxfp4_roundtrip(w[k].float()).bfloat16()
    llm = LLM(Mamba1LM(cfg, w, device=cuda), EngineConfig(max_num_seqs=4, max_model_len=256, num_blocks=64,
                                                          chunk_size=40))
    oracle = Mamba1Oracle(cfg, {k: v.float() for k, v in w.items()})
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, 512, (53,), generator=g).tolist()
    lg = llm.logits(ids).float().cpu()
    ref = oracle.logits(ids)
    row = (lg - ref).norm(dim=-1) / ref.norm(dim=-1)
    assert row.median() < 3e-2 and (row > 0.1).float().mean() <= 0.15, row
    llm.engine.capture_graphs()
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (6, 90)]
    sp = SamplingParams(max_new_tokens=8, ignore_eos=True)
    singles = [llm.generate(p, sp)[0].token_ids for p in prompts]
    for p, toks in zip(prompts, singles):
        for t, r in zip(toks, oracle.logits(p + toks[:-1])[len(p) - 1:]):
            assert r[t] >= r.max() - 0.05 * (r.max() - r.min())
    assert [o.token_ids for o in llm.generate(prompts, sp)] == singles
