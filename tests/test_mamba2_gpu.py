"""Mamba-2 (SSD) on the GPU: the fused decode kernel against the recurrence,
and Mamba-2 / Bamba models against the fp32 oracle through the engine (graph
decode with per-sequence SSM state, chunked prefill continuing a state)."""
import pytest
import torch

from rlx_models_b200.models.mamba2 import SSMConfig, SSMHybridLM, SSMOracle, conv_window, random_weights

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("N,P", [(128, 64), (16, 32)])
def test_ssd_decode_kernel(cuda, N, P):
    from rlx_models_b200.ops._ext import ext
    g = torch.Generator().manual_seed(0)
    B, H, G, K, S = 3, 8, 2, 4, 5
    I, C = H * P, H * P + 2 * G * N
    proj = torch.randn(B, I + C + H, generator=g).bfloat16().to(cuda)
    conv_w, conv_b = (torch.randn(C, K, generator=g) * 0.5).to(cuda), (0.1 * torch.randn(C, generator=g)).to(cuda)
    A_log, dt_bias, D = torch.rand(H, generator=g).to(cuda), torch.randn(H, generator=g).to(cuda), \
        torch.randn(H, generator=g).to(cuda)
    conv = torch.randn(S, 2, C, K - 1, generator=g).bfloat16().to(cuda)
    ssm = (0.1 * torch.randn(S, H, N, P, generator=g)).to(cuda)
    slots = torch.tensor([4, -1, 1], dtype=torch.int32, device=cuda)
    pos = torch.tensor([3, 0, 8], dtype=torch.int32, device=cuda)
    conv0, ssm0 = conv.clone(), ssm.clone()
    out = torch.empty(B, I, dtype=torch.bfloat16, device=cuda)
    ext().ssd_decode(proj, I, I + C, conv_w, conv_b, A_log, dt_bias, D, 0.0, 3.0e38, conv, ssm, slots, pos, out, G)
    torch.cuda.synchronize()
    for b in range(B):
        s, p = int(slots[b]), int(pos[b])
        if s < 0:
            assert out[b].abs().max() == 0
            continue
        xbc, win = conv_window(proj[b, I:I + C, None], conv_w, conv_b, conv0[s, p & 1])
        assert torch.equal(conv[s, (p + 1) & 1], win)
        x, Bm, Cm = xbc[:, 0].float().split([I, G * N, G * N])
        dt = torch.nn.functional.softplus(proj[b, I + C:].float() + dt_bias)
        dA = torch.exp(-A_log.exp() * dt)
        Bh = Bm.view(G, N).repeat_interleave(H // G, 0)
        Ch = Cm.view(G, N).repeat_interleave(H // G, 0)
        xh = x.view(H, P)
        Sn = ssm0[s] * dA[:, None, None] + (dt[:, None, None] * Bh[:, :, None] * xh[:, None, :])
        assert torch.allclose(ssm[s], Sn, atol=1e-4, rtol=1e-3)
        y = torch.einsum("hnp,hn->hp", Sn, Ch) + D[:, None] * xh
        assert ((out[b].float() - y.reshape(-1)).norm() / y.norm()) < 1e-2


@pytest.mark.parametrize("family", ["mamba2", "bamba"])
def test_ssm_model_and_engine_vs_oracle(cuda, family):
    from rlx_models_b200.api import LLM
    from rlx_models_b200.runtime.engine import EngineConfig, SamplingParams
    if family == "mamba2":
        cfg = SSMConfig(model_type="mamba2", vocab_size=512, hidden_size=256, num_hidden_layers=3, num_heads=8,
                        head_dim=64, state_size=128, n_groups=2)
    else:
        cfg = SSMConfig(model_type="bamba", vocab_size=512, hidden_size=256, num_hidden_layers=3, num_heads=8,
                        head_dim=64, state_size=128, n_groups=2, attn_layer_indices=[1], num_attention_heads=4,
                        num_key_value_heads=2, attn_head_dim=64, intermediate_size=512)
    w = random_weights(cfg, seed=4)
    llm = LLM(SSMHybridLM(cfg, w, device=cuda), EngineConfig(max_num_seqs=4, max_model_len=256, num_blocks=64,
                                                             chunk_size=40))
    oracle = SSMOracle(cfg, {k: v.float() for k, v in w.items()})
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, 512, (61,), generator=g).tolist()
    lg = llm.logits(ids).float().cpu()
    ref = oracle.logits(ids)
    row = (lg - ref).norm(dim=-1) / ref.norm(dim=-1)
    assert row.median() < 3e-2 and (row > 0.1).float().mean() <= 0.1, row
    llm.engine.capture_graphs()
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (7, 95)]
    sp = SamplingParams(max_new_tokens=8, ignore_eos=True)
    singles = [llm.generate(p, sp)[0].token_ids for p in prompts]
    for p, toks in zip(prompts, singles):
        for t, r in zip(toks, oracle.logits(p + toks[:-1])[len(p) - 1:]):
            assert r[t] >= r.max() - 0.05 * (r.max() - r.min())
    assert [o.token_ids for o in llm.generate(prompts, sp)] == singles


@pytest.mark.parametrize("latent", [None, 128])
def test_nemotron_h_moe_model_and_engine_vs_oracle(cuda, latent):
    """Nemotron-H on the GPU: Mamba-2, NoPE attention and MoE blocks; the
    squared-ReLU experts run on the grouped MXFP4 GEMM (gate rows = up rows,
    relu(u) * u epilogue), optionally inside the latent projections; oracle on
    the same MXFP4-rounded experts."""
    import math
    from transformers import NemotronHConfig, NemotronHForCausalLM
    from rlx_models_b200.api import LLM
    from rlx_models_b200.quant.mxfp4 import mxfp4_roundtrip
    from rlx_models_b200.runtime.engine import EngineConfig, SamplingParams
    d = dict(vocab_size=512, hidden_size=256, layers_block_type=["mamba", "moe", "attention", "moe", "mamba"],
             num_attention_heads=4, num_key_value_heads=2, head_dim=64, mamba_num_heads=8, mamba_head_dim=64,
             ssm_state_size=128, n_groups=2, conv_kernel=4, expand=2, n_routed_experts=8, num_experts_per_tok=2,
             moe_intermediate_size=128, moe_shared_expert_intermediate_size=128, moe_latent_size=latent, n_group=2,
             topk_group=1, routed_scaling_factor=2.0, norm_topk_prob=True, chunk_size=16, tie_word_embeddings=False)
    torch.manual_seed(0)
    m = NemotronHForCausalLM(NemotronHConfig(**d)).eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2 and "conv1d" not in n:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
            elif n.endswith("norm.weight"):
                p.normal_(1.0, 0.2)
        for mod in m.modules():
            if hasattr(mod, "e_score_correction_bias"):
                mod.e_score_correction_bias.normal_(0, 0.2)
    w = {}
    for k, v in m.state_dict().items():
        v = v.detach().float()
        if ".experts." in k:  # the MXFP4 rounding the grouped GEMM stores (along each row's input dim)
            v = torch.stack([mxfp4_roundtrip(e.contiguous()) for e in v]) if v.dim() == 3 else mxfp4_roundtrip(v)
        w[k] = v.bfloat16()
    cfg = SSMConfig.from_dict(m.config.to_dict())
    llm = LLM(SSMHybridLM(cfg, w, device=cuda), EngineConfig(max_num_seqs=4, max_model_len=256, num_blocks=64,
                                                             chunk_size=40))
    oracle = SSMOracle(cfg, {k: v.float() for k, v in w.items()})
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, 512, (61,), generator=g).tolist()
    lg = llm.logits(ids).float().cpu()
    ref = oracle.logits(ids)
    row = (lg - ref).norm(dim=-1) / ref.norm(dim=-1)
    assert row.median() < 3e-2 and (row > 0.1).float().mean() <= 0.1, row
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (7, 95)]
    sp = SamplingParams(max_new_tokens=6, ignore_eos=True)
    for p, o in zip(prompts, llm.generate(prompts, sp)):
        for t, r in zip(o.token_ids, oracle.logits(p + o.token_ids[:-1])[len(p) - 1:]):
            assert r[t] >= r.max() - 0.05 * (r.max() - r.min())
