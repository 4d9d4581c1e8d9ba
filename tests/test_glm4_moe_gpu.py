"""GLM-4.5 family (glm4_moe) on the GPU: partial RoPE in the fused QK kernel,
sigmoid group-limited routing, shared experts and a dense first layer, against
the fp32 oracle with the same MXFP4-rounded expert weights; engine decode."""
import pytest
import torch

from rlx_models_b200 import config as C
from rlx_models_b200.models.moe import MoEDecoderLM
from rlx_models_b200.models.oracle import DecoderOracle
from rlx_models_b200.weights.init import random_weights

pytestmark = pytest.mark.gpu


def _cfg(D, **kw):
    return C.tiny("glm4_moe", hidden_size=256, num_attention_heads=4, num_key_value_heads=2, head_dim=D,
                  partial_rotary_factor=0.5, num_experts=16, num_experts_per_tok=4, moe_intermediate_size=128,
                  vocab_size=512, num_hidden_layers=3, qk_norm=False, attention_bias=True, router_scoring="sigmoid",
                  n_group=4, topk_group=2, routed_scaling_factor=2.0, n_shared_experts=1, first_k_dense_replace=1,
                  rms_norm_eps=1e-5, rope_theta=1e4, **kw)


@pytest.mark.parametrize("D", [128, 64])
def test_glm4_moe_vs_oracle(cuda, D):
    from rlx_models_b200.models.decoder import ForwardBatch
    from rlx_models_b200.quant.mxfp4 import mxfp4_roundtrip
    cfg = _cfg(D)
    w = random_weights(cfg, seed=7, dtype=torch.bfloat16)
    for k in list(w):
        if ".mlp.experts." in k:
            w[k] = mxfp4_roundtrip(w[k].float()).bfloat16()
        elif k.endswith("_proj.bias"):
            w[k] = (torch.randn(w[k].shape, generator=torch.Generator().manual_seed(len(k))) * 0.1).bfloat16()
    model = MoEDecoderLM(cfg, w, device=cuda)
    oracle = DecoderOracle(cfg, {k: v.float() for k, v in w.items()})
    T = 45
    ids = torch.randint(0, cfg.vocab_size, (T,), generator=torch.Generator().manual_seed(2))
    nb = (T + 15) // 16
    fb = ForwardBatch(input_ids=ids.int().to(cuda), positions=torch.arange(T, dtype=torch.int32, device=cuda),
                      slots=torch.arange(T, dtype=torch.int64, device=cuda), num_decode=0,
                      pre_block_tables=torch.arange(nb, dtype=torch.int32, device=cuda).view(1, -1),
                      pre_ctx_lens=torch.tensor([T], dtype=torch.int32, device=cuda),
                      pre_cu_q=torch.tensor([0, T], dtype=torch.int32, device=cuda), pre_max_q=T)
    lg = model.forward(fb, model.make_kv_cache(nb))
    ref, _ = oracle.forward(ids)
    row = (lg.cpu().float() - ref).norm(dim=-1) / ref.norm(dim=-1)
    assert row.median() < 2e-2, row
    assert (row > 0.1).float().mean() <= 0.1, row
    # engine: graph decode continues the prompt with the oracle's argmax tokens (within bf16 noise)
    from rlx_models_b200.api import LLM
    from rlx_models_b200.runtime.engine import EngineConfig, SamplingParams
    llm = LLM(model, EngineConfig(max_num_seqs=4, max_model_len=256, kv_memory_gb=0.1))
    llm.engine.capture_graphs()
    toks = llm.generate(ids.tolist(), SamplingParams(max_new_tokens=6, ignore_eos=True))[0].token_ids
    lg2, _ = oracle.forward(torch.tensor(ids.tolist() + toks[:-1]))
    for t, r in zip(toks, lg2[T - 1:]):
        assert r[t] >= r.max() - 0.05 * (r.max() - r.min())
