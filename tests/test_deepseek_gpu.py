"""DeepSeek-V3 family on the GPU: MLA with the paged latent cache and the
absorbed decode, DeepSeekMoE on the grouped MXFP4 GEMM, served by the engine
(prefill, CUDA-graph decode, continuous batching) against the fp32 oracle
with the same MXFP4-rounded expert weights."""
import json
import os

import pytest
import torch

from rlx_models_b200.models.deepseek import DeepseekConfig, DeepseekOracle, random_weights

pytestmark = pytest.mark.gpu


def _cfg(**kw):
    d = dict(model_type="deepseek_v3", vocab_size=512, hidden_size=256, intermediate_size=512,
             moe_intermediate_size=128, num_hidden_layers=3, num_attention_heads=4, n_shared_experts=1,
             n_routed_experts=16, routed_scaling_factor=2.5, kv_lora_rank=128, q_lora_rank=128, qk_rope_head_dim=64,
             v_head_dim=64, qk_nope_head_dim=64, n_group=4, topk_group=2, num_experts_per_tok=4,
             first_k_dense_replace=1, max_position_embeddings=1024,
             rope_scaling={"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 256,
                           "mscale": 1.0, "mscale_all_dim": 1.0, "beta_fast": 32, "beta_slow": 1})
    d.update(kw)
    return DeepseekConfig.from_dict(d)


def _weights(cfg, seed=5):
    from rlx_models_b200.quant.mxfp4 import mxfp4_roundtrip
    w = random_weights(cfg, seed=seed, dtype=torch.bfloat16)
    for k in list(w):
        if ".mlp.experts." in k:
            w[k] = mxfp4_roundtrip(w[k].float()).bfloat16()
    return w


def _rows(a, b):
    return (a.cpu().float() - b).norm(dim=-1) / b.norm(dim=-1)


@pytest.mark.parametrize("q_lora", [128, None])
def test_deepseek_prefill_vs_oracle(cuda, q_lora):
    from rlx_models_b200.api import LLM
    from rlx_models_b200.runtime.engine import EngineConfig
    cfg = _cfg(q_lora_rank=q_lora)
    w = _weights(cfg)
    from rlx_models_b200.models.deepseek import DeepseekLM
    llm = LLM(DeepseekLM(cfg, w, device=cuda), EngineConfig(max_num_seqs=8, max_model_len=512, kv_memory_gb=0.25))
    oracle = DeepseekOracle(cfg, {k: v.float() for k, v in w.items()})
    ids = torch.randint(0, cfg.vocab_size, (53,), generator=torch.Generator().manual_seed(2)).tolist()
    row = _rows(llm.logits(ids), oracle.logits(ids))
    assert row.median() < 2e-2, row
    assert (row > 0.1).float().mean() <= 0.1, row


def test_deepseek_engine_decode_vs_oracle(cuda, tmp_path):
    """Greedy generation through ``api.load`` of a checkpoint directory: every
    generated token is (within bf16 noise) the oracle's argmax at that
    position; batched generation of different prompts gives each prompt's
    single-sequence tokens (graphs + continuous batching over the latent cache)."""
    from rlx_models_b200.api import load
    from rlx_models_b200.runtime.engine import EngineConfig, SamplingParams
    from rlx_models_b200.weights.safetensors_io import save_file
    cfg = _cfg()
    w = _weights(cfg, seed=6)
    d = tmp_path / "ds"
    os.makedirs(d)
    (d / "config.json").write_text(json.dumps(cfg.to_hf_dict()))
    save_file({k: v.contiguous() for k, v in w.items()}, str(d / "model.safetensors"))
    llm = load(str(d), device=cuda, engine_config=EngineConfig(max_num_seqs=8, max_model_len=512, kv_memory_gb=0.25))
    llm.engine.capture_graphs()
    oracle = DeepseekOracle(cfg, {k: v.float() for k, v in w.items()})
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (7, 30, 45)]
    sp = SamplingParams(max_new_tokens=12, ignore_eos=True)
    singles = [llm.generate(p, sp)[0].token_ids for p in prompts]
    for p, toks in zip(prompts, singles):
        lg = oracle.logits(p + toks[:-1])[len(p) - 1:]
        for t, row in zip(toks, lg):
            assert row[t] >= row.max() - 0.05 * (row.max() - row.min()), (t, int(row.argmax()))
    batched = [o.token_ids for o in llm.generate(prompts, sp)]
    assert batched == singles
    assert llm.engine.stats["graph_steps"] > 0
