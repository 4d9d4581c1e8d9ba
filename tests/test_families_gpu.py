"""Dense decoder families beyond Qwen3 on the GPU against the fp32 oracle
(Llama: no QK-norm, untied head; Qwen2: q/k/v biases; Mistral), and the
``LLM.embed`` entry point against the oracle's final hidden states."""
import pytest
import torch

from rlx_models_b200 import config as C
from rlx_models_b200.models.decoder import DecoderLM, ForwardBatch
from rlx_models_b200.models.oracle import DecoderOracle
from rlx_models_b200.weights.init import random_weights

pytestmark = pytest.mark.gpu


def _prefill(model, ids, dev):
    T = len(ids)
    nb = (T + 15) // 16
    fb = ForwardBatch(input_ids=torch.tensor(ids, dtype=torch.int32, device=dev),
                      positions=torch.arange(T, dtype=torch.int32, device=dev),
                      slots=torch.arange(T, dtype=torch.int64, device=dev), num_decode=0,
                      pre_block_tables=torch.arange(nb, dtype=torch.int32, device=dev).view(1, -1),
                      pre_ctx_lens=torch.tensor([T], dtype=torch.int32, device=dev),
                      pre_cu_q=torch.tensor([0, T], dtype=torch.int32, device=dev), pre_max_q=T)
    return model.forward(fb, model.make_kv_cache(nb))


@pytest.mark.parametrize("family,over", [
    ("llama", dict(qk_norm=False, tie_word_embeddings=False, rope_theta=5e5)),
    ("qwen2", dict(qk_norm=False, attention_bias=True, tie_word_embeddings=True)),
    ("mistral", dict(qk_norm=False, tie_word_embeddings=False, rope_theta=1e6)),
    ("granite", dict(qk_norm=False, tie_word_embeddings=True, embedding_multiplier=12.0, residual_multiplier=0.22,
                     attention_multiplier=0.0078125, logits_scaling=8.0)),
])
def test_family_vs_oracle(cuda, family, over):
    cfg = C.tiny(family, num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=64, vocab_size=512, **over)
    w = random_weights(cfg, 1, dtype=torch.bfloat16)
    for k in list(w):
        if k.endswith(".bias"):  # biases start at zero: make them matter
            w[k] = (torch.randn(w[k].shape, generator=torch.Generator().manual_seed(7)) * 0.2).bfloat16()
    model = DecoderLM(cfg, w, device=cuda)
    ids = torch.randint(0, 512, (45,), generator=torch.Generator().manual_seed(2)).tolist()
    lg = _prefill(model, ids, cuda).float().cpu()
    ref, _ = DecoderOracle(cfg, {k: v.float() for k, v in w.items()}).forward(torch.tensor(ids))
    rel = ((lg - ref).norm() / ref.norm()).item()
    assert rel < 2e-2, rel
    assert (lg.argmax(-1) == ref.argmax(-1)).float().mean() > 0.9


def test_embed_matches_oracle_hidden(cuda):
    from rlx_models_b200.api import LLM
    from rlx_models_b200.runtime.engine import EngineConfig
    cfg = C.tiny(num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=64, vocab_size=512)
    w = random_weights(cfg, 3, dtype=torch.bfloat16)
    llm = LLM(DecoderLM(cfg, w, device=cuda), EngineConfig(max_num_seqs=4, max_model_len=128, num_blocks=32))
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (5, 33, 17)]
    oracle = DecoderOracle(cfg, {k: v.float() for k, v in w.items()})
    for pooling in ("last", "mean"):
        e = llm.embed(prompts, pooling=pooling).cpu()
        for i, p in enumerate(prompts):
            h, _ = oracle.forward_hidden(torch.tensor(p))
            r = h[-1] if pooling == "last" else h.mean(0)
            r = r / r.norm()
            assert torch.nn.functional.cosine_similarity(e[i], r, dim=0) > 0.999
    assert torch.allclose(e.norm(dim=-1), torch.ones(3), atol=1e-4)


def test_phi3_fused_longrope_partial_vs_oracle(cuda):
    """Phi-3 layout (fused qkv_proj / gate_up_proj), LongRoPE short factors with
    the attention factor, RoPE on 3/4 of each head."""
    g = torch.Generator().manual_seed(9)
    rot = 48
    rs = {"rope_type": "longrope", "short_factor": (1 + 2 * torch.rand(rot // 2, generator=g)).tolist(),
          "long_factor": (2 + 8 * torch.rand(rot // 2, generator=g)).tolist(), "original_max_position_embeddings": 256}
    cfg = C.tiny("phi3", num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=64, vocab_size=512, qk_norm=False, tie_word_embeddings=False,
                 partial_rotary_factor=0.75, rope_scaling=rs, max_position_embeddings=1024, rope_theta=1e4)
    w = random_weights(cfg, 5, dtype=torch.bfloat16)
    fused = {}
    for k, v in w.items():
        if ".self_attn.q_proj." in k:
            p = k.replace("q_proj", "qkv_proj")
            fused[p] = torch.cat([v, w[k.replace("q_proj", "k_proj")], w[k.replace("q_proj", "v_proj")]], 0)
        elif ".mlp.gate_proj." in k:
            fused[k.replace("gate_proj", "gate_up_proj")] = torch.cat([v, w[k.replace("gate_proj", "up_proj")]], 0)
        elif not any(s in k for s in (".k_proj.", ".v_proj.", ".up_proj.")):
            fused[k] = v
    model = DecoderLM(cfg, fused, device=cuda)
    ids = torch.randint(0, 512, (200,), generator=torch.Generator().manual_seed(2)).tolist()
    lg = _prefill(model, ids, cuda).float().cpu()
    ref, _ = DecoderOracle(cfg, {k: v.float() for k, v in fused.items()}).forward(torch.tensor(ids))
    rel = ((lg - ref).norm() / ref.norm()).item()
    assert rel < 2e-2, rel
    assert (lg.argmax(-1) == ref.argmax(-1)).float().mean() > 0.9


@pytest.mark.parametrize("family,D", [("gemma", 256), ("gemma2", 256), ("gemma3_text", 128), ("gemma3_text", 256)])
def test_gemma_vs_oracle(cuda, family, D):
    """Gemma 1 / 2 / 3 on the GPU: GeGLU epilogue, (1 + w) norms, sandwich norms,
    attention (Gemma-2) and final logit softcapping in the kernels, sliding
    layers shorter than the prompt, Gemma-3 local RoPE base and QK-norm;
    head_dim 256 through the QK-norm/RoPE, prefill and decode kernels."""
    from rlx_models_b200.api import LLM
    from rlx_models_b200.runtime.engine import EngineConfig, SamplingParams
    over = dict(qk_norm=family == "gemma3_text", norm_unit_offset=True, sandwich_norm=family != "gemma",
                mlp_act="gelu_tanh", embedding_multiplier=16.0, tie_word_embeddings=True, rms_norm_eps=1e-6)
    if family != "gemma":
        over.update(sliding_window=32, attention_multiplier=D ** -0.5,
                    layer_types=["sliding_attention", "full_attention", "sliding_attention", "full_attention"])
    if family == "gemma2":
        over.update(attn_softcap=20.0, final_softcap=15.0)
    if family == "gemma3_text":
        over.update(rope_local_theta=1e4, rope_theta=1e6, rope_scaling={"rope_type": "linear", "factor": 4.0})
    cfg = C.tiny(family, num_hidden_layers=4, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=D, vocab_size=512, **over)
    w = random_weights(cfg, 11, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(12)
    for k in list(w):
        if k.endswith("norm.weight"):  # (1 + w) norms: weights around zero
            w[k] = (torch.randn(w[k].shape, generator=g) * 0.2).bfloat16()
    model = DecoderLM(cfg, w, device=cuda)
    oracle = DecoderOracle(cfg, {k: v.float() for k, v in w.items()})
    ids = torch.randint(0, 512, (70,), generator=torch.Generator().manual_seed(2)).tolist()
    lg = _prefill(model, ids, cuda).float().cpu()
    ref, _ = oracle.forward(torch.tensor(ids))
    rel = ((lg - ref).norm() / ref.norm()).item()
    assert rel < 3e-2, rel
    assert (lg.argmax(-1) == ref.argmax(-1)).float().mean() > 0.85
    llm = LLM(model, EngineConfig(max_num_seqs=4, max_model_len=256, num_blocks=64))
    llm.engine.capture_graphs()
    toks = llm.generate(ids, SamplingParams(max_new_tokens=6, ignore_eos=True))[0].token_ids
    lg2, _ = oracle.forward(torch.tensor(ids + toks[:-1]))
    for t, r in zip(toks, lg2[len(ids) - 1:]):
        assert r[t] >= r.max() - 0.05 * (r.max() - r.min())


def test_qwen3_vl_text_checkpoint_loads_and_serves(cuda, tmp_path):
    """A Qwen3-VL checkpoint (the text model under ``model.language_model.``, a
    vision tower beside it) loads through ``api.load`` as its Qwen3 language model
    and serves text; first generated tokens against the oracle."""
    import json
    import math
    import transformers as T
    from rlx_models_b200.api import load
    from rlx_models_b200.runtime.engine import EngineConfig, SamplingParams
    from rlx_models_b200.weights.aliases import LanguageModelView
    from rlx_models_b200.weights.safetensors_io import save_file
    tc = dict(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
              num_key_value_heads=2, head_dim=64, tie_word_embeddings=False,
              rope_parameters={"rope_type": "default", "rope_theta": 1e6, "mrope_section": [8, 12, 12],
                               "mrope_interleaved": True})
    vc = dict(depth=1, hidden_size=32, intermediate_size=64, num_heads=2, out_hidden_size=256,
              deepstack_visual_indexes=[0])
    cfg = T.Qwen3VLConfig(text_config=tc, vision_config=vc)
    m = T.Qwen3VLForConditionalGeneration(cfg)
    torch.manual_seed(0)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
            else:
                p.normal_(1.0 if n.endswith("norm.weight") else 0.0, 0.1)
    sd = {k: v.detach().bfloat16().contiguous() for k, v in m.state_dict().items()}
    d = tmp_path / "q3vl"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(cfg.to_dict()))
    save_file(sd, str(d / "model.safetensors"))
    llm = load(str(d), device=cuda, engine_config=EngineConfig(max_num_seqs=2, max_model_len=128, num_blocks=32))
    prompt = torch.randint(0, 500, (30,), generator=torch.Generator().manual_seed(3)).tolist()
    out = llm.generate(prompt, SamplingParams(max_new_tokens=4, ignore_eos=True))[0].token_ids
    oracle = DecoderOracle(llm.config, {k: v.float() for k, v in LanguageModelView(sd).as_dict().items()})
    lg, _ = oracle.forward(torch.tensor(prompt + out[:-1]))
    for t, r in zip(out, lg[len(prompt) - 1:]):
        assert r[t] >= r.max() - 0.05 * (r.max() - r.min())
