"""Voxtral served by the engine on the GPU: projected audio tokens injected at
the placeholder rows (runs crossing prefill chunks), each generated token
checked against the fp32 CPU oracle of the same checkpoint."""
import json
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rand(m):
    torch.manual_seed(0)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p[0].numel()))
            else:
                p.normal_(1.0 if ("norm" in n and n.endswith("weight")) else 0.0, 0.1)
    return m.eval()


def test_voxtral_engine_vs_oracle(cuda, tmp_path):
    import transformers as T
    from rlx_models_b200.api import load_audio_llm
    from rlx_models_b200.models.voxtral import VoxtralConfig, VoxtralModel
    from rlx_models_b200.runtime.engine import EngineConfig, SamplingParams
    from rlx_models_b200.weights.safetensors_io import save_file
    ac = dict(model_type="voxtral_encoder", num_mel_bins=16, d_model=64, encoder_layers=2, encoder_attention_heads=4,
              encoder_ffn_dim=256, max_source_positions=32)
    tc = dict(model_type="llama", vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
              num_attention_heads=4, num_key_value_heads=2, rms_norm_eps=1e-6)
    hcfg = T.VoxtralConfig(audio_config=ac, text_config=tc, audio_token_id=511)
    m = _rand(T.VoxtralForConditionalGeneration(hcfg))
    sd = {k: v.detach().contiguous() for k, v in m.state_dict().items()}
    d = tmp_path / "voxtral"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(hcfg.to_dict()))
    save_file({k: v.bfloat16() for k, v in sd.items()}, str(d / "model.safetensors"))
    llm = load_audio_llm(str(d), device=cuda, engine_config=EngineConfig(max_num_seqs=4, max_model_len=256,
                                                                         num_blocks=64, chunk_size=16))
    g = torch.Generator().manual_seed(3)
    mels = [torch.randn(1, 16, 64, generator=g), torch.randn(2, 16, 64, generator=g)]
    t = lambda n: torch.randint(0, 500, (n,), generator=g).tolist()  # noqa: E731
    n_tok = 8                                   # 32 frames / 4 per group
    prompts = [t(5) + [511] * n_tok + t(9), t(3) + [511] * (2 * n_tok) + t(7)]
    outs = llm.generate(prompts, mels, SamplingParams(max_new_tokens=6, ignore_eos=True))
    oracle = VoxtralModel(VoxtralConfig.from_dict(hcfg.to_dict()), {k: v.bfloat16().float() for k, v in sd.items()})
    for p, mel, o in zip(prompts, mels, outs):
        lg = oracle.oracle_logits(p + o.token_ids[:-1], mel)[len(p) - 1:]
        for tok, r in zip(o.token_ids, lg):
            assert r[tok] >= r.max() - 0.05 * (r.max() - r.min()), (tok, int(r.argmax()))
