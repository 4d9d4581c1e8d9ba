"""LLaVA-form VLM served by the engine on the GPU: image features injected at
the placeholder rows (also when chunked prefill splits an image's run), each
generated token checked against the fp32 CPU oracle of the same checkpoint."""
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


def test_llava_engine_vs_oracle(cuda, tmp_path):
    import transformers as T
    from rlx_models_b200.api import load_vlm
    from rlx_models_b200.models.llava import LlavaConfig, LlavaVLM
    from rlx_models_b200.runtime.engine import EngineConfig, SamplingParams
    from rlx_models_b200.weights.safetensors_io import save_file
    vc = dict(model_type="clip_vision_model", hidden_size=64, intermediate_size=128, num_hidden_layers=3,
              num_attention_heads=4, image_size=28, patch_size=7)
    tc = dict(model_type="llama", vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
              num_attention_heads=4, num_key_value_heads=2, rms_norm_eps=1e-6)
    hcfg = T.LlavaConfig(vision_config=vc, text_config=tc, image_token_index=511)
    m = _rand(T.LlavaForConditionalGeneration(hcfg))
    sd = {k: v.detach().contiguous() for k, v in m.state_dict().items()}
    d = tmp_path / "llava"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(hcfg.to_dict()))
    save_file({k: v.bfloat16() for k, v in sd.items()}, str(d / "model.safetensors"))
    vlm = load_vlm(str(d), device=cuda, engine_config=EngineConfig(max_num_seqs=4, max_model_len=256,
                                                                   num_blocks=64, chunk_size=16))
    n_img = vlm.image_tokens
    assert n_img == 16
    g = torch.Generator().manual_seed(3)
    px = [torch.randn(1, 3, 28, 28, generator=g), torch.randn(2, 3, 28, 28, generator=g)]
    t = lambda n: torch.randint(0, 500, (n,), generator=g).tolist()  # noqa: E731
    prompts = [t(5) + [511] * n_img + t(9),
               t(3) + [511] * n_img + t(20) + [511] * n_img + t(2)]  # runs cross 16-token prefill chunks
    outs = vlm.generate(prompts, px, SamplingParams(max_new_tokens=6, ignore_eos=True))
    oracle = LlavaVLM(LlavaConfig.from_dict(hcfg.to_dict()), {k: v.bfloat16().float() for k, v in sd.items()})
    for p, im, o in zip(prompts, px, outs):
        lg = oracle.oracle_logits(p + o.token_ids[:-1], im)[len(p) - 1:]
        for tok, r in zip(o.token_ids, lg):
            assert r[tok] >= r.max() - 0.05 * (r.max() - r.min()), (tok, int(r.argmax()))
