"""Text paths of multimodal checkpoints (Qwen3-VL dense and MoE, Gemma-3):
the language model (``model.language_model.*``, fused expert banks) through
the decoder's config and names, against transformers on text-only input."""
import math

import pytest
import torch


def _rand(m):
    torch.manual_seed(0)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
            else:
                p.normal_(1.0 if n.endswith("norm.weight") else 0.0, 0.1)
    return m.eval()


@pytest.mark.parametrize("moe", [False, True])
def test_qwen3_vl_text_matches_transformers(moe):
    import transformers as T
    from rlx_models_b200.config import DecoderConfig
    from rlx_models_b200.models.oracle import DecoderOracle
    from rlx_models_b200.weights.aliases import LanguageModelView
    tc = dict(vocab_size=128, hidden_size=64, intermediate_size=96, num_hidden_layers=2, num_attention_heads=4,
              num_key_value_heads=2, head_dim=16, tie_word_embeddings=False,
              rope_parameters={"rope_type": "default", "rope_theta": 1e6, "mrope_section": [2, 3, 3],
                               "mrope_interleaved": True})
    vc = dict(depth=1, hidden_size=32, intermediate_size=64, num_heads=2, out_hidden_size=64,
              deepstack_visual_indexes=[0])
    if moe:
        tc.update(num_experts=4, num_experts_per_tok=2, moe_intermediate_size=32, decoder_sparse_step=1)
        cfg = T.Qwen3VLMoeConfig(text_config=tc, vision_config=vc)
        m = _rand(T.Qwen3VLMoeForConditionalGeneration(cfg))
    else:
        cfg = T.Qwen3VLConfig(text_config=tc, vision_config=vc)
        m = _rand(T.Qwen3VLForConditionalGeneration(cfg))
    ids = torch.randint(0, 120, (1, 17), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        ref = m(input_ids=ids).logits[0]
    dc = DecoderConfig.from_hf_dict(cfg.to_dict())
    assert dc.model_type == ("qwen3_moe" if moe else "qwen3") and dc.qk_norm and dc.rope_scaling is None
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    assert LanguageModelView.applies(sd)
    o = DecoderOracle(dc, LanguageModelView(sd).as_dict())
    lg, _ = o.forward(ids[0])
    assert (lg - ref).abs().max() < 1e-3, (lg - ref).abs().max()


def test_gemma3_multimodal_text_matches_transformers():
    import transformers as T
    from rlx_models_b200.config import DecoderConfig
    from rlx_models_b200.models.oracle import DecoderOracle
    from rlx_models_b200.weights.aliases import LanguageModelView
    tc = dict(vocab_size=300, hidden_size=64, intermediate_size=96, num_hidden_layers=2, num_attention_heads=4,
              num_key_value_heads=2, head_dim=16, sliding_window=8)
    vc = dict(hidden_size=32, intermediate_size=64, num_hidden_layers=1, num_attention_heads=2, image_size=28,
              patch_size=14)
    cfg = T.Gemma3Config(text_config=tc, vision_config=vc, mm_tokens_per_image=4, image_token_index=299)
    m = _rand(T.Gemma3ForConditionalGeneration(cfg))
    ids = torch.randint(0, 290, (1, 19), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = m(input_ids=ids).logits[0]
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    o = DecoderOracle(DecoderConfig.from_hf_dict(cfg.to_dict()), LanguageModelView(sd).as_dict())
    lg, _ = o.forward(ids[0])
    assert (lg - ref).abs().max() < 1e-3
