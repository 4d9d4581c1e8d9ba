"""FLUX text encoders on CPU against the transformers implementations of the
same architectures (tiny random configs, HF tensor names)."""
import pytest
import torch

transformers = pytest.importorskip("transformers")

from rlx_models_b200.models.flux_text import (CLIPTextConfig, CLIPTextEncoder, T5Config, T5Encoder,  # noqa: E402
                                              relative_position_bucket)


def test_t5_encoder_matches_transformers():
    from transformers import T5Config as HC, T5EncoderModel
    hc = HC(vocab_size=300, d_model=64, d_kv=16, d_ff=96, num_layers=3, num_heads=4,
            relative_attention_num_buckets=32, relative_attention_max_distance=128,
            feed_forward_proj="gated-gelu", dropout_rate=0.0)
    torch.manual_seed(0)
    ref = T5EncoderModel(hc).eval()
    sd = {k: v.detach().clone() for k, v in ref.state_dict().items()}
    ours = T5Encoder(T5Config.from_dict(hc.to_dict()), sd)
    ids = torch.randint(0, 300, (2, 40))
    with torch.no_grad():
        want = ref(input_ids=ids).last_hidden_state
    got = ours(ids)
    assert torch.allclose(got, want, atol=1e-4, rtol=1e-4), (got - want).abs().max()


def test_relative_position_buckets():
    from transformers.models.t5.modeling_t5 import T5Attention
    rel = torch.arange(-300, 300)[None, :]
    want = T5Attention._relative_position_bucket(rel, bidirectional=True, num_buckets=32, max_distance=128)
    assert torch.equal(relative_position_bucket(rel, 32, 128), want)


@pytest.mark.parametrize("eos", [2, 7])
def test_clip_text_matches_transformers(eos):
    from transformers import CLIPTextConfig as HC, CLIPTextModel
    hc = HC(vocab_size=100, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
            max_position_embeddings=20, eos_token_id=eos, hidden_act="quick_gelu")
    torch.manual_seed(1)
    ref = CLIPTextModel(hc).eval()
    sd = {k: v.detach().clone() for k, v in ref.state_dict().items()}
    ours = CLIPTextEncoder(CLIPTextConfig.from_dict(hc.to_dict()), sd)
    ids = torch.randint(8, 90, (3, 20))
    ids[:, 12] = eos if eos != 2 else 99  # an end-of-text token
    with torch.no_grad():
        out = ref(input_ids=ids)
    h, pooled = ours(ids)
    assert torch.allclose(h, out.last_hidden_state, atol=1e-4)
    assert torch.allclose(pooled, out.pooler_output, atol=1e-4)
