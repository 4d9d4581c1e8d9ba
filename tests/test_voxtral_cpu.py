"""Voxtral on CPU against transformers' VoxtralForConditionalGeneration (the
fp32 oracle): projected audio tokens (Whisper encoder + frame-group projector)
and the LM logits of a prompt whose audio placeholders receive them, one or
two audio windows, placeholders split across two runs."""
import pytest
import torch

from rlx_models_b200.models.voxtral import VoxtralConfig, VoxtralModel

transformers = pytest.importorskip("transformers")

AC = dict(model_type="voxtral_encoder", num_mel_bins=16, d_model=32, encoder_layers=2, encoder_attention_heads=4,
          encoder_ffn_dim=64, max_source_positions=20)
TC = dict(model_type="llama", vocab_size=64, hidden_size=48, intermediate_size=96, num_hidden_layers=2,
          num_attention_heads=4, num_key_value_heads=2, head_dim=12)


@pytest.fixture(scope="module")
def pair():
    torch.manual_seed(0)
    hc = transformers.VoxtralConfig(audio_config=AC, text_config=TC, audio_token_id=60)
    hm = transformers.VoxtralForConditionalGeneration(hc).eval()
    sd = {k: v + 0.05 * torch.randn_like(v) for k, v in hm.state_dict().items()}
    hm.load_state_dict(sd)
    return hc, hm, sd, VoxtralModel(VoxtralConfig.from_dict(hc.to_dict()), sd)


@pytest.mark.parametrize("windows,ids", [
    (1, [1, 5, 7] + [60] * 10 + [9, 11, 2]),
    (2, [1] + [60] * 10 + [3, 4] + [60] * 10 + [8]),
])
def test_logits_match_transformers(pair, windows, ids):
    _, hm, _, m = pair
    mel = torch.randn(windows, 16, 40)
    with torch.no_grad():
        ref = hm(input_ids=torch.tensor([ids]), input_features=mel).logits[0]
    lg = m.oracle_logits(ids, mel)
    torch.testing.assert_close(lg, ref, atol=1e-4, rtol=1e-4)


def test_placeholder_count_is_checked(pair):
    _, _, _, m = pair
    with pytest.raises(ValueError):
        m.mm_segments([1] + [60] * 9 + [2], torch.randn(1, 16, 40))
