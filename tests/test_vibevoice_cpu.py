"""VibeVoice-ASR on CPU against transformers VibeVoiceAsrForConditionalGeneration
(vae_std 0, so its acoustic sampling is the mean): the two causal ConvNeXt
tokenizer encoders, the summed speech connectors, and the logits of a prompt
whose audio-token run carries the features; a signal longer than the model's
chunk size (streamed with padding caches there, one causal pass here)."""
import math

import pytest
import torch

AUD = 90


def _rand(m):
    torch.manual_seed(0)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p[0].numel()))
            elif "gamma" in n:
                p.normal_(0.5, 0.1)
            else:
                p.normal_(1.0 if "norm" in n else 0.0, 0.1)
    return m.eval()


def _model(chunk):
    import transformers as T
    enc = dict(num_filters=8, downsampling_ratios=[2, 3], depths=[1, 2, 1], kernel_size=5, hidden_size=12,
               vae_std=0.0, ffn_expansion=2)
    tc = dict(model_type="qwen2", vocab_size=96, hidden_size=64, intermediate_size=96, num_hidden_layers=2,
              num_attention_heads=4, num_key_value_heads=2, rms_norm_eps=1e-6)
    cfg = T.VibeVoiceAsrConfig(acoustic_tokenizer_encoder_config=dict(enc),
                               semantic_tokenizer_encoder_config=dict(enc, hidden_size=20), text_config=tc,
                               audio_token_id=AUD, acoustic_tokenizer_chunk_size=chunk)
    return cfg, _rand(T.VibeVoiceAsrForConditionalGeneration(cfg))


@pytest.mark.parametrize("chunk", [600, 96])
def test_vibevoice_asr_matches_transformers(chunk):
    from rlx_models_b200.models.vibevoice import VibeVoiceAsr, VibeVoiceAsrConfig
    hcfg, m = _model(chunk)
    g = torch.Generator().manual_seed(2)
    audio = torch.randn(1, 1, 360, generator=g)  # hop 6 -> 60 audio tokens
    with torch.no_grad():
        ref_feat = m.get_audio_features(input_values=audio).pooler_output
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    asr = VibeVoiceAsr(VibeVoiceAsrConfig.from_dict(hcfg.to_dict()), sd)
    feat = asr.audio_features(audio[:, 0])
    assert feat.shape == ref_feat.reshape(feat.shape).shape
    assert (feat - ref_feat.reshape(feat.shape)).abs().max() < 1e-4
    text = torch.randint(0, 85, (9,), generator=g).tolist()
    ids = text[:4] + [AUD] * 60 + text[4:]
    with torch.no_grad():
        ref = m(input_ids=torch.tensor([ids]), input_values=audio).logits[0]
    lg = asr.oracle_logits(ids, audio[:, 0])
    assert (lg - ref).abs().max() < 2e-4, (lg - ref).abs().max()
    with pytest.raises(ValueError):
        asr.mm_segments(ids[:-6], audio[:, 0][:, :300])
