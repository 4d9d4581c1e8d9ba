"""Whisper on CPU against the transformers implementation (tiny random
config): log-mel front end, encoder states, decoder logits with a K/V cache,
greedy generation."""
import numpy as np
import pytest
import torch

transformers = pytest.importorskip("transformers")

from rlx_models_b200.models import whisper as W  # noqa: E402


def test_log_mel_matches_feature_extractor():
    from transformers import WhisperFeatureExtractor
    g = np.random.default_rng(0)
    audio = (g.standard_normal(16000 * 3) * 0.1).astype(np.float32)
    fe = WhisperFeatureExtractor(feature_size=80)
    want = fe(audio, sampling_rate=16000, return_tensors="np").input_features[0]
    got = W.log_mel(torch.from_numpy(audio), 80).numpy()
    assert got.shape == want.shape == (80, 3000)
    np.testing.assert_allclose(got, want, atol=2e-4)
    np.testing.assert_allclose(W.mel_filters(80).numpy(), fe.mel_filters.astype(np.float32), atol=1e-6)


def _tiny():
    from transformers import WhisperConfig, WhisperForConditionalGeneration
    hc = WhisperConfig(vocab_size=120, num_mel_bins=16, d_model=64, encoder_layers=2, decoder_layers=2,
                       encoder_attention_heads=4, decoder_attention_heads=4, encoder_ffn_dim=128,
                       decoder_ffn_dim=128, max_source_positions=50, max_target_positions=40,
                       decoder_start_token_id=100, eos_token_id=101, pad_token_id=101, bos_token_id=101)
    torch.manual_seed(0)
    ref = WhisperForConditionalGeneration(hc).eval()
    sd = {k: v.detach().clone() for k, v in ref.state_dict().items()}
    return hc, ref, W.WhisperModel(W.WhisperConfig.from_dict(hc.to_dict()), sd)


def test_encoder_decoder_match_transformers():
    hc, ref, ours = _tiny()
    mel = torch.randn(2, 16, 100)
    ids = torch.randint(0, 100, (2, 7))
    with torch.no_grad():
        out = ref(input_features=mel, decoder_input_ids=ids)
        enc_ref = ref.model.encoder(mel).last_hidden_state
    enc = ours.encode(mel)
    assert torch.allclose(enc, enc_ref, atol=1e-4)
    xkv = ours.cross_kv(enc)
    lg, _ = ours.decode(ids, xkv)
    assert torch.allclose(lg, out.logits, atol=1e-4)
    # incremental decoding with the cache equals one pass
    a, cache = ours.decode(ids[:, :4], xkv)
    b, _ = ours.decode(ids[:, 4:], xkv, cache, 4)
    assert torch.allclose(torch.cat([a, b], 1), lg, atol=1e-4)


def test_greedy_generate_matches_transformers():
    hc, ref, ours = _tiny()
    mel = torch.randn(1, 16, 100)
    prefix = [100, 5, 6]
    toks = ours.generate(mel, prefix, max_new_tokens=12)[0]
    want, ids = [], list(prefix)
    with torch.no_grad():  # plain greedy over the transformers model (no suppression processors)
        for _ in range(12):
            t = int(ref(input_features=mel, decoder_input_ids=torch.tensor([ids])).logits[0, -1].argmax())
            if t == 101:
                break
            want.append(t)
            ids.append(t)
    assert toks == want
    s2t = W.SpeechToText(ours, tokenizer=None)
    out = s2t.transcribe(torch.randn(8000) * 0.1, sample_rate=8000, max_new_tokens=5)
    assert isinstance(out, list) and len(out) <= 5


def test_load_transcriber_from_directory(tmp_path):
    from rlx_models_b200.api import load_transcriber
    from rlx_models_b200.weights.weight_map import WeightMap
    hc, ref, ours = _tiny()
    d = tmp_path / "whisper"
    WeightMap({k: v.detach().clone() for k, v in ref.state_dict().items()}).save(str(d))
    hc.save_pretrained(str(d))
    t = load_transcriber(str(d), device="cpu")
    out = t.transcribe(torch.randn(16000) * 0.1, max_new_tokens=4)
    assert isinstance(out, list) and len(out) <= 4
