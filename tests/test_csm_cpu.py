"""CSM (Sesame) on CPU against transformers' CsmForConditionalGeneration (the
fp32 oracle): greedy frame generation (backbone -> codebook 0 -> depth decoder
for the other codebooks, both with K / V caches), depth-decoder codes for a
given backbone state, and the Mimi decode of the generated frames."""
import pytest
import torch

from rlx_models_b200.models.csm import CsmConfig, CsmModel

transformers = pytest.importorskip("transformers")

CODEC = dict(model_type="mimi", hidden_size=32, num_filters=8, upsampling_ratios=[4, 2], codebook_size=16,
             codebook_dim=16, num_quantizers=4, vector_quantization_hidden_dimension=16, upsample_groups=32,
             num_hidden_layers=1, intermediate_size=64, num_attention_heads=4, num_key_value_heads=4, head_dim=8,
             sliding_window=5, sampling_rate=800)
DEPTH = dict(model_type="csm_depth_decoder_model", num_codebooks=4, backbone_hidden_size=64, vocab_size=16,
             hidden_size=32, intermediate_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
             head_dim=8, max_position_embeddings=5)


@pytest.fixture(scope="module")
def pair():
    torch.manual_seed(0)
    hc = transformers.CsmConfig(num_codebooks=4, vocab_size=16, text_vocab_size=50, hidden_size=64,
                                intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                                num_key_value_heads=2, head_dim=16, codebook_pad_token_id=15, codebook_eos_token_id=0,
                                audio_token_id=48, audio_eos_token_id=49, pad_token_id=48, bos_token_id=1,
                                depth_decoder_config=DEPTH, codec_config=CODEC)
    hm = transformers.CsmForConditionalGeneration(hc).eval()
    sd = {}
    for k, v in hm.state_dict().items():
        if v.dtype.is_floating_point:
            v = v + 0.1 * torch.randn_like(v)
            if k.endswith("cluster_usage"):
                v = v.abs() + 0.5
        sd[k] = v
    sd["depth_decoder.model.embed_tokens.weight"] = sd["backbone_model.embed_tokens.embed_audio_tokens.weight"]
    hm.load_state_dict(sd, strict=False)
    return hm, sd, CsmModel(CsmConfig.from_dict(hc.to_dict()), sd)


@pytest.mark.parametrize("prompt", [[1, 5, 7, 9, 11, 13], [1, 20, 3]])
def test_greedy_frames_match_transformers(pair, prompt):
    hm, _, m = pair
    ids = torch.tensor([prompt])
    with torch.no_grad():
        ref = hm.generate(input_ids=ids, do_sample=False, depth_decoder_do_sample=False, max_new_tokens=6)
    got = m.generate_frames(m.text_prompt(ids), max_frames=6)
    n = min(ref.shape[1], got.shape[1])
    assert n > 0 and torch.equal(got[:, :n], ref[:, :n])


def test_codec_decode_of_frames(pair):
    hm, _, m = pair
    frames = m.generate_frames(m.text_prompt(torch.tensor([[1, 5, 7, 9]])), max_frames=5)[0]
    with torch.no_grad():
        ref = hm.codec_model.decode(frames.t()[None]).audio_values
    torch.testing.assert_close(m.codec.decode(frames.t()[None]), ref, atol=1e-4 * ref.abs().max().item(), rtol=1e-4)


def test_load_speech_generator(pair, tmp_path):
    import json

    from rlx_models_b200.api import load_speech_generator
    from rlx_models_b200.weights.safetensors_io import save_file
    hm, sd, m = pair
    d = tmp_path / "csm"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(hm.config.to_dict()))
    save_file({k: v.contiguous() for k, v in sd.items()}, str(d / "model.safetensors"))
    gen = load_speech_generator(str(d), device="cpu")
    ids = torch.tensor([1, 5, 7, 9])
    audio = gen.model.speak(ids, max_frames=4)
    assert audio.dim() == 1 and audio.numel() > 0 and torch.isfinite(audio).all()
    torch.testing.assert_close(audio, m.speak(ids, max_frames=4))
