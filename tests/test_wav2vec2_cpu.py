"""wav2vec 2.0 CTC on CPU against transformers' Wav2Vec2ForCTC (the fp32
oracle): the "group"-norm post-norm layout and the "layer"-norm stable-layer-norm
layout, a padded batch with an attention mask, greedy CTC decoding, the
channels-last GELU-fused conv front end against F.conv1d, and the transcriber
through ``load_transcriber``."""
import json

import pytest
import torch

from rlx_models_b200.models.wav2vec2 import Wav2Vec2Config, Wav2Vec2CTC

transformers = pytest.importorskip("transformers")

SMALL = dict(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, intermediate_size=128, conv_dim=[32] * 7,
             num_conv_pos_embeddings=16, num_conv_pos_embedding_groups=4, vocab_size=20)
LAYOUTS = {"group_postnorm": {}, "layer_stable": dict(feat_extract_norm="layer", do_stable_layer_norm=True,
                                                        conv_bias=True)}


def _pair(kw, seed=0):
    torch.manual_seed(seed)
    hc = transformers.Wav2Vec2Config(**SMALL, **kw)
    hm = transformers.Wav2Vec2ForCTC(hc).eval()
    sd = {k: (v + 0.05 * torch.randn_like(v)) if v.dtype.is_floating_point else v for k, v in hm.state_dict().items()}
    hm.load_state_dict(sd)
    return hc, hm, sd, Wav2Vec2CTC(Wav2Vec2Config.from_dict(hc.to_dict()), sd)


@pytest.mark.parametrize("layout", list(LAYOUTS))
def test_logits_match_transformers(layout):
    _, hm, _, m = _pair(LAYOUTS[layout])
    x = torch.randn(2, 4000)
    with torch.no_grad():
        ref = hm(x).logits
    lg, n = m.logits(x)
    torch.testing.assert_close(lg, ref, atol=1e-4, rtol=1e-4)
    assert n.tolist() == [ref.shape[1]] * 2
    greedy = m.greedy(x)
    ids = ref.argmax(-1)
    for b in range(2):
        want = [int(t) for i, t in enumerate(ids[b]) if (i == 0 or t != ids[b][i - 1]) and int(t) != 0]
        assert greedy[b] == want


def test_padded_batch_with_mask():
    _, hm, _, m = _pair(LAYOUTS["layer_stable"], seed=1)
    x = torch.randn(2, 4000)
    x[1, 2500:] = 0
    am = torch.ones(2, 4000, dtype=torch.long)
    am[1, 2500:] = 0
    with torch.no_grad():
        ref = hm(x, attention_mask=am).logits
    lg, n = m.logits(x, lengths=[4000, 2500])
    assert n.tolist() == [12, 7]
    torch.testing.assert_close(lg[0], ref[0], atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(lg[1, :7], ref[1, :7], atol=1e-4, rtol=1e-4)


def test_load_transcriber_wav2vec2(tmp_path):
    from rlx_models_b200.api import load_transcriber
    from rlx_models_b200.models.wav2vec2 import Wav2Vec2Transcriber
    from rlx_models_b200.weights.safetensors_io import save_file
    hc, _, sd, m = _pair({}, seed=2)
    d = tmp_path / "w2v"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(hc.to_dict()))
    save_file({k: v.contiguous() for k, v in sd.items()}, str(d / "model.safetensors"))
    tr = load_transcriber(str(d), device="cpu")
    assert isinstance(tr, Wav2Vec2Transcriber)
    audio = torch.randn(8000)
    a = (audio - audio.mean()) / torch.sqrt(audio.var(unbiased=False) + 1e-7)
    assert tr.transcribe(audio) == m.greedy(a[None])[0]
