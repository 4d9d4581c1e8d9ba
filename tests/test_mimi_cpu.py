"""Mimi on CPU against transformers' MimiModel (the fp32 oracle): latents after
the SEANet encoder, the sliding-window Transformer and the downsampling conv;
split-RVQ codes at full and reduced depth; decoded audio; ``load_codec``."""
import json

import pytest
import torch

from rlx_models_b200.models.mimi import MimiConfig, MimiModel

transformers = pytest.importorskip("transformers")

SMALL = dict(hidden_size=32, num_filters=8, upsampling_ratios=[4, 2], codebook_size=16, codebook_dim=16,
             num_quantizers=4, vector_quantization_hidden_dimension=16, upsample_groups=32, num_hidden_layers=2,
             intermediate_size=64, num_attention_heads=4, num_key_value_heads=4, head_dim=8, sliding_window=5,
             sampling_rate=800)


@pytest.fixture(scope="module")
def pair():
    torch.manual_seed(0)
    hc = transformers.MimiConfig(**SMALL)
    hm = transformers.MimiModel(hc).eval()
    sd = {}
    for k, v in hm.state_dict().items():
        if v.dtype.is_floating_point:
            v = v + 0.1 * torch.randn_like(v)
            if k.endswith("cluster_usage"):
                v = v.abs() + 0.5
        sd[k] = v
    hm.load_state_dict(sd)
    return hc, hm, sd, MimiModel(MimiConfig.from_dict(hc.to_dict()), sd)


def test_latents_codes_audio(pair):
    _, hm, _, m = pair
    x = 0.3 * torch.randn(2, 1, 320)
    with torch.no_grad():
        emb = hm.encoder(x)
        et = hm.encoder_transformer(emb.transpose(1, 2))[0]
        z_ref = hm.downsample(et.transpose(1, 2)).transpose(1, 2)
        out = hm.encode(x)
        out2 = hm.encode(x, num_quantizers=2)
        a_ref = hm.decode(out.audio_codes).audio_values
    z = m.encode_latents(x)
    torch.testing.assert_close(z, z_ref, atol=1e-4 * z_ref.abs().max().item(), rtol=1e-4)
    assert torch.equal(m.encode(x), out.audio_codes)
    assert torch.equal(m.encode(x, num_quantizers=2), out2.audio_codes)
    a = m.decode(out.audio_codes)
    torch.testing.assert_close(a, a_ref, atol=1e-4 * a_ref.abs().max().item(), rtol=1e-4)


def test_load_codec_mimi(pair, tmp_path):
    from rlx_models_b200.api import load_codec
    from rlx_models_b200.weights.safetensors_io import save_file
    hc, _, sd, m = pair
    d = tmp_path / "mimi"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(hc.to_dict()))
    save_file({k: v.contiguous() for k, v in sd.items()}, str(d / "model.safetensors"))
    codec = load_codec(str(d), device="cpu")
    assert isinstance(codec, MimiModel)
    x = 0.3 * torch.randn(1, 1, 160)
    assert torch.equal(codec.encode(x), m.encode(x))
