"""Parakeet FastConformer CTC on CPU against transformers ParakeetForCTC:
logits of padded batches (subsampling masks, relative-position attention with
padding, the convolution module's masked frames) and greedy CTC decoding;
log-mel features by their definition."""
import math

import torch


def _rand(m):
    torch.manual_seed(0)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2:
                fan = p[0].numel()
                p.normal_(0, 1 / math.sqrt(fan))
            elif "norm" in n and n.endswith("weight"):
                p.normal_(1.0, 0.1)
            else:
                p.normal_(0.0, 0.1)
        for mod in m.modules():
            if isinstance(mod, torch.nn.BatchNorm1d):
                mod.running_mean.normal_(0, 0.1)
                mod.running_var.uniform_(0.5, 1.5)
    return m.eval()


def _model():
    import transformers as T
    enc = dict(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, intermediate_size=96,
               conv_kernel_size=5, subsampling_factor=8, subsampling_conv_channels=16, num_mel_bins=32,
               max_position_embeddings=512)
    cfg = T.ParakeetCTCConfig(encoder_config=enc, vocab_size=41, pad_token_id=40)
    return cfg, _rand(T.ParakeetForCTC(cfg))


def test_parakeet_ctc_matches_transformers():
    from rlx_models_b200.models.parakeet import ParakeetConfig, ParakeetCTC
    hc, m = _model()
    g = torch.Generator().manual_seed(1)
    feats = torch.randn(2, 96, 32, generator=g)
    mask = torch.ones(2, 96, dtype=torch.long)
    mask[1, 70:] = 0
    with torch.no_grad():
        ref = m(input_features=feats, attention_mask=mask).logits
    pk = ParakeetCTC(ParakeetConfig.from_dict(hc.to_dict()), {k: v.detach() for k, v in m.state_dict().items()})
    lg, n = pk.logits(feats, mask.sum(-1))
    assert lg.shape == ref.shape and n.tolist() == [12, 9]
    assert (lg[0] - ref[0]).abs().max() < 1e-3
    assert (lg[1, :9] - ref[1, :9]).abs().max() < 1e-3  # valid frames of the padded sequence
    # full-length batch without a mask
    with torch.no_grad():
        ref2 = m(input_features=feats[:1]).logits
    assert (pk.logits(feats[:1])[0] - ref2).abs().max() < 1e-3
    seq = pk.greedy(feats[:1])[0]
    best = ref2[0].argmax(-1).tolist()
    exp, prev = [], None
    for t in best:
        if t != prev and t != 40:
            exp.append(t)
        prev = t
    assert seq == exp


def test_log_mel_features_definition():
    from rlx_models_b200.models.parakeet import log_mel_features
    sr = 16000
    t = torch.arange(sr) / sr
    audio = torch.sin(2 * math.pi * 440 * t) + 0.01 * torch.randn(sr, generator=torch.Generator().manual_seed(0))
    f = log_mel_features(audio, sr, 80)
    assert f.shape == (100, 80)  # (16000 + 512 - 512) // 160 valid frames
    assert f.mean(0).abs().max() < 1e-4
    assert (f.std(0) - 1).abs().max() < 1e-3


def test_load_transcriber_parakeet(tmp_path):
    import json
    from rlx_models_b200.api import load_transcriber
    from rlx_models_b200.models.parakeet import ParakeetConfig, ParakeetCTC, log_mel_features
    from rlx_models_b200.weights.safetensors_io import save_file
    hc, m = _model()
    hc2 = hc.to_dict()
    hc2["encoder_config"]["num_mel_bins"] = 80
    import transformers as T
    cfg = T.ParakeetCTCConfig(**{k: v for k, v in hc2.items() if k in ("encoder_config", "vocab_size", "pad_token_id")})
    m = _rand(T.ParakeetForCTC(cfg))
    d = tmp_path / "pk"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(cfg.to_dict()))
    save_file({k: v.detach().contiguous() for k, v in m.state_dict().items()}, str(d / "model.safetensors"))
    tr = load_transcriber(str(d), device="cpu")
    audio = torch.randn(8000, generator=torch.Generator().manual_seed(2))
    ids = tr.transcribe(audio, 16000)
    feats = log_mel_features(audio, 16000, 80)
    with torch.no_grad():
        ref = m(input_features=feats[None]).logits[0].argmax(-1).tolist()
    exp, prev = [], None
    for t in ref:
        if t != prev and t != 40:
            exp.append(t)
        prev = t
    assert ids == exp
