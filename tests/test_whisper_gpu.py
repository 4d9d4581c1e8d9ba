"""Whisper on the GPU (bf16 GEMMs on the tcgen05 linear) against the fp32 CPU
path of the same model."""
import pytest
import torch

from rlx_models_b200.models import whisper as W

pytestmark = pytest.mark.gpu


def test_whisper_gpu_matches_cpu(cuda):
    cfg = W.WhisperConfig(vocab_size=512, num_mel_bins=80, d_model=256, encoder_layers=2, decoder_layers=2,
                          encoder_attention_heads=4, decoder_attention_heads=4, encoder_ffn_dim=512,
                          decoder_ffn_dim=512, max_source_positions=100, max_target_positions=64,
                          decoder_start_token_id=500, eos_token_id=501)
    g = torch.Generator().manual_seed(0)
    d = cfg.d_model
    w = {"model.encoder.conv1.weight": torch.randn(d, 80, 3, generator=g) * 0.05,
         "model.encoder.conv1.bias": torch.zeros(d), "model.encoder.conv2.weight": torch.randn(d, d, 3, generator=g) * 0.03,
         "model.encoder.conv2.bias": torch.zeros(d), "model.encoder.embed_positions.weight": W.sinusoids(100, d),
         "model.decoder.embed_tokens.weight": torch.randn(512, d, generator=g) * 0.05,
         "model.decoder.embed_positions.weight": torch.randn(64, d, generator=g) * 0.02}
    for side, n, x in (("encoder", cfg.encoder_layers, False), ("decoder", cfg.decoder_layers, True)):
        p = f"model.{side}."
        w[p + "layer_norm.weight"], w[p + "layer_norm.bias"] = torch.ones(d), torch.zeros(d)
        for i in range(n):
            q = f"{p}layers.{i}."
            atts = ["self_attn"] + (["encoder_attn"] if x else [])
            for a in atts:
                for m in "qkvo":
                    nm = "out_proj" if m == "o" else f"{m}_proj"
                    w[f"{q}{a}.{nm}.weight"] = torch.randn(d, d, generator=g) * 0.05
                    if m != "k":
                        w[f"{q}{a}.{nm}.bias"] = torch.zeros(d)
                lnn = "self_attn_layer_norm" if a == "self_attn" else "encoder_attn_layer_norm"
                w[q + lnn + ".weight"], w[q + lnn + ".bias"] = torch.ones(d), torch.zeros(d)
            w[q + "final_layer_norm.weight"], w[q + "final_layer_norm.bias"] = torch.ones(d), torch.zeros(d)
            w[q + "fc1.weight"], w[q + "fc1.bias"] = torch.randn(512, d, generator=g) * 0.05, torch.zeros(512)
            w[q + "fc2.weight"], w[q + "fc2.bias"] = torch.randn(d, 512, generator=g) * 0.05, torch.zeros(d)
    cpu = W.WhisperModel(cfg, w)
    gpu = W.WhisperModel(cfg, w, device=cuda)
    audio = torch.randn(16000 * 2, generator=g) * 0.1
    mel = W.log_mel(audio, 80, pad_to=2 * cfg.max_source_positions * W.HOP).unsqueeze(0)
    ids = torch.tensor([[500, 7, 9, 11]])
    lc, _ = cpu.decode(ids, cpu.cross_kv(cpu.encode(mel)))
    lg, _ = gpu.decode(ids, gpu.cross_kv(gpu.encode(mel)))
    rel = ((lg.cpu() - lc).norm() / lc.norm()).item()
    assert rel < 3e-2, rel
    toks = W.SpeechToText(gpu).transcribe(audio, max_new_tokens=6)
    assert isinstance(toks, list) and len(toks) <= 6
