"""Moonshine on CPU against transformers MoonshineForConditionalGeneration:
encoder states from raw audio, teacher-forced decoder logits (incremental, with
the self-attention cache), greedy transcription ids."""
import math

import torch


def _model():
    import transformers as T
    cfg = T.MoonshineConfig(vocab_size=96, hidden_size=64, intermediate_size=96, encoder_num_hidden_layers=2,
                            decoder_num_hidden_layers=2, encoder_num_attention_heads=4,
                            decoder_num_attention_heads=4, encoder_num_key_value_heads=4,
                            decoder_num_key_value_heads=4, decoder_start_token_id=1, eos_token_id=2,
                            bos_token_id=1, pad_token_id=0)
    m = T.MoonshineForConditionalGeneration(cfg).eval()
    torch.manual_seed(0)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p[0].numel()))
            else:
                p.normal_(1.0 if "norm" in n and n.endswith("weight") else 0.0, 0.1)
    return cfg, m


def test_moonshine_matches_transformers():
    from rlx_models_b200.models.moonshine import MoonshineConfig, MoonshineModel
    hc, m = _model()
    audio = torch.randn(2, 16000, generator=torch.Generator().manual_seed(1)) * 0.3
    ids = torch.tensor([[1, 5, 9, 33, 7, 60], [1, 8, 8, 41, 3, 12]])
    with torch.no_grad():
        ref = m(input_values=audio, decoder_input_ids=ids)
    mm = MoonshineModel(MoonshineConfig.from_dict(hc.to_dict()), {k: v.detach() for k, v in m.state_dict().items()})
    enc = mm.encode(audio)
    assert (enc - ref.encoder_last_hidden_state).abs().max() < 1e-4
    cross = mm._cross_kv(enc)
    cache = [None] * 2
    a = mm.decode_step(ids[:, :4], 0, cache, cross)
    b = mm.decode_step(ids[:, 4:], 4, cache, cross)
    lg = torch.cat([a, b], 1)
    assert (lg - ref.logits).abs().max() < 1e-3
    with torch.no_grad():
        gen = m.generate(input_values=audio[:1], max_new_tokens=8, do_sample=False)[0].tolist()
    exp = [t for t in gen[1:] if t not in (0,)]
    if 2 in exp:
        exp = exp[:exp.index(2)]
    assert mm.greedy(audio[:1], max_new_tokens=8)[0] == exp[:8]
