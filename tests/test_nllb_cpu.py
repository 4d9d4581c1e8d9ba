"""NLLB / M2M-100 translation on CPU against transformers'
M2M100ForConditionalGeneration (the fp32 oracle): encoder states of a padded
batch, teacher-forced decoder logits (one prompt pass, then token by token
through the K / V cache), and greedy generation with a forced target-language
token."""
import pytest
import torch

from rlx_models_b200.models.nllb import NllbConfig, NllbTranslator

transformers = pytest.importorskip("transformers")


@pytest.fixture(scope="module")
def pair():
    torch.manual_seed(0)
    hc = transformers.M2M100Config(vocab_size=96, d_model=64, encoder_layers=2, decoder_layers=2,
                                   encoder_attention_heads=4, decoder_attention_heads=4, encoder_ffn_dim=128,
                                   decoder_ffn_dim=128, max_position_embeddings=64, dropout=0.0,
                                   attention_dropout=0.0, activation_dropout=0.0)
    hm = transformers.M2M100ForConditionalGeneration(hc).eval()
    sd = {k: (v + 0.02 * torch.randn_like(v)) if v.dtype.is_floating_point and "embed_positions" not in k else v
          for k, v in hm.state_dict().items()}
    sd["lm_head.weight"] = sd["model.shared.weight"]
    sd["model.encoder.embed_tokens.weight"] = sd["model.shared.weight"]
    sd["model.decoder.embed_tokens.weight"] = sd["model.shared.weight"]
    hm.load_state_dict(sd, strict=False)
    return hm, NllbTranslator(NllbConfig.from_dict(hc.to_dict()), {k: v for k, v in sd.items()
                                                                    if "embed_positions" not in k})


def test_encoder_and_teacher_forced_logits(pair):
    hm, m = pair
    src = torch.tensor([[5, 17, 33, 40, 2], [9, 12, 2, 1, 1]])
    am = src.ne(1).long()
    tgt = torch.tensor([[2, 50, 7, 8, 9], [2, 50, 11, 12, 13]])
    with torch.no_grad():
        enc_ref = hm.model.encoder(input_ids=src, attention_mask=am).last_hidden_state
        ref = hm(input_ids=src, attention_mask=am, decoder_input_ids=tgt).logits
    enc, mask = m.encode(src)
    torch.testing.assert_close(enc[0], enc_ref[0], atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(enc[1, :3], enc_ref[1, :3], atol=1e-4, rtol=1e-4)
    cross = m.cross_kv(enc)
    cache = []
    lg = m.decode_step(tgt[:, :3], 0, cache, cross, mask)
    torch.testing.assert_close(lg, ref[:, :3], atol=1e-4, rtol=1e-4)
    for t in range(3, 5):
        lg = m.decode_step(tgt[:, t:t + 1], t, cache, cross, mask)
        torch.testing.assert_close(lg[:, 0], ref[:, t], atol=1e-4, rtol=1e-4)


def test_greedy_generation_with_forced_language(pair):
    hm, m = pair
    src = torch.tensor([[5, 17, 33, 40, 2], [9, 12, 2, 1, 1]])
    with torch.no_grad():
        ref = hm.generate(input_ids=src, attention_mask=src.ne(1).long(), forced_bos_token_id=60, max_new_tokens=12,
                          do_sample=False, num_beams=1)
    got = m.generate(src, forced_bos=60, max_new_tokens=12)
    for b in range(2):
        want = [int(t) for t in ref[b, 1:]]
        while want and want[-1] == 1:
            want.pop()
        assert got[b] == want[:len(got[b])] and len(got[b]) >= min(len(want), 11)


def test_load_translator_ids(pair, tmp_path):
    import json

    from rlx_models_b200.api import load_translator
    from rlx_models_b200.weights.safetensors_io import save_file
    hm, m = pair
    d = tmp_path / "nllb"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(hm.config.to_dict()))
    save_file({k: v.contiguous() for k, v in hm.state_dict().items() if "embed_positions" not in k},
              str(d / "model.safetensors"))
    tr = load_translator(str(d), device="cpu")
    src = torch.tensor([[5, 17, 33, 40, 2]])
    assert tr.model.generate(src, forced_bos=60, max_new_tokens=6) == m.generate(src, forced_bos=60, max_new_tokens=6)
    with pytest.raises(ValueError):
        tr.translate("hello", "eng_Latn", "fra_Latn")
