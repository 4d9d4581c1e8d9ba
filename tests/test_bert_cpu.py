"""BERT encoder embeddings on CPU against transformers' BertModel."""
import pytest
import torch

transformers = pytest.importorskip("transformers")

from rlx_models_b200.models.bert import BertConfig, BertEncoder  # noqa: E402


def test_bert_matches_transformers():
    from transformers import BertConfig as HC, BertModel
    hc = HC(vocab_size=200, hidden_size=64, num_hidden_layers=2, num_attention_heads=4, intermediate_size=128,
            max_position_embeddings=64, hidden_dropout_prob=0.0, attention_probs_dropout_prob=0.0)
    torch.manual_seed(0)
    ref = BertModel(hc).eval()
    sd = {k: v.detach().clone() for k, v in ref.state_dict().items()}
    enc = BertEncoder(BertConfig.from_dict(hc.to_dict()), sd)
    ids = torch.randint(5, 200, (3, 20))
    mask = torch.ones(3, 20, dtype=torch.long)
    mask[1, 12:] = 0
    mask[2, 5:] = 0
    with torch.no_grad():
        out = ref(input_ids=ids, attention_mask=mask)
    h = enc(ids, mask)
    valid = mask.bool()
    assert torch.allclose(h[valid], out.last_hidden_state[valid], atol=1e-4)
    pooled = enc.embed(ids, mask, pooling="pooler", normalize=False)
    assert torch.allclose(pooled, out.pooler_output, atol=1e-4)
    mean = enc.embed(ids, mask, pooling="mean")
    want = (out.last_hidden_state * mask[..., None]).sum(1) / mask.sum(1, keepdim=True)
    assert torch.allclose(mean, torch.nn.functional.normalize(want, dim=-1), atol=1e-4)
    # prefixed task-model names ("bert.") load too
    enc2 = BertEncoder(BertConfig.from_dict(hc.to_dict()), {"bert." + k: v for k, v in sd.items()})
    assert torch.allclose(enc2(ids, mask)[valid], h[valid])


def test_load_embedder_from_directory(tmp_path):
    from transformers import BertConfig as HC, BertModel
    from rlx_models_b200.api import load_embedder
    from rlx_models_b200.weights.weight_map import WeightMap
    hc = HC(vocab_size=100, hidden_size=32, num_hidden_layers=1, num_attention_heads=4, intermediate_size=64,
            max_position_embeddings=32)
    ref = BertModel(hc).eval()
    d = tmp_path / "bert"
    WeightMap({k: v.detach().clone() for k, v in ref.state_dict().items()}).save(str(d))
    hc.save_pretrained(str(d))
    emb = load_embedder(str(d), device="cpu")
    e = emb.embed([[3, 4, 5], [6, 7, 8, 9, 10]])
    assert e.shape == (2, 32) and torch.allclose(e.norm(dim=-1), torch.ones(2), atol=1e-5)


def test_nomic_bert_matches_transformers(tmp_path):
    """NomicBERT (rotary, SwiGLU, post-norms) == transformers NomicBertModel on a
    padded batch, and load_embedder picks it from config.json."""
    import math
    from transformers import NomicBertConfig as HFC, NomicBertModel
    from rlx_models_b200.models.bert import NomicBertConfig, NomicBertEncoder
    hc = HFC(vocab_size=100, hidden_size=64, num_hidden_layers=2, num_attention_heads=4, intermediate_size=96,
             max_position_embeddings=64)
    torch.manual_seed(0)
    m = NomicBertModel(hc).eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
            else:
                p.normal_(1.0 if n.endswith("weight") else 0.0, 0.1)
    ids = torch.randint(1, 100, (2, 11), generator=torch.Generator().manual_seed(1))
    mask = torch.ones(2, 11, dtype=torch.long)
    mask[1, 7:] = 0
    with torch.no_grad():
        ref = m(input_ids=ids, attention_mask=mask).last_hidden_state
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    enc = NomicBertEncoder(NomicBertConfig.from_dict(hc.to_dict()), sd)
    got = enc(ids, mask)
    keep = mask.bool()
    assert (got[keep] - ref[keep]).abs().max() < 1e-4
    e = enc.embed(ids, mask, pooling="mean")
    assert torch.allclose(e.norm(dim=-1), torch.ones(2), atol=1e-5)


def test_eurobert_bidirectional_trunk(tmp_path):
    """EuroBERT (Llama-shaped trunk with bidirectional attention): the decoder
    oracle with causal=False == transformers EuroBertModel, and
    load_embedder builds a DecoderEmbedder over a saved checkpoint."""
    import json
    import math
    from transformers import EuroBertConfig, EuroBertModel
    from rlx_models_b200.api import DecoderEmbedder, load_embedder
    from rlx_models_b200.weights.safetensors_io import save_file
    hc = EuroBertConfig(vocab_size=128, hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                        num_key_value_heads=2, intermediate_size=96, pad_token_id=0, bos_token_id=1, eos_token_id=2)
    torch.manual_seed(0)
    m = EuroBertModel(hc).eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p.shape[-1]))
            else:
                p.normal_(1.0, 0.1)
    d = tmp_path / "eb"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(hc.to_dict()))
    save_file({k: v.detach().contiguous() for k, v in m.state_dict().items()}, str(d / "model.safetensors"))
    emb = load_embedder(str(d), device="cpu", pooling="mean")
    assert isinstance(emb, DecoderEmbedder) and not emb.cfg.causal
    ids = torch.randint(3, 128, (2, 13), generator=torch.Generator().manual_seed(1))
    mask = torch.ones(2, 13, dtype=torch.long)
    mask[1, 9:] = 0
    with torch.no_grad():
        ref = m(input_ids=ids, attention_mask=mask).last_hidden_state
    got = emb(ids, mask)
    keep = mask.bool()
    assert (got[keep] - ref[keep]).abs().max() < 1e-4
    e = emb.embed([ids[0].tolist(), ids[1, :9].tolist()])
    r = torch.stack([ref[0].mean(0), ref[1, :9].mean(0)])
    assert torch.allclose(e, torch.nn.functional.normalize(r, dim=-1), atol=1e-4)


def test_embeddinggemma_trunk_and_dense_head(tmp_path):
    """EmbeddingGemma: the Gemma-3 trunk with bidirectional attention (sliding
    layers see |q - k| < window // 2 + 1), mean pooling and the
    sentence-transformers Dense stack, against transformers on CPU."""
    import json
    import math
    from transformers import Gemma3TextConfig, Gemma3TextModel
    from rlx_models_b200.api import DecoderEmbedder, load_embedder
    from rlx_models_b200.weights.safetensors_io import save_file
    kw = dict(vocab_size=128, hidden_size=64, intermediate_size=96, num_hidden_layers=3, num_attention_heads=4,
              num_key_value_heads=1, head_dim=16, sliding_window=8, use_bidirectional_attention=True,
              layer_types=["sliding_attention", "sliding_attention", "full_attention"], query_pre_attn_scalar=16)
    m = Gemma3TextModel(Gemma3TextConfig(**kw)).eval()
    torch.manual_seed(0)
    with torch.no_grad():
        for n, p in m.named_parameters():
            p.normal_(0, 1 / math.sqrt(p.shape[-1])) if p.dim() >= 2 else p.normal_(0, 0.1)
    d = tmp_path / "eg"
    d.mkdir()
    cfg = m.config.to_dict()
    cfg["sliding_window"] = 8  # files keep the full window
    (d / "config.json").write_text(json.dumps(cfg))
    save_file({k: v.detach().contiguous() for k, v in m.state_dict().items()}, str(d / "model.safetensors"))
    g = torch.Generator().manual_seed(2)
    W1, W2 = torch.randn(96, 64, generator=g) / 8, torch.randn(32, 96, generator=g) / 10
    (d / "modules.json").write_text(json.dumps([
        {"idx": 0, "type": "sentence_transformers.models.Transformer", "path": ""},
        {"idx": 1, "type": "sentence_transformers.models.Pooling", "path": "1_Pooling"},
        {"idx": 2, "type": "sentence_transformers.models.Dense", "path": "2_Dense"},
        {"idx": 3, "type": "sentence_transformers.models.Dense", "path": "3_Dense"}]))
    for sub, W in (("2_Dense", W1), ("3_Dense", W2)):
        (d / sub).mkdir()
        (d / sub / "config.json").write_text(json.dumps({"in_features": W.shape[1], "out_features": W.shape[0],
                                                         "bias": False, "activation_function":
                                                         "torch.nn.modules.linear.Identity"}))
        save_file({"linear.weight": W.contiguous()}, str(d / sub / "model.safetensors"))
    (d / "1_Pooling").mkdir()
    (d / "1_Pooling" / "config.json").write_text(json.dumps({"pooling_mode_mean_tokens": True}))
    emb = load_embedder(str(d), device="cpu")
    assert isinstance(emb, DecoderEmbedder) and not emb.cfg.causal and emb.cfg.layer_window(0) == 5
    ids = torch.randint(1, 128, (1, 23), generator=g)
    with torch.no_grad():
        ref = m(input_ids=ids).last_hidden_state[0]
    got = emb.hidden(ids[0].tolist())
    assert (got - ref).abs().max() < 1e-4
    e = emb.embed([ids[0].tolist()])
    r = torch.nn.functional.normalize(ref.mean(0) @ W1.t() @ W2.t(), dim=-1)
    assert torch.allclose(e[0], r, atol=1e-4)
