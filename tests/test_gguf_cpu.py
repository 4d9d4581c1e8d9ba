"""GGUF checkpoints on CPU: every block format against an independent
implementation (the ``gguf`` package, when installed), file interop both
ways, HF name mapping, the llama q/k row permutation, and a model built from a
GGUF file matching the same weights from safetensors."""
import numpy as np
import pytest
import torch

from rlx_models_b200.weights import gguf as G

KINDS = ["Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"]
# byte offsets of fp16 scale fields inside each block (random bytes there could be inf / nan)
HALF_FIELDS = {"Q4_0": [0], "Q4_1": [0, 2], "Q5_0": [0], "Q5_1": [0, 2], "Q8_0": [0], "Q2_K": [80, 82],
               "Q3_K": [108], "Q4_K": [0, 2], "Q5_K": [0, 2], "Q6_K": [208]}


def random_blocks(kind, nb, seed=0):
    """Random blocks with finite fp16 / fp32 scale fields."""
    tid = G.TYPE_ID[kind]
    _, be, bb = G.GGML_TYPES[tid]
    g = torch.Generator().manual_seed(seed)
    b = torch.randint(0, 256, (nb, bb), generator=g, dtype=torch.int64).to(torch.uint8)
    for off in HALF_FIELDS.get(kind, []):
        h = (torch.rand(nb, generator=g) * 0.02 + 1e-3).half()
        b[:, off:off + 2] = h.view(torch.uint8).view(nb, 2)
    if kind == "Q8_K":
        b[:, 0:4] = (torch.rand(nb, generator=g) * 0.01).float().view(torch.uint8).view(nb, 4)
    return b.reshape(-1), be


@pytest.mark.parametrize("kind", KINDS)
def test_dequant_matches_gguf_package(kind):
    gq = pytest.importorskip("gguf.quants")
    import gguf
    raw, be = random_blocks(kind, 24)
    ours = G.dequantize_blocks(raw, kind)
    qt = getattr(gguf.GGMLQuantizationType, kind)
    ref = gq.dequantize(raw.numpy().reshape(1, -1), qt).reshape(-1)
    assert ours.shape[0] == 24 * be
    np.testing.assert_allclose(ours.numpy(), ref.astype(np.float32), rtol=1e-6, atol=1e-7)


def test_q8k_dequant():
    """Q8_K (fp32 scale, 256 int8, int16 block sums): value = d * q."""
    raw, _ = random_blocks("Q8_K", 5)
    b = raw.view(5, 292)
    d = b[:, 0:4].contiguous().view(torch.float32)
    q = b[:, 4:260].view(torch.int8).float()
    assert torch.equal(G.dequantize_blocks(raw, "Q8_K"), (q * d).reshape(-1))


@pytest.mark.parametrize("kind,tol", [("Q8_0", 0.01), ("Q4_0", 0.12), ("Q4_K", 0.1), ("Q6_K", 0.03),
                                      ("F16", 1e-3), ("BF16", 5e-3)])
def test_quantize_roundtrip(kind, tol):
    x = torch.randn(16, 512, generator=torch.Generator().manual_seed(1))
    y = G.dequantize(G.quantize(x, kind), kind, x.shape)
    assert ((y - x).norm() / x.norm()).item() < tol


def test_our_file_reads_with_gguf_package_and_back(tmp_path):
    gg = pytest.importorskip("gguf")
    x = torch.randn(8, 256, generator=torch.Generator().manual_seed(2))
    p = str(tmp_path / "a.gguf")
    w = G.GGUFWriter(p)
    w.add("general.architecture", "qwen3")
    w.add("qwen3.block_count", 3)
    w.add("some.float", 0.5)
    w.add("tokenizer.ggml.tokens", ["a", "b", "c"])
    w.add_tensor("blk.0.attn_q.weight", x, "Q8_0")
    w.add_tensor("output_norm.weight", x[0], "F32")
    w.add_tensor("blk.0.ffn_up.weight", x, "Q6_K")
    w.write()
    r = gg.GGUFReader(p)
    names = {t.name: t for t in r.tensors}
    assert set(names) == {"blk.0.attn_q.weight", "output_norm.weight", "blk.0.ffn_up.weight"}
    t = names["blk.0.attn_q.weight"]
    deq = gg.quants.dequantize(t.data, t.tensor_type).reshape(8, 256)
    ours = G.GGUFReader(p)
    assert ours.metadata["qwen3.block_count"] == 3 and ours.metadata["tokenizer.ggml.tokens"] == ["a", "b", "c"]
    np.testing.assert_allclose(ours.get("blk.0.attn_q.weight").numpy(), deq, rtol=1e-6)
    assert torch.equal(ours.get("output_norm.weight"), x[0])
    assert ((ours.get("blk.0.ffn_up.weight") - x).norm() / x.norm()) < 0.03


def test_gguf_package_file_reads_with_ours(tmp_path):
    gg = pytest.importorskip("gguf")
    p = str(tmp_path / "b.gguf")
    w = gg.GGUFWriter(p, "llama")
    w.add_block_count(2)
    a = np.random.default_rng(0).standard_normal((4, 64)).astype(np.float32)
    w.add_tensor("token_embd.weight", a)
    w.add_tensor("blk.1.attn_k.weight", a.astype(np.float16))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    r = G.GGUFReader(p)
    assert r.metadata["general.architecture"] == "llama" and r.metadata["llama.block_count"] == 2
    np.testing.assert_array_equal(r.get("token_embd.weight").numpy(), a)
    np.testing.assert_array_equal(r.get("blk.1.attn_k.weight").numpy(), a.astype(np.float16).astype(np.float32))


def test_names_and_permutation():
    for hf in ["model.embed_tokens.weight", "lm_head.weight", "model.norm.weight",
               "model.layers.3.self_attn.q_proj.weight", "model.layers.0.mlp.down_proj.weight",
               "model.layers.11.self_attn.k_norm.weight", "model.layers.2.self_attn.v_proj.bias"]:
        assert G.gguf_to_hf_name(G.hf_to_gguf_name(hf)) == hf
    assert G.hf_to_gguf_name("model.layers.3.self_attn.q_proj.weight") == "blk.3.attn_q.weight"
    w = torch.randn(4 * 16, 8)
    assert torch.equal(G.unpermute_qk(G.permute_qk(w, 4), 4), w)
    assert not torch.equal(G.permute_qk(w, 4), w)


@pytest.mark.parametrize("model_type", ["qwen3", "llama"])
def test_model_from_gguf_matches_safetensors(tmp_path, model_type):
    from rlx_models_b200 import config as C
    from rlx_models_b200.models.oracle import DecoderOracle
    from rlx_models_b200.weights.init import random_weights
    over = {} if model_type == "qwen3" else dict(qk_norm=False)
    cfg = C.tiny(model_type, num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=64, vocab_size=256, tie_word_embeddings=False, **over)
    w = random_weights(cfg, 0)
    p = G.save_gguf(str(tmp_path / "m.gguf"), w, cfg, kind="F32")
    gw = G.GGUFWeights(p, dtype=torch.float32)
    c2 = gw.config
    assert (c2.num_hidden_layers, c2.hidden_size, c2.num_key_value_heads, c2.head_dim, c2.qk_norm,
            c2.tie_word_embeddings) == (2, 256, 2, 64, model_type == "qwen3", False)
    assert set(gw.keys()) == set(w.keys())
    for k in w:
        assert torch.equal(gw.take(k), w[k].float()), k
    ids = torch.randint(0, 256, (12,), generator=torch.Generator().manual_seed(3))
    a, _ = DecoderOracle(cfg, {k: v.float() for k, v in w.items()}).forward(ids)
    b, _ = DecoderOracle(c2, {k: gw.take(k) for k in gw.keys()}).forward(ids)
    assert torch.allclose(a, b, atol=1e-5)
    # quantised file: logits close to the unquantised model
    pq = G.save_gguf(str(tmp_path / "q.gguf"), w, cfg, kind="Q8_0")
    gq = G.GGUFWeights(pq, dtype=torch.float32)
    c, _ = DecoderOracle(gq.config, {k: gq.take(k) for k in gq.keys()}).forward(ids)
    assert ((c - a).norm() / a.norm()) < 2e-2


# -- MLX quantised checkpoints ---------------------------------------------------

@pytest.mark.parametrize("bits", [2, 4, 8])
def test_mlx_pack_roundtrip(bits):
    from rlx_models_b200.weights import mlx as M
    w = torch.randn(48, 256, generator=torch.Generator().manual_seed(bits))
    wq, sc, bi = M.quantize(w, bits, 64)
    assert wq.dtype == torch.int32 and wq.shape == (48, 256 * bits // 32) and sc.shape == (48, 4)
    q = M.unpack_codes(wq, bits)
    assert int(q.min()) >= 0 and int(q.max()) <= (1 << bits) - 1
    # code j of a row sits at bits [(j % per) * bits, ...) of word j // per, least significant first
    per = 32 // bits
    word = (wq[3, 1].item() & 0xFFFFFFFF)
    assert q[3, per + 2].item() == (word >> (2 * bits)) & ((1 << bits) - 1)
    y = M.dequantize(wq, sc, bi, bits, 64)
    err = ((y - w).norm() / w.norm()).item()
    assert err < {2: 0.5, 4: 0.12, 8: 0.01}[bits]


def test_mlx_checkpoint_loads_into_model(tmp_path):
    from rlx_models_b200 import config as C
    from rlx_models_b200.models.oracle import DecoderOracle
    from rlx_models_b200.weights import mlx as M
    from rlx_models_b200.weights.init import random_weights
    cfg = C.tiny(num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=64, vocab_size=256)
    w = random_weights(cfg, 0)
    d = str(tmp_path / "mlx")
    cfg.save(d)
    import json
    raw = json.load(open(tmp_path / "mlx" / "config.json"))
    M.save_mlx(d, w, raw, bits=8, group_size=64)
    assert M.MLXWeights.is_mlx_dir(d)
    mw = M.MLXWeights(d, dtype=torch.float32)
    assert set(mw.keys()) == set(w.keys())
    ids = torch.randint(0, 256, (10,), generator=torch.Generator().manual_seed(0))
    a, _ = DecoderOracle(cfg, {k: v.float() for k, v in w.items()}).forward(ids)
    b, _ = DecoderOracle(cfg, {k: mw.take(k) for k in mw.keys()}).forward(ids)
    assert ((b - a).norm() / a.norm()).item() < 3e-2
