"""Quantisation formats and calibration (CPU): round trips, and AWQ / GPTQ
beating round-to-nearest on the layer output for correlated activations."""
import os

import torch

from rlx_models_b200.quant.calib import (awq, dequantize_fp8, dequantize_nvfp4, gptq, mxfp4_rtn, output_error,
                                         quantize_fp8, quantize_nvfp4)


def _data(out_f=96, in_f=256, n=512, seed=0):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(out_f, in_f, generator=g) * 0.05
    # activations with a few large channels and correlation (like LLM hidden states)
    base = torch.randn(n, 16, generator=g) @ torch.randn(16, in_f, generator=g)
    x = base + 0.3 * torch.randn(n, in_f, generator=g)
    x[:, :8] *= 12.0
    return w, x


def test_nvfp4_and_fp8_roundtrip():
    w = torch.randn(64, 128) * 0.1
    c, bs, ts = quantize_nvfp4(w)
    assert c.dtype == torch.uint8 and bs.dtype == torch.float8_e4m3fn and bs.shape == (64, 8)
    assert ((dequantize_nvfp4(c, bs, ts) - w).norm() / w.norm()) < 0.15
    q, s = quantize_fp8(w)
    assert ((dequantize_fp8(q, s) - w).norm() / w.norm()) < 0.05


def test_awq_and_gptq_beat_rtn():
    w, x = _data()
    e_rtn = output_error(w, mxfp4_rtn(w), x)
    wq_awq, s, a = awq(w, x, "mxfp4")
    e_awq = output_error(w, wq_awq, x)
    e_gptq = output_error(w, gptq(w, x, "mxfp4"), x)
    assert e_awq <= e_rtn + 1e-9 and e_gptq < e_rtn, (e_rtn, e_awq, e_gptq)
    # fp8 per-channel GPTQ is at least as good as its RTN
    e8 = output_error(w, dequantize_fp8(*quantize_fp8(w)), x)
    assert output_error(w, gptq(w, x, "fp8"), x) <= e8 * 1.01


def test_gptq_output_is_on_the_mxfp4_grid():
    w, x = _data(32, 64, 128)
    q = gptq(w, x, "mxfp4")
    # every value = E2M1 * 2^e for one e per (row, 32-group)
    g = q.reshape(32, 2, 32)
    for r in range(32):
        for k in range(2):
            v = g[r, k]
            nz = v[v != 0].abs()
            if nz.numel():
                e = torch.floor(torch.log2(nz.max() / 6.0 * 1.0000001)) + 0
                ratios = v / torch.pow(2.0, torch.ceil(torch.log2(nz.max() / 6.0)))
                assert torch.allclose(ratios * 2, torch.round(ratios * 2)), (r, k)


def test_quantize_checkpoint_roundtrip_and_algorithms():
    import tempfile

    from rlx_models_b200 import config as C
    from rlx_models_b200.models.oracle import DecoderOracle
    from rlx_models_b200.quant.tool import load_quantized, quantize_checkpoint
    from rlx_models_b200.weights.init import random_weights
    from rlx_models_b200.weights.weight_map import WeightMap

    cfg = C.tiny(num_hidden_layers=2, hidden_size=64, intermediate_size=128, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=16, vocab_size=128)
    w = random_weights(cfg, 0, dtype=torch.float32)
    calib = [torch.randint(0, 128, (64,), generator=torch.Generator().manual_seed(s)) for s in range(3)]
    ids = torch.randint(0, 128, (32,), generator=torch.Generator().manual_seed(9))
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "src")
        WeightMap(dict(w)).save(src)
        cfg.save(src)
        ref, _ = DecoderOracle(cfg, w).forward(ids)
        errs = {}
        for algo in ("rtn", "awq", "gptq"):
            for fmt in (("mxfp4", "fp8", "nvfp4") if algo == "rtn" else ("mxfp4",)):
                out = os.path.join(d, f"{algo}_{fmt}")
                rep = quantize_checkpoint(src, out, algo, fmt, calib)
                assert len(rep) == 2 * 7
                wq = load_quantized(out)
                assert set(k for k in wq) >= set(k for k in w if k.endswith(".weight"))
                lg, _ = DecoderOracle(cfg, {k: v.float() for k, v in wq.items()}).forward(ids)
                errs[(algo, fmt)] = float((lg - ref).norm() / ref.norm())
        assert errs[("rtn", "fp8")] < errs[("rtn", "mxfp4")]
        assert all(e < 0.5 for e in errs.values()), errs


def test_int_group_bitnet_formats():
    from rlx_models_b200.quant import calib as Q
    w = torch.randn(64, 256, generator=torch.Generator().manual_seed(0))
    for fmt, tol in (("int8", 0.01), ("int4", 0.15)):
        e = ((Q.FORMATS[fmt](w) - w).norm() / w.norm()).item()
        assert e < tol, (fmt, e)
    q, s = Q.quantize_bitnet(w)
    assert set(q.unique().tolist()) <= {-1, 0, 1} and abs(float(s) - w.abs().mean().item()) < 1e-6
    assert torch.equal(Q.unpack_ternary(Q.pack_ternary(q)), q)
    x = torch.randn(5, 256)
    xq, xs = Q.bitnet_activation_quant(x)
    assert xq.dtype == torch.int8 and ((xq.float() * xs - x).abs().max() <= xs.max() / 2 + 1e-6)
    xa = torch.randn(512, 256)
    g = Q.gptq(w, xa, "int4")
    assert Q.output_error(w, g, xa) < Q.output_error(w, Q.FORMATS["int4"](w), xa)


def test_quantize_checkpoint_int_bitnet_and_gguf_sink(tmp_path):
    from rlx_models_b200 import config as C
    from rlx_models_b200.models.oracle import DecoderOracle
    from rlx_models_b200.quant.tool import load_quantized, quantize_checkpoint
    from rlx_models_b200.weights.gguf import GGUFWeights
    from rlx_models_b200.weights.init import random_weights
    from rlx_models_b200.weights.weight_map import WeightMap

    cfg = C.tiny(num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=64, vocab_size=256)
    w = random_weights(cfg, 0, dtype=torch.float32)
    calib = [torch.randint(0, 256, (64,), generator=torch.Generator().manual_seed(s)) for s in range(2)]
    ids = torch.randint(0, 256, (16,), generator=torch.Generator().manual_seed(9))
    src = str(tmp_path / "src")
    WeightMap(dict(w)).save(src)
    cfg.save(src)
    ref, _ = DecoderOracle(cfg, w).forward(ids)
    errs = {}
    for algo, fmt in (("rtn", "int8"), ("gptq", "int4"), ("rtn", "bitnet")):
        out = str(tmp_path / f"{algo}_{fmt}")
        quantize_checkpoint(src, out, algo, fmt, calib)
        wq = load_quantized(out)
        lg, _ = DecoderOracle(cfg, {k: v.float() for k, v in wq.items()}).forward(ids)
        errs[fmt] = float((lg - ref).norm() / ref.norm())
    assert errs["int8"] < errs["int4"] < errs["bitnet"] and errs["int8"] < 0.02, errs
    for algo in ("rtn", "awq"):
        out = str(tmp_path / f"gguf_{algo}")
        quantize_checkpoint(src, out, algo, "gguf:Q8_0", calib)
        gw = GGUFWeights(os.path.join(out, "model-Q8_0.gguf"), dtype=torch.float32)
        lg, _ = DecoderOracle(gw.config, {k: gw.take(k) for k in gw.keys()}).forward(ids)
        assert float((lg - ref).norm() / ref.norm()) < 0.03


def test_dwq_heals_quantised_layer():
    from rlx_models_b200.quant.dwq import heal_linear
    g = torch.Generator().manual_seed(0)
    w = torch.randn(96, 128, generator=g) * 0.05
    # activations occupy a low-dimensional subspace (as real layer inputs do), so the
    # quantisation error they see has low rank and a rank-32 adapter can absorb it
    x = torch.randn(512, 24, generator=g) @ torch.randn(24, 128, generator=g) + 0.01 * torch.randn(512, 128,
                                                                                                     generator=g)
    r = heal_linear(w, x, "int4", rank=32, steps=400)
    assert r.healed_weight.shape == w.shape
    assert r.dwq_error < 0.3 * r.quant_error, (r.quant_error, r.dwq_error)


def test_qat_training_steps_and_ste():
    from rlx_models_b200 import config as C
    from rlx_models_b200.quant.dwq import fake_quant
    from rlx_models_b200.train.trainer import TrainConfig, Trainer
    from rlx_models_b200.weights.init import random_weights
    w = torch.randn(8, 64, requires_grad=True)
    y = fake_quant(w, "int4")
    assert not torch.equal(y, w) and torch.allclose(y, w, atol=0.5 * w.abs().max().item() / 7 + 1e-6)  # half an int4 step
    y.sum().backward()
    assert torch.equal(w.grad, torch.ones_like(w))  # straight-through
    cfg = C.tiny(num_hidden_layers=2, hidden_size=64, intermediate_size=128, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=16, vocab_size=96)
    b = torch.randint(0, 96, (4, 17), generator=torch.Generator().manual_seed(1))
    t = Trainer(cfg, TrainConfig(lr=1e-2, micro_batch=2, param_dtype="float32", qat="int4",
                                 activation_checkpointing=False), random_weights(cfg, 0), device="cpu")
    plain = Trainer(cfg, TrainConfig(lr=1e-2, micro_batch=2, param_dtype="float32",
                                     activation_checkpointing=False), random_weights(cfg, 0), device="cpu")
    lq = [t.step(b).loss for _ in range(4)]
    lp = plain.step(b).loss
    assert lq[-1] < lq[0] and abs(lq[0] - lp) > 1e-6  # trains, and the forward sees quantised weights
