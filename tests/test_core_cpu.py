"""CPU tests: configs, safetensors / WeightMap round-trip, seeded init, fp32
oracle, MXFP4 packing and the native scheduler (driven with fake tokens)."""
import json
import os

import pytest
import torch

from rlx_models_b200 import config as C
from rlx_models_b200.models.oracle import DecoderOracle
from rlx_models_b200.quant.mxfp4 import dequantize_mxfp4, quantize_mxfp4
from rlx_models_b200.weights.init import random_weights
from rlx_models_b200.weights.safetensors_io import Checkpoint, save_file, save_sharded
from rlx_models_b200.weights.weight_map import UnusedWeights, WeightMap


def test_legacy_rope_and_text_config():
    raw = {"model_type": "qwen3", "hidden_size": 64, "num_attention_heads": 4, "num_hidden_layers": 1,
           "intermediate_size": 128, "vocab_size": 100,
           "rope_parameters": {"rope_theta": 5e5, "rope_type": "yarn", "factor": 4.0}}
    c = C.DecoderConfig.from_hf_dict(raw)
    assert c.rope_theta == 5e5 and c.rope_scaling["factor"] == 4.0 and c.head_dim == 16
    assert c.num_key_value_heads == 4
    wrapped = {"model_type": "qwen3_vl", "text_config": dict(raw, model_type="qwen3")}
    c2 = C.DecoderConfig.from_hf_dict(wrapped)
    assert c2.hidden_size == 64


def test_preset_shapes():
    q8 = C.qwen3_8b()
    assert (q8.hidden_size, q8.num_hidden_layers, q8.intermediate_size) == (4096, 36, 12288)
    assert 8.0e9 < q8.num_params() < 8.3e9
    g = C.gpt_oss_120b()
    assert g.layer_window(0) == 128 and g.layer_window(1) == 0 and g.num_experts == 128


def test_config_roundtrip(tmp_path):
    c = C.tiny()
    c.save(str(tmp_path))
    c2 = C.DecoderConfig.from_file(str(tmp_path))
    assert c2.hidden_size == c.hidden_size and c2.num_hidden_layers == c.num_hidden_layers


def test_safetensors_roundtrip(tmp_path):
    t = {"a": torch.randn(3, 5).bfloat16(), "b": torch.arange(10, dtype=torch.int32),
         "c": torch.randn(7).float(), "e": torch.zeros(0)}
    p = str(tmp_path / "x.safetensors")
    save_file(t, p, {"format": "pt"})
    ck = Checkpoint(p)
    for k, v in t.items():
        assert torch.equal(ck.get(k), v)
    files = save_sharded(t, str(tmp_path / "sh"), max_shard_bytes=40)
    assert len(files) > 1
    ck2 = Checkpoint(str(tmp_path / "sh"))
    assert sorted(ck2.keys()) == sorted(t) and torch.equal(ck2.get("a"), t["a"])
    idx = json.load(open(tmp_path / "sh" / "model.safetensors.index.json"))
    assert set(idx["weight_map"]) == set(t)


def test_weight_map_strict_and_shards(tmp_path):
    c = C.tiny()
    w = random_weights(c, seed=0)
    wm = WeightMap(w)
    wm.take("model.embed_tokens.weight")
    with pytest.raises(UnusedWeights):
        wm.finish(strict=True)
    q = wm.take_shard("model.layers.0.self_attn.q_proj.weight", 0, 1, 2)
    assert torch.equal(q, w["model.layers.0.self_attn.q_proj.weight"][128:256])


def test_seeded_init_is_subset_stable():
    c = C.tiny()
    a = random_weights(c, seed=5)
    b = random_weights(c, seed=5, names={"model.layers.1.mlp.up_proj.weight"})
    assert torch.equal(a["model.layers.1.mlp.up_proj.weight"], b["model.layers.1.mlp.up_proj.weight"])
    d = random_weights(c, seed=6, names={"model.layers.1.mlp.up_proj.weight"})
    assert not torch.equal(a["model.layers.1.mlp.up_proj.weight"], d["model.layers.1.mlp.up_proj.weight"])
    # per-layer distinct
    assert not torch.equal(a["model.layers.0.mlp.up_proj.weight"], a["model.layers.1.mlp.up_proj.weight"])


def test_oracle_decode_matches_prefill():
    """Incremental KV decode == recomputing the longer prefill (fp32)."""
    c = C.tiny(num_hidden_layers=2)
    w = random_weights(c, seed=1, dtype=torch.float32)
    o = DecoderOracle(c, w)
    ids = torch.randint(0, c.vocab_size, (12,), generator=torch.Generator().manual_seed(1))
    full, _ = o.forward(ids)
    part, kv = o.forward(ids[:8])
    for t in range(8, 12):
        lg, kv = o.forward(ids[t:t + 1], kv)
        assert torch.allclose(lg[-1], full[t], atol=1e-4, rtol=1e-4)


def test_oracle_safetensors_roundtrip_logits(tmp_path):
    c = C.tiny()
    w = random_weights(c, seed=2, dtype=torch.float32)
    WeightMap(w).save(str(tmp_path))
    c.save(str(tmp_path))
    w2 = WeightMap.from_dir(str(tmp_path)).to_dict()
    ids = torch.arange(10)
    a, _ = DecoderOracle(c, w).forward(ids)
    b, _ = DecoderOracle(C.DecoderConfig.from_file(str(tmp_path)), w2).forward(ids)
    assert torch.equal(a, b)


def test_gpt_oss_oracle_runs_and_window_matters():
    c = C.tiny("gpt_oss")
    w = random_weights(c, seed=3, dtype=torch.float32)
    o = DecoderOracle(c, w)
    ids = torch.randint(0, c.vocab_size, (40,), generator=torch.Generator().manual_seed(2))
    lg, _ = o.forward(ids)
    assert lg.shape == (40, c.vocab_size) and torch.isfinite(lg).all()
    c_full = C.tiny("gpt_oss", layer_types=["full_attention", "full_attention"])
    lg2, _ = DecoderOracle(c_full, w).forward(ids)
    assert torch.allclose(lg[:16], lg2[:16], atol=1e-4)      # inside the window: identical
    assert not torch.allclose(lg[30:], lg2[30:], atol=1e-4)  # beyond it: differs


def test_mxfp4_roundtrip():
    w = torch.randn(4, 64, 96) * 0.03
    b, s = quantize_mxfp4(w)
    assert b.shape == (4, 64, 3, 16) and s.shape == (4, 64, 3)
    d = dequantize_mxfp4(b, s)
    rel = (d - w).norm() / w.norm()
    assert rel < 0.2
    # exactly representable values survive
    x = torch.tensor([[0.5, -1.0, 6.0, 3.0] * 8])
    assert torch.equal(dequantize_mxfp4(*quantize_mxfp4(x)), x)


# ---------------------------------------------------------------------------
# native scheduler
# ---------------------------------------------------------------------------

def _staging(T=4096, S=64, W=64):
    i32, i64 = torch.int32, torch.int64
    return [torch.zeros(T, dtype=i32), torch.zeros(T, dtype=i32), torch.zeros(T, dtype=i64),
            torch.zeros(S, W, dtype=i32), torch.zeros(S, dtype=i32), torch.zeros(S, W, dtype=i32),
            torch.zeros(S, dtype=i32), torch.zeros(S + 1, dtype=i32), torch.zeros(T, dtype=i64),
            torch.zeros(T, dtype=i64)]


def _drive(sched, bufs, eos=-1, max_steps=10000):
    """Run the scheduler with a fake model that emits token = position % 97."""
    steps = []
    for _ in range(max_steps):
        if not sched.has_work():
            break
        info = sched.schedule(*bufs)
        R = info["num_logits"]
        rows = bufs[8][:R].tolist()
        sids = bufs[9][:R].tolist()
        toks = [int(bufs[1][r]) % 97 + 1 for r in rows]
        steps.append(info)
        sched.update(sids, toks, eos)
    return steps


def test_scheduler_chunked_prefill_and_decode():
    from rlx_models_b200 import _runtime
    s = _runtime.Scheduler(num_blocks=200, max_num_seqs=8, max_batched_tokens=64, max_blocks_per_seq=64,
                           prefix_caching=False, chunk_size=0)
    bufs = _staging()
    lens = [5, 70, 33, 16, 1]
    ids = [s.add_request(list(range(1, l + 1)), 10, True, []) for l in lens]
    steps = _drive(s, bufs)
    assert all(st["num_tokens"] <= 64 for st in steps)
    for sid, l in zip(ids, lens):
        out = s.output_tokens(sid)
        assert len(out) == 10
        # fake model: first token from the last prompt position, then +1 per step
        assert out[0] == (l - 1) % 97 + 1
        assert out[1:] == [((l + j) % 97) + 1 for j in range(9)]
    assert s.stats()["free_blocks"] == 200


def test_scheduler_positions_slots_consistent():
    from rlx_models_b200 import _runtime
    s = _runtime.Scheduler(50, 4, 40, 16, False, 0)
    bufs = _staging(W=16)
    s.add_request(list(range(30)), 4, True, [])
    info = s.schedule(*bufs)
    T = info["num_tokens"]
    assert T == 30 and info["num_prefill"] == 1 and info["num_decode"] == 0
    pos = bufs[1][:T].tolist()
    assert pos == list(range(30))
    slots = bufs[2][:T]
    tab = bufs[5][0]
    for p in range(T):
        assert int(slots[p]) == int(tab[p // 16]) * 16 + p % 16
    assert int(bufs[7][1]) == 30 and int(bufs[6][0]) == 30


def test_scheduler_prefix_cache_hits():
    from rlx_models_b200 import _runtime
    s = _runtime.Scheduler(100, 4, 256, 32, True, 0)
    bufs = _staging(W=32)
    prefix = list(range(100, 164))  # 4 full blocks
    a = s.add_request(prefix + [1, 2, 3], 2, True, [])
    _drive(s, bufs)
    b = s.add_request(prefix + [7, 8], 2, True, [])
    _drive(s, bufs)
    assert s.num_cached_prompt_tokens(b) == 64
    assert s.stats()["prefix_hits"] >= 4


def test_scheduler_preemption_recompute():
    from rlx_models_b200 import _runtime
    # 6 blocks total: two sequences that each grow to 3+ blocks must preempt
    s = _runtime.Scheduler(6, 4, 64, 16, False, 0)
    bufs = _staging(W=16)
    ids = [s.add_request(list(range(1, 31)), 20, True, []) for _ in range(2)]
    _drive(s, bufs)
    for sid in ids:
        out = s.output_tokens(sid)
        assert out == [((29 + j) % 97) + 1 for j in range(20)]
    assert s.stats()["preemptions"] >= 1


def test_scheduler_stop_and_abort():
    from rlx_models_b200 import _runtime
    s = _runtime.Scheduler(50, 4, 64, 16, False, 0)
    bufs = _staging(W=16)
    a = s.add_request([1, 2, 3], 50, False, [6])  # fake model emits 3,4,5,6 -> stops at 6
    b = s.add_request([1, 2, 3, 4], 50, False, [])
    info = s.schedule(*bufs)
    s.abort(b)
    R = info["num_logits"]
    s.update(bufs[9][:R].tolist(), [int(bufs[1][r]) % 97 + 1 for r in bufs[8][:R].tolist()], -1)
    _drive(s, bufs)
    assert s.output_tokens(a)[-1] == 6 and s.finish_reason(a) == 2
    assert s.finish_reason(b) == 3


def test_mxfp4_tile_roundtrip():
    from rlx_models_b200.quant.mxfp4 import quantize_mxfp4, tile_mxfp4, untile_mxfp4, dequantize_mxfp4
    w = torch.randn(3, 200, 192) * torch.logspace(-3, 1, 200)[None, :, None]
    b, s = quantize_mxfp4(w)
    t, rexp = tile_mxfp4(b, s)
    assert t.shape == (3, 2, 3, 4352) and rexp.shape == (3, 256)
    b2, s2 = untile_mxfp4(t, rexp, 200)
    assert torch.equal(b, b2) and torch.equal(s, s2)
    # offsets are the distance below each row's largest exponent
    offs = t[..., 4096:]
    assert int(offs.max()) <= int((s.amax(-1, keepdim=True) - s).max())
    assert torch.allclose(dequantize_mxfp4(b2, s2), dequantize_mxfp4(b, s))


def test_flux_oracle_deinterleaved_rope_matches():
    """Half-split RoPE on de-interleaved q/k rows == BFL interleaved-pair RoPE."""
    from rlx_models_b200.models.flux_common import (apply_rope_interleaved, deinterleave_perm, position_ids,
                                                     rope_tables)
    D = 128
    ids = position_ids(4, 3, 5)
    cos, sin = rope_tables(ids)
    q = torch.randn(2, 3, ids.shape[0], D, dtype=torch.float64)
    k = torch.randn(2, 3, ids.shape[0], D, dtype=torch.float64)
    ref = apply_rope_interleaved(q, cos.double(), sin.double()) @ apply_rope_interleaved(k, cos.double(), sin.double()).transpose(-1, -2)
    p = deinterleave_perm(D)

    def half(x):
        x1, x2 = x[..., :D // 2], x[..., D // 2:]
        c, s = cos.double(), sin.double()
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)

    got = half(q[..., p]) @ half(k[..., p]).transpose(-1, -2)
    assert torch.allclose(got, ref, atol=1e-9)


def test_flux_schedule_and_pack():
    from rlx_models_b200.models.flux_common import pack, schedule, unpack
    ts = schedule(28, 4096)
    assert ts[0] == 1.0 and ts[-1] == 0.0 and all(a > b for a, b in zip(ts, ts[1:]))
    x = torch.randn(2, 16, 8, 6)
    assert torch.equal(unpack(pack(x), 16, 8, 6), x)
    assert schedule(4, 4096, shift=False) == [1.0, 0.75, 0.5, 0.25, 0.0]


def test_mixtral_and_qwen2_moe_configs_and_names():
    import json
    import tempfile
    from rlx_models_b200.config import DecoderConfig
    from rlx_models_b200.models.oracle import DecoderOracle
    from rlx_models_b200.weights.aliases import canonical_name
    from rlx_models_b200.weights.init import random_weights
    mx = DecoderConfig.from_hf_dict({"model_type": "mixtral", "hidden_size": 64, "intermediate_size": 128,
                                     "num_hidden_layers": 1, "num_attention_heads": 4, "num_key_value_heads": 2,
                                     "vocab_size": 50, "num_local_experts": 4, "num_experts_per_tok": 2})
    assert (mx.num_experts, mx.moe_intermediate_size, mx.qk_norm, mx.is_moe) == (4, 128, False, True)
    with tempfile.TemporaryDirectory() as d:
        mx.save(d)
        assert json.load(open(d + "/config.json"))["num_local_experts"] == 4
    assert canonical_name("mixtral", "model.layers.3.block_sparse_moe.experts.7.w3.weight") == \
        "model.layers.3.mlp.experts.7.up_proj.weight"
    assert canonical_name("mixtral", "model.layers.0.block_sparse_moe.gate.weight") == "model.layers.0.mlp.gate.weight"
    # a Mixtral-named checkpoint gives the same oracle logits as the canonical names
    w = random_weights(mx, 0)
    mixnames = {}
    for k, v in w.items():
        k2 = k.replace(".mlp.gate.", ".block_sparse_moe.gate.")
        for a, b in (("gate_proj", "w1"), ("up_proj", "w3"), ("down_proj", "w2")):
            k2 = k2.replace(f".mlp.experts.", ".block_sparse_moe.experts.").replace(f".{a}.", f".{b}.") \
                if ".mlp.experts." in k2 or ".block_sparse_moe.experts." in k2 else k2
        mixnames[k2] = v
    ids = torch.randint(0, 50, (9,), generator=torch.Generator().manual_seed(0))
    a, _ = DecoderOracle(mx, {k: v.float() for k, v in w.items()}).forward(ids)
    b, _ = DecoderOracle(mx, {k: v.float() for k, v in mixnames.items()}).forward(ids)
    assert torch.equal(a, b)
    q2 = DecoderConfig.from_hf_dict({"model_type": "qwen2_moe", "hidden_size": 64, "num_hidden_layers": 1,
                                     "num_attention_heads": 4, "num_key_value_heads": 2, "vocab_size": 50,
                                     "num_experts": 4, "num_experts_per_tok": 2, "moe_intermediate_size": 64,
                                     "shared_expert_intermediate_size": 128, "intermediate_size": 256})
    assert q2.attention_bias and q2.shared_expert_intermediate_size == 128 and not q2.norm_topk_prob
    w2 = random_weights(q2, 1)
    assert "model.layers.0.mlp.shared_expert_gate.weight" in w2
    lg, _ = DecoderOracle(q2, {k: v.float() for k, v in w2.items()}).forward(ids)
    assert torch.isfinite(lg).all()


def _drive_overlap(sched, bufs, eos=-1, max_steps=10000):
    """Overlapped scheduling with the same fake model (token = position % 97 + 1):
    step n+1 is scheduled before step n's tokens are handed back; decode inputs
    that are still placeholders name a row of the previous step's output, which
    must hold exactly the token the synchronous loop would have fed."""
    T = bufs[0].numel()
    src = torch.full((T,), -1, dtype=torch.int32)
    inflight, prev_out, steps = None, [], []
    for _ in range(max_steps):
        if not sched.has_work() and inflight is None:
            break
        launched = None
        if sched.has_work():
            info = sched.schedule(*bufs, src, True)
            T_, R, nd = info["num_tokens"], info["num_logits"], info["num_decode"]
            if T_:
                ids = bufs[0][:T_].tolist()
                srcs = src[:T_].tolist()
                pos = bufs[1][:T_].tolist()
                fed = [prev_out[srcs[t]] if srcs[t] >= 0 else ids[t] for t in range(T_)]
                for t in range(nd):  # a decode input is the token sampled at the previous position
                    assert fed[t] == (pos[t] - 1) % 97 + 1, (t, fed[t], pos[t])
                rows = bufs[8][:R].tolist()
                launched = (bufs[9][:R].tolist(), [pos[r] % 97 + 1 for r in rows])
                steps.append(info)
        if inflight is not None:
            sched.update(inflight[0], inflight[1], eos)
        if launched is not None:
            prev_out = launched[1]
        inflight = launched
    return steps


def test_scheduler_overlap_matches_sync():
    from rlx_models_b200 import _runtime
    lens = [5, 70, 33, 16, 1]
    outs = {}
    for mode in ("sync", "overlap"):
        s = _runtime.Scheduler(num_blocks=200, max_num_seqs=8, max_batched_tokens=64, max_blocks_per_seq=64,
                               prefix_caching=False, chunk_size=0)
        bufs = _staging()
        ids = [s.add_request([1 + (i % 90) for i in range(l)], 10, True, []) for l in lens]
        (_drive if mode == "sync" else _drive_overlap)(s, bufs)
        outs[mode] = [s.output_tokens(i) for i in ids]
        assert s.stats()["free_blocks"] == 200
    assert outs["sync"] == outs["overlap"]


def test_scheduler_overlap_preemption_and_stop():
    from rlx_models_b200 import _runtime
    s = _runtime.Scheduler(6, 4, 64, 16, False, 0)
    bufs = _staging(W=16)
    ids = [s.add_request(list(range(1, 31)), 20, True, []) for _ in range(2)]
    _drive_overlap(s, bufs)
    for sid in ids:
        assert s.output_tokens(sid) == [((29 + j) % 97) + 1 for j in range(20)]
    assert s.stats()["preemptions"] >= 1 and s.stats()["free_blocks"] == 6
    # stop id: the row scheduled behind the stop is discarded
    s = _runtime.Scheduler(50, 4, 64, 16, False, 0)
    bufs = _staging(W=16)
    a = s.add_request([1, 2, 3], 50, False, [6])
    b = s.add_request([1, 2, 3, 4], 5, False, [])
    _drive_overlap(s, bufs)
    assert s.output_tokens(a) == [3, 4, 5, 6] and s.finish_reason(a) == 2
    assert s.output_tokens(b) == [4, 5, 6, 7, 8] and s.finish_reason(b) == 1
    assert s.stats()["free_blocks"] == 50


def test_scheduler_prefix_export_import():
    """prefix_blocks finds a prompt's cached blocks; import_prefix registers blocks
    that a fresh scheduler then reuses for a request with that prefix."""
    from rlx_models_b200 import _runtime
    s = _runtime.Scheduler(100, 4, 256, 32, True, 0)
    bufs = _staging(W=32)
    prompt = list(range(100, 150))  # 3 full blocks + 2 tokens
    s.add_request(prompt, 2, True, [])
    _drive(s, bufs)
    assert len(s.prefix_blocks(prompt)) == 3
    assert s.prefix_blocks([7] * 40) == []
    s2 = _runtime.Scheduler(100, 4, 256, 32, True, 0)
    blocks = s2.import_prefix(prompt)
    assert len(blocks) == 3 and all(b >= 0 for b in blocks)
    assert s2.import_prefix(prompt) == [-1, -1, -1]  # already cached: nothing to fill
    sid = s2.add_request(prompt + [1, 2, 3], 2, True, [])
    info = s2.schedule(*_staging(W=32))
    assert s2.num_cached_prompt_tokens(sid) == 48 and info["num_tokens"] == 53 - 48
