"""MTP heads (Qwen3.5 / Qwen3-Next ``mtp.*``): the head's math against the
published equations written out here, the layer mapping onto the model's own
layer code, and greedy drafting."""
import torch

from rlx_models_b200.models.qwen35 import Qwen35Config, Qwen35Oracle, random_weights
from rlx_models_b200.runtime.mtp import MTPHead, has_mtp, random_mtp_weights


def _cfg(moe: bool):
    kw = dict(vocab_size=97, hidden_size=64, intermediate_size=96, num_hidden_layers=2, num_attention_heads=4,
              num_key_value_heads=2, head_dim=16, linear_key_head_dim=16, linear_value_head_dim=16,
              linear_num_key_heads=2, linear_num_value_heads=4, tie_word_embeddings=False,
              layer_types=["linear_attention", "full_attention"])
    if moe:
        kw.update(num_experts=4, num_experts_per_tok=2, moe_intermediate_size=32, shared_expert_intermediate_size=48)
    return Qwen35Config(**kw)


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * (1.0 + w.float())


def _check(moe: bool):
    cfg = _cfg(moe)
    w = random_weights(cfg, 0, dtype=torch.float32)
    w.update(random_mtp_weights(cfg, 5, dtype=torch.float32))
    assert has_mtp(w)
    head = MTPHead(cfg, w)
    g = torch.Generator().manual_seed(3)
    W, H = 6, cfg.hidden_size
    h = torch.randn(W, H, generator=g)
    toks = torch.randint(0, cfg.vocab_size, (W,), generator=g)
    pos = torch.arange(10, 10 + W)
    y = head.features(h, toks, pos)
    # the same computation written out: the MTP layer is the model's layer code run
    # on the mtp.layers.0 tensors relabelled as an extra model layer
    e = _rms(w["model.embed_tokens.weight"][toks], w["mtp.pre_fc_norm_embedding.weight"], cfg.rms_norm_eps)
    x = torch.cat([e, _rms(h, w["mtp.pre_fc_norm_hidden.weight"], cfg.rms_norm_eps)], -1) @ w["mtp.fc.weight"].t()
    n = cfg.num_hidden_layers
    relab = dict(w)
    for k, v in w.items():
        if k.startswith("mtp.layers.0."):
            relab[f"model.layers.{n}." + k[len("mtp.layers.0."):]] = v
    cfg2 = Qwen35Config(**{**cfg.__dict__, "num_hidden_layers": n + 1,
                           "layer_types": cfg.layer_types + ["full_attention"]})
    o = Qwen35Oracle(cfg2, relab)
    p = f"model.layers.{n}."
    x = x + o.attention(n, o._rms(x, p + "input_layernorm.weight"), pos)
    xn = o._rms(x, p + "post_attention_layernorm.weight")
    x = x + (o.moe(n, xn) if moe else o._swiglu(xn, p + "mlp."))
    ref = _rms(x, w["mtp.norm.weight"], cfg.rms_norm_eps)
    assert (y - ref).abs().max() < 1e-4
    lg = head.logits(y)
    assert torch.allclose(lg, ref @ w["lm_head.weight"].t(), atol=1e-4)
    # greedy drafting chains on the head's own normalised output
    props = head.propose(h, toks.tolist(), 3, pos0=10)
    assert len(props) == 3 and props[0] == int(lg[-1].argmax())


def test_mtp_head_dense():
    _check(moe=False)


def test_mtp_head_moe():
    _check(moe=True)
