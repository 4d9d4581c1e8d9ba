"""Llama-4 text (iRoPE: interleaved-pair RoPE + weightless QK norm on 3 of 4
layers, NoPE layers with query temperature; chunked attention on the RoPE
layers; top-1 sigmoid experts scaling the expert input + a shared expert;
dense / MoE interleave) on the fp32 oracle against transformers."""
import math

import pytest
import torch


def _rand(m):
    torch.manual_seed(0)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p.shape[-1] if "experts" not in n else p.shape[-2]))
            else:
                p.normal_(1.0 if n.endswith("norm.weight") else 0.0, 0.1)
    return m.eval()


def _hf(chunk=8, floor=4, step=2, qk=True):
    import transformers as T
    cfg = T.Llama4TextConfig(vocab_size=128, hidden_size=64, intermediate_size=48, intermediate_size_mlp=96,
                             num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2, head_dim=16,
                             num_local_experts=4, num_experts_per_tok=1, interleave_moe_layer_step=step,
                             attention_chunk_size=chunk, floor_scale=floor, attn_scale=0.1, use_qk_norm=qk,
                             rope_parameters={"rope_type": "default", "rope_theta": 500000.0},
                             max_position_embeddings=256, tie_word_embeddings=False)
    cfg._attn_implementation = "eager"
    return cfg, _rand(T.Llama4ForCausalLM(cfg))


@pytest.mark.parametrize("chunk,floor,step,qk", [(8, 4, 2, True), (0, 8192, 1, False)])
def test_llama4_text_oracle_matches_transformers(chunk, floor, step, qk):
    from rlx_models_b200.config import DecoderConfig
    from rlx_models_b200.models.oracle import DecoderOracle
    hc, m = _hf(chunk or 8192, floor, step, qk)
    cfg = DecoderConfig.from_hf_dict(hc.to_dict())
    assert cfg.model_type == "llama4_text" and cfg.rope_layers == [1, 1, 1, 0]
    assert cfg.moe_layers == list(range(step - 1, 4, step))
    ids = torch.randint(0, 128, (1, 21), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = m(input_ids=ids).logits[0]
    o = DecoderOracle(cfg, {k: v.detach() for k, v in m.state_dict().items()})
    lg, kv = o.forward(ids[0])
    assert (lg - ref).abs().max() < 1e-3, (lg - ref).abs().max()
    # incremental decode through the oracle's cache equals the full pass
    lg2, _ = o.forward(ids[0, :15])
    o2 = DecoderOracle(cfg, {k: v.detach() for k, v in m.state_dict().items()})
    a, kv2 = o2.forward(ids[0, :15])
    b, _ = o2.forward(ids[0, 15:], kv2)
    assert (torch.cat([a, b]) - ref).abs().max() < 1e-3


def test_interleaved_rope_is_half_split_rope_on_reordered_rows():
    """The GPU path's claim: rows reordered [0, 2, .., D-2, 1, 3, .., D-1] turn the
    interleaved-pair rotation into the half-split one (same dot products)."""
    from rlx_models_b200.ops import reference as R
    g = torch.Generator().manual_seed(0)
    D = 16
    q, k = torch.randn(7, 2, D, generator=g), torch.randn(7, 2, D, generator=g)
    pos = torch.arange(3, 10)
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2).float() / D))
    perm = torch.cat([torch.arange(0, D, 2), torch.arange(1, D, 2)])
    a = R.rope_interleaved(q, pos, inv)
    b = R.rope(q[..., perm], pos, inv)
    assert torch.allclose(a[..., perm], b, atol=1e-5)
    s1 = torch.einsum("thd,shd->hts", R.rope_interleaved(q, pos, inv), R.rope_interleaved(k, pos, inv))
    s2 = torch.einsum("thd,shd->hts", R.rope(q[..., perm], pos, inv), R.rope(k[..., perm], pos, inv))
    assert torch.allclose(s1, s2, atol=1e-4)
