"""FLUX.1 DiT on the GPU against the fp32 oracle (tiny config), plus the
DiT-specific kernels (LayerNorm+modulate, QK-norm + 3-axis RoPE, gated /
GELU GEMM epilogues, non-causal paged attention)."""

import pytest
import torch
import torch.nn.functional as F

from rlx_models_b200 import ops
from rlx_models_b200.config import flux_tiny
from rlx_models_b200.models.flux import FluxDiT, generate_latents
from rlx_models_b200.models.flux_common import flux_random_weights, position_ids
from rlx_models_b200.models.flux_oracle import FluxOracle
from rlx_models_b200.ops._ext import ext

pytestmark = pytest.mark.gpu


def rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-9)).item()


def test_ln_modulate(cuda):
    R, H, B = 96, 512, 3
    x = torch.randn(R, H, device=cuda).bfloat16()
    mod = (torch.randn(B, 4 * H, device=cuda) * 0.3).bfloat16()
    out = torch.empty_like(x)
    split, r1, r2 = 30, 10, 22  # rows < 30: batch row // 10; else (row - 30) // 22
    ext().ln_modulate(x, out, mod, H, 2 * H, 1e-6, split, r1, r2)
    b = torch.tensor([r // r1 if r < split else (r - split) // r2 for r in range(R)], device=cuda)
    ref = F.layer_norm(x.float(), (H,), eps=1e-6) * (1 + mod[b, 2 * H:3 * H].float()) + mod[b, H:2 * H].float()
    assert rel(out, ref) < 1e-2


def test_linear_gate_gelu(cuda):
    M, N, K, B = 256, 384, 512, 2
    x = torch.randn(M, K, device=cuda).bfloat16()
    w = (torch.randn(N, K, device=cuda) * 0.05).bfloat16()
    bias = (torch.randn(N, device=cuda) * 0.1).bfloat16()
    res = torch.randn(M, N, device=cuda).bfloat16()
    gate = torch.randn(B, N, device=cuda).bfloat16()
    y = ops.linear(x, w, bias=bias, residual=res, gate=gate, gate_rows=(0, 1, M // B))
    ref = res.float() + gate.float().repeat_interleave(M // B, 0) * (x.float() @ w.float().T + bias.float())
    assert rel(y, ref) < 1e-2
    y2 = ops.linear(x, w, bias=bias, gelu_from=128)
    lin = x.float() @ w.float().T + bias.float()
    ref2 = torch.cat([lin[:, :128], F.gelu(lin[:, 128:], approximate="tanh")], 1)
    assert rel(y2, ref2) < 1e-2


def test_flux_dit_vs_oracle(cuda):
    cfg = flux_tiny()
    w = flux_random_weights(cfg, seed=0, bias_std=0.02)
    B, Lt, h, wd = 2, 16, 4, 8
    Li = h * wd
    g = torch.Generator().manual_seed(1)
    img = torch.randn(B, Li, cfg.in_channels, generator=g)
    txt = torch.randn(B, Lt, cfg.context_in_dim, generator=g)
    y = torch.randn(B, cfg.vec_in_dim, generator=g)
    t = torch.tensor([0.8, 0.3])
    gd = torch.tensor([3.5, 2.0])
    ids = position_ids(Lt, h, wd)
    ref = FluxOracle(cfg, w).forward(img, ids[Lt:], txt, ids[:Lt], t, y, gd)
    model = FluxDiT(cfg, w, device=cuda)
    out = model.forward(img.to(cuda).bfloat16(), txt.to(cuda).bfloat16(), t, y.to(cuda).bfloat16(), gd, h, wd,
                        graph=False).clone()
    torch.cuda.synchronize()
    ops.check_errors(cuda)
    assert rel(out.cpu(), ref) < 3e-2, rel(out.cpu(), ref)
    out_g = model.forward(img.to(cuda).bfloat16(), txt.to(cuda).bfloat16(), t, y.to(cuda).bfloat16(), gd, h, wd)
    torch.cuda.synchronize()
    assert torch.equal(out_g, out)


def test_flux_generate_runs(cuda):
    cfg = flux_tiny()
    model = FluxDiT(cfg, flux_random_weights(cfg, seed=0), device=cuda)
    txt = torch.randn(2, 16, cfg.context_in_dim, device=cuda).bfloat16()
    pooled = torch.randn(2, cfg.vec_in_dim, device=cuda).bfloat16()
    lat = generate_latents(model, txt, pooled, height=64, width=64, steps=4)
    assert lat.shape == (2, 4, 8, 8) and torch.isfinite(lat).all()


def test_flux_pipeline_text_to_image(cuda):
    """T5 + CLIP encoders (HF layouts, random tiny weights), the DiT on this
    package's kernels with a LoRA merged in, the VAE decoder: prompt ids ->
    image tensor of the requested size."""
    from rlx_models_b200.models.flux_lora import merge_lora
    from rlx_models_b200.models.flux_text import CLIPTextConfig, CLIPTextEncoder, T5Config, T5Encoder
    from rlx_models_b200.models.flux_vae import FluxPipeline, VAEConfig, VAEDecoder, to_image, vae_random_weights
    cfg = flux_tiny()
    g = torch.Generator().manual_seed(0)
    tc = T5Config(vocab_size=100, d_model=cfg.context_in_dim, d_kv=16, d_ff=64, num_layers=2, num_heads=4)
    t5w = {"shared.weight": torch.randn(100, tc.d_model, generator=g),
           "encoder.block.0.layer.0.SelfAttention.relative_attention_bias.weight": torch.randn(32, 4, generator=g),
           "encoder.final_layer_norm.weight": torch.ones(tc.d_model)}
    inner = tc.num_heads * tc.d_kv
    for i in range(tc.num_layers):
        p = f"encoder.block.{i}.layer."
        for n in "qkv":
            t5w[p + f"0.SelfAttention.{n}.weight"] = torch.randn(inner, tc.d_model, generator=g) * 0.05
        t5w[p + "0.SelfAttention.o.weight"] = torch.randn(tc.d_model, inner, generator=g) * 0.05
        t5w[p + "0.layer_norm.weight"] = torch.ones(tc.d_model)
        t5w[p + "1.layer_norm.weight"] = torch.ones(tc.d_model)
        for n in ("wi_0", "wi_1"):
            t5w[p + f"1.DenseReluDense.{n}.weight"] = torch.randn(tc.d_ff, tc.d_model, generator=g) * 0.05
        t5w[p + "1.DenseReluDense.wo.weight"] = torch.randn(tc.d_model, tc.d_ff, generator=g) * 0.05
    cc = CLIPTextConfig(vocab_size=100, hidden_size=cfg.vec_in_dim, intermediate_size=2 * cfg.vec_in_dim,
                        num_hidden_layers=1, num_attention_heads=4, max_position_embeddings=16)
    H = cc.hidden_size
    cw = {"text_model.embeddings.token_embedding.weight": torch.randn(100, H, generator=g),
          "text_model.embeddings.position_embedding.weight": torch.randn(16, H, generator=g),
          "text_model.final_layer_norm.weight": torch.ones(H), "text_model.final_layer_norm.bias": torch.zeros(H)}
    q = "text_model.encoder.layers.0."
    for n in ("q", "k", "v", "out"):
        cw[q + f"self_attn.{n}_proj.weight"] = torch.randn(H, H, generator=g) * 0.05
        cw[q + f"self_attn.{n}_proj.bias"] = torch.zeros(H)
    for n in ("layer_norm1", "layer_norm2"):
        cw[q + n + ".weight"], cw[q + n + ".bias"] = torch.ones(H), torch.zeros(H)
    cw[q + "mlp.fc1.weight"], cw[q + "mlp.fc1.bias"] = torch.randn(2 * H, H, generator=g) * 0.05, torch.zeros(2 * H)
    cw[q + "mlp.fc2.weight"], cw[q + "mlp.fc2.bias"] = torch.randn(H, 2 * H, generator=g) * 0.05, torch.zeros(H)
    dw = flux_random_weights(cfg, seed=0)
    lora = {"double_blocks.0.img_attn.qkv.lora_A.weight": torch.randn(4, cfg.hidden_size, generator=g) * 0.01,
            "double_blocks.0.img_attn.qkv.lora_B.weight": torch.randn(3 * cfg.hidden_size, 4, generator=g) * 0.01}
    dw = merge_lora(dw, lora, cfg.hidden_size, cfg.mlp_hidden)
    vcfg = VAEConfig(latent_channels=cfg.in_channels // 4, block_out_channels=[32, 32, 64, 64], norm_num_groups=8)
    pipe = FluxPipeline(FluxDiT(cfg, dw, device=cuda), VAEDecoder(vcfg, vae_random_weights(vcfg), device=cuda),
                        T5Encoder(tc, t5w, device=cuda), CLIPTextEncoder(cc, cw, device=cuda))
    t5_ids = torch.randint(0, 100, (1, 32), generator=g)  # text length: a multiple of 16
    clip_ids = torch.randint(3, 90, (1, 16), generator=g)
    img = pipe(t5_ids=t5_ids, clip_ids=clip_ids, height=64, width=64, steps=3, seed=1)
    torch.cuda.synchronize()
    ops.check_errors(cuda)
    assert img.shape == (1, 3, 64, 64) and torch.isfinite(img).all()
    assert to_image(img).shape == (1, 64, 64, 3)
