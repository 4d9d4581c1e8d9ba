"""FLUX pipeline parts on CPU: VAE decoder shapes and the LDM -> diffusers
name mapping, LoRA merging in the three key dialects."""
import torch

from rlx_models_b200.models import flux_lora as FL
from rlx_models_b200.models import flux_vae as FV


def _ldm_name(d: str, levels: int = 4) -> str:
    """Inverse of ldm_to_diffusers for the test (diffusers -> LDM)."""
    r = d[len("decoder."):]
    if r.startswith("mid_block.resnets."):
        i, _, t = r[len("mid_block.resnets."):].partition(".")
        return f"decoder.mid.block_{int(i) + 1}.{t}"
    if r.startswith("mid_block.attentions.0."):
        n, _, p = r[len("mid_block.attentions.0."):].rpartition(".")
        n = {"group_norm": "norm", "to_q": "q", "to_k": "k", "to_v": "v", "to_out.0": "proj_out"}[n]
        return f"decoder.mid.attn_1.{n}.{p}"
    if r.startswith("up_blocks."):
        i, _, rest = r[len("up_blocks."):].partition(".")
        k = levels - 1 - int(i)
        if rest.startswith("resnets."):
            j, _, t = rest[len("resnets."):].partition(".")
            return f"decoder.up.{k}.block.{j}.{t.replace('conv_shortcut', 'nin_shortcut')}"
        return f"decoder.up.{k}.upsample.conv.{rest.split('.')[-1]}"
    if r.startswith("conv_norm_out."):
        return "decoder.norm_out." + r.split(".")[-1]
    return d


def test_vae_decoder_shapes_and_ldm_names():
    cfg = FV.VAEConfig(block_out_channels=[16, 16, 32, 32], norm_num_groups=8)
    w = FV.vae_random_weights(cfg, 0)
    z = torch.randn(1, 16, 6, 5)
    img = FV.VAEDecoder(cfg, w).decode(z)
    assert img.shape == (1, 3, 48, 40) and torch.isfinite(img).all()
    for d in w:
        assert FV.ldm_to_diffusers(_ldm_name(d)) in (d, None)
    ldm = {}
    for d, t in w.items():
        n = _ldm_name(d)
        ldm[n] = t.view(*t.shape, 1, 1) if (".attn_1." in n and n.endswith(".weight") and t.dim() == 2
                                            and not n.endswith("norm.weight")) else t
    img2 = FV.VAEDecoder(cfg, ldm).decode(z)
    assert torch.allclose(img, img2, atol=1e-5)
    u8 = FV.to_image(img)
    assert u8.dtype == torch.uint8 and u8.shape == (1, 48, 40, 3)


def test_flux_lora_three_dialects_agree():
    from rlx_models_b200.config import FluxConfig
    from rlx_models_b200.models.flux_common import flux_random_weights
    cfg = FluxConfig(hidden_size=64, num_heads=2, depth=1, depth_single_blocks=1, context_in_dim=32,
                     vec_in_dim=16, mlp_ratio=4.0)
    base = flux_random_weights(cfg, 0, dtype=torch.float32)
    H, mlp = cfg.hidden_size, int(cfg.hidden_size * cfg.mlp_ratio)
    g = torch.Generator().manual_seed(1)
    r = 4
    A_q, B_q = torch.randn(r, H, generator=g), torch.randn(H, r, generator=g)
    A_mlp, B_mlp = torch.randn(r, H, generator=g), torch.randn(mlp, r, generator=g)
    A_n, B_n = torch.randn(r, H, generator=g), torch.randn(2 * H, r, generator=g)
    # the same three updates in each dialect
    bfl_q = torch.zeros(3 * H, r)
    bfl_q[H:2 * H] = B_q  # to_k band of img_attn.qkv
    bfl_l1 = torch.zeros(3 * H + mlp, r)
    bfl_l1[3 * H:] = B_mlp  # proj_mlp band of linear1
    bfl_n = torch.cat([B_n[H:], B_n[:H]], 0)  # BFL order (shift, scale)
    bfl = {"double_blocks.0.img_attn.qkv.lora_A.weight": A_q, "double_blocks.0.img_attn.qkv.lora_B.weight": bfl_q,
           "single_blocks.0.linear1.lora_A.weight": A_mlp, "single_blocks.0.linear1.lora_B.weight": bfl_l1,
           "final_layer.adaLN_modulation.1.lora_A.weight": A_n,
           "final_layer.adaLN_modulation.1.lora_B.weight": bfl_n}
    diff = {"transformer.transformer_blocks.0.attn.to_k.lora_A.weight": A_q,
            "transformer.transformer_blocks.0.attn.to_k.lora_B.weight": B_q,
            "transformer.single_transformer_blocks.0.proj_mlp.lora_A.weight": A_mlp,
            "transformer.single_transformer_blocks.0.proj_mlp.lora_B.weight": B_mlp,
            "transformer.norm_out.linear.lora_A.weight": A_n, "transformer.norm_out.linear.lora_B.weight": B_n}
    kohya = {}
    for k, v in bfl.items():
        mod, _, suf = k.partition(".lora_")
        kk = "lora_unet_" + mod.replace(".", "_")
        kohya[kk + (".lora_down.weight" if suf.startswith("A") else ".lora_up.weight")] = v
        kohya[kk + ".alpha"] = torch.tensor(float(2 * r))  # alpha 2r -> scale 2
    m1 = FL.merge_lora(base, bfl, H, mlp, scale=2.0)
    m2 = FL.merge_lora(base, diff, H, mlp, scale=2.0)
    m3 = FL.merge_lora(base, kohya, H, mlp, scale=1.0)
    for k in base:
        assert torch.allclose(m1[k], m2[k], atol=1e-5), k
        assert torch.allclose(m1[k], m3[k], atol=1e-5), k
    n = "double_blocks.0.img_attn.qkv.weight"
    assert torch.allclose(m1[n] - base[n], 2.0 * bfl_q @ A_q, atol=1e-5)
    assert torch.equal(m1["double_blocks.0.txt_attn.qkv.weight"], base["double_blocks.0.txt_attn.qkv.weight"])
