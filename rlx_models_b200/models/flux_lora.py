"""LoRA adapters for the FLUX.1 DiT, merged into the BFL-named base weights
(W[rows] += scale * B @ A, scale = user_scale * alpha / rank, alpha = rank
when absent) before the model is built, so inference runs the plain kernels.

Three key dialects:
* BFL module names: ``double_blocks.3.img_attn.qkv.lora_A.weight`` (also under
  ``diffusion_model.`` / ``transformer.``);
* kohya: ``lora_unet_double_blocks_3_img_attn_qkv.lora_down.weight`` with
  ``.lora_up.weight`` and ``.alpha``;
* diffusers / PEFT: ``transformer.transformer_blocks.3.attn.to_q.lora_A.weight``.
  diffusers splits projections that BFL fuses (``to_q`` / ``to_k`` /
  ``to_v`` -> ``img_attn.qkv``; single blocks' q / k / v / ``proj_mlp`` ->
  ``linear1``), so such an adapter updates a row band of the fused matrix;
  ``norm_out.linear`` orders its halves (scale, shift) where BFL has
  (shift, scale), so its rows are swapped.

Reference: crates/rlx-flux1/src/lora.rs (the same three dialects, row bands,
norm_out half swap).
"""
from __future__ import annotations

import re

import torch


def _diffusers_target(mod: str, H: int, mlp: int):
    """diffusers module path -> (BFL module, row offset, rows or None, swap_halves)."""
    m = re.match(r"transformer_blocks\.(\d+)\.(.+)$", mod)
    if m:
        i, r = m.group(1), m.group(2)
        p = f"double_blocks.{i}."
        table = {"attn.to_q": ("img_attn.qkv", 0), "attn.to_k": ("img_attn.qkv", H), "attn.to_v": ("img_attn.qkv", 2 * H),
                 "attn.add_q_proj": ("txt_attn.qkv", 0), "attn.add_k_proj": ("txt_attn.qkv", H),
                 "attn.add_v_proj": ("txt_attn.qkv", 2 * H), "attn.to_out.0": ("img_attn.proj", 0),
                 "attn.to_add_out": ("txt_attn.proj", 0), "ff.net.0.proj": ("img_mlp.0", 0), "ff.net.2": ("img_mlp.2", 0),
                 "ff_context.net.0.proj": ("txt_mlp.0", 0), "ff_context.net.2": ("txt_mlp.2", 0),
                 "norm1.linear": ("img_mod.lin", 0), "norm1_context.linear": ("txt_mod.lin", 0)}
        if r in table:
            t, off = table[r]
            return p + t, off, False
        return None
    m = re.match(r"single_transformer_blocks\.(\d+)\.(.+)$", mod)
    if m:
        i, r = m.group(1), m.group(2)
        p = f"single_blocks.{i}."
        table = {"attn.to_q": ("linear1", 0), "attn.to_k": ("linear1", H), "attn.to_v": ("linear1", 2 * H),
                 "proj_mlp": ("linear1", 3 * H), "proj_out": ("linear2", 0), "norm.linear": ("modulation.lin", 0)}
        if r in table:
            t, off = table[r]
            return p + t, off, False
        return None
    glob = {"x_embedder": ("img_in", False), "context_embedder": ("txt_in", False),
            "time_text_embed.timestep_embedder.linear_1": ("time_in.in_layer", False),
            "time_text_embed.timestep_embedder.linear_2": ("time_in.out_layer", False),
            "time_text_embed.guidance_embedder.linear_1": ("guidance_in.in_layer", False),
            "time_text_embed.guidance_embedder.linear_2": ("guidance_in.out_layer", False),
            "time_text_embed.text_embedder.linear_1": ("vector_in.in_layer", False),
            "time_text_embed.text_embedder.linear_2": ("vector_in.out_layer", False),
            "norm_out.linear": ("final_layer.adaLN_modulation.1", True), "proj_out": ("final_layer.linear", False)}
    if mod in glob:
        t, swap = glob[mod]
        return t, 0, swap
    return None


def lora_patches(lora: dict[str, torch.Tensor], base_modules: set[str], hidden: int, mlp_hidden: int,
                 user_scale: float = 1.0) -> dict[str, list[tuple[int, torch.Tensor, bool]]]:
    """-> {BFL weight name: [(row offset, delta [rows, in], swap_halves)]}."""
    kohya = {m.replace(".", "_"): m for m in base_modules}
    groups: dict[str, dict] = {}
    for k, v in lora.items():
        for suf, role in ((".lora_A.weight", "A"), (".lora_B.weight", "B"), (".lora_down.weight", "A"),
                          (".lora_up.weight", "B"), (".alpha", "alpha")):
            if k.endswith(suf):
                groups.setdefault(k[:-len(suf)], {})[role] = v
                break
    out: dict[str, list] = {}
    for mod, parts in groups.items():
        if "A" not in parts or "B" not in parts:
            raise ValueError(f"LoRA module {mod}: needs both down (A) and up (B) matrices")
        A, B = parts["A"].float(), parts["B"].float()
        rank = A.shape[0]
        alpha = float(parts["alpha"]) if "alpha" in parts else float(rank)
        delta = (B @ A) * (user_scale * alpha / rank)
        name = mod
        for pre in ("diffusion_model.", "transformer.", "base_model.model."):
            if name.startswith(pre):
                name = name[len(pre):]
        target, off, swap = None, 0, False
        if name.startswith("lora_unet_"):
            target = kohya.get(name[len("lora_unet_"):])
        elif name in base_modules:
            target = name
        else:
            t = _diffusers_target(name, hidden, mlp_hidden)
            if t is not None:
                target, off, swap = t
        if target is None or target not in base_modules:
            raise KeyError(f"LoRA module {mod!r} does not map onto a FLUX DiT weight")
        out.setdefault(target + ".weight", []).append((off, delta, swap))
    return out


def merge_lora(base: dict[str, torch.Tensor], lora: dict[str, torch.Tensor], hidden: int, mlp_hidden: int,
               scale: float = 1.0) -> dict[str, torch.Tensor]:
    """New weight dict with every adapter merged (only the patched tensors are copied)."""
    mods = {n[:-len(".weight")] for n in base if n.endswith(".weight")}
    out = dict(base)
    for name, patches in lora_patches(lora, mods, hidden, mlp_hidden, scale).items():
        w = base[name].float().clone()
        for off, delta, swap in patches:
            if swap:  # (scale, shift) adapter rows onto BFL's (shift, scale)
                h = delta.shape[0] // 2
                delta = torch.cat([delta[h:], delta[:h]], 0)
            w[off:off + delta.shape[0]] += delta
        out[name] = w.to(base[name].dtype)
    return out
