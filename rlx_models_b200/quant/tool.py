"""Checkpoint quantisation tool (``python -m rlx_models_b200.quant.tool``).

    python -m rlx_models_b200.quant.tool --model DIR --out DIR2 --algo gptq --format mxfp4 \\
        [--calib calib.jsonl | --calib-tokens 4096] [--skip lm_head,embed]

Calibration activations of every dense linear come from the fp32 oracle
(forward over the calibration tokens with input taps); each projection is
quantised with RTN, AWQ or GPTQ into MXFP4, NVFP4 or FP8. The output is an
HF-layout checkpoint: MXFP4 weights as ``<name>_blocks`` / ``<name>_scales``
(the gpt-oss packing), FP8 as an ``float8_e4m3fn`` tensor + ``<name>_scale``,
NVFP4 as codes + block scales + tensor scale; ``config.json`` gains a
``quantization_config``. AWQ input scales are folded into the producing norm
(q/k/v: input_layernorm, gate/up: post_attention_layernorm) and left
unfolded (RTN) where no norm produces the input (o_proj, down_proj).
``load_quantized`` reads such a checkpoint back into bf16 weights.

Reference: rlx-quant-calib (calibration CLI, RTN / AWQ / GPTQ, packing sinks).
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from ..config import DecoderConfig
from ..models.oracle import DecoderOracle
from ..weights.safetensors_io import save_file
from ..weights.weight_map import WeightMap
from .calib import FORMATS, awq, gptq, quantize_fp8, quantize_nvfp4
from .mxfp4 import dequantize_mxfp4, quantize_mxfp4

LINEARS = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj", "mlp.gate_proj",
           "mlp.up_proj", "mlp.down_proj")
NORM_OF = {"self_attn.q_proj": "input_layernorm", "self_attn.k_proj": "input_layernorm",
           "self_attn.v_proj": "input_layernorm", "mlp.gate_proj": "post_attention_layernorm",
           "mlp.up_proj": "post_attention_layernorm"}


def pack(name: str, w: torch.Tensor, fmt: str) -> dict[str, torch.Tensor]:
    from .calib import pack_ternary, quantize_bitnet, quantize_int_group
    base = name[:-len(".weight")]
    if fmt in ("int4", "int8"):
        q, sc = quantize_int_group(w, 4 if fmt == "int4" else 8)
        if fmt == "int4":  # two codes per byte, low nibble first (two's complement nibbles)
            u = (q.to(torch.int16) & 0xF).to(torch.uint8)
            q = (u[:, 0::2] | (u[:, 1::2] << 4))
        return {base + f".weight_{fmt}": q, base + ".weight_group_scale": sc}
    if fmt == "bitnet":
        q, sc = quantize_bitnet(w)
        return {base + ".weight_ternary": pack_ternary(q), base + ".weight_scale": sc.reshape(1)}
    if fmt == "mxfp4":
        b, s = quantize_mxfp4(w.float())
        return {base + ".weight_blocks": b, base + ".weight_scales": s}
    if fmt == "fp8":
        q, s = quantize_fp8(w)
        return {name: q, base + ".weight_scale": s}
    c, bs, ts = quantize_nvfp4(w)
    packed = (c[..., 0::2] | (c[..., 1::2] << 4)).to(torch.uint8)
    return {base + ".weight_nvfp4": packed, base + ".weight_block_scale": bs, base + ".weight_tensor_scale":
            ts.reshape(1)}


def load_quantized(path: str) -> dict[str, torch.Tensor]:
    """Quantised checkpoint -> {hf name: bf16 weight} (dequantised)."""
    wm = WeightMap.from_dir(path)
    names = list(wm.keys())
    get = wm.peek
    out = {}
    for n in names:
        if n.endswith(".weight_blocks"):
            base = n[:-len(".weight_blocks")]
            out[base + ".weight"] = dequantize_mxfp4(get(n), get(base + ".weight_scales")).bfloat16()
        elif n.endswith(".weight_nvfp4"):
            base = n[:-len(".weight_nvfp4")]
            p = get(n)
            c = torch.stack([p & 0xF, p >> 4], -1).reshape(*p.shape[:-1], -1)
            from .calib import dequantize_nvfp4
            out[base + ".weight"] = dequantize_nvfp4(c, get(base + ".weight_block_scale"),
                                                     get(base + ".weight_tensor_scale").float()).bfloat16()
        elif n.endswith((".weight_int4", ".weight_int8")):
            from .calib import dequantize_int_group
            base, kind = n.rsplit(".weight_", 1)
            q = get(n)
            if kind == "int4":
                lo = (q & 0xF).to(torch.int8)
                hi = (q >> 4).to(torch.int8)
                lo = torch.where(lo > 7, lo - 16, lo)
                hi = torch.where(hi > 7, hi - 16, hi)
                q = torch.stack([lo, hi], -1).reshape(q.shape[0], -1)
            out[base + ".weight"] = dequantize_int_group(q, get(base + ".weight_group_scale").float()).bfloat16()
        elif n.endswith(".weight_ternary"):
            from .calib import unpack_ternary
            base = n[:-len(".weight_ternary")]
            out[base + ".weight"] = (unpack_ternary(get(n)).float() * get(base + ".weight_scale").float()).bfloat16()
        elif n.endswith(("_scales", "_scale", ".weight_block_scale", ".weight_tensor_scale", ".weight_group_scale")):
            continue
        elif get(n).dtype == torch.float8_e4m3fn:
            out[n] = (get(n).float() * get(n[:-len(".weight")] + ".weight_scale")[:, None]).bfloat16()
        else:
            out[n] = get(n)
    return out


def quantize_checkpoint(src: str, out: str, algo: str = "gptq", fmt: str = "mxfp4", calib_ids=None,
                        device="cpu") -> dict:
    """Quantise every dense decoder linear of ``src`` into ``out``; returns the
    per-linear relative output error on the calibration activations."""
    from .calib import output_error
    gguf_kind = None
    if fmt.startswith("gguf:"):  # e.g. gguf:Q4_K - GGUF output, RTN / AWQ on the ggml block format
        gguf_kind = fmt.split(":", 1)[1]
        from ..weights.gguf import dequantize, quantize
        FORMATS[fmt] = lambda w, k=gguf_kind: dequantize(quantize(w, k), k, w.shape)
        if algo == "gptq":
            raise ValueError("GPTQ targets the group-wise formats; use rtn or awq with a GGUF output")
    cfg = DecoderConfig.from_file(src)
    wm = WeightMap.from_dir(src)
    weights = {n: wm.peek(n) for n in wm.keys()}
    taps: dict = {}
    if algo != "rtn" or calib_ids is not None:
        oracle = DecoderOracle(cfg, weights, device=device)
        oracle.taps = taps
        for ids in calib_ids or []:
            oracle.forward(torch.as_tensor(ids))
        oracle.taps = None
    result, report = {}, {}
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        groups = [(["self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"], "input_layernorm"),
                  (["self_attn.o_proj"], None), (["mlp.gate_proj", "mlp.up_proj"], "post_attention_layernorm"),
                  (["mlp.down_proj"], None)]
        for lins, norm in groups:
            names = [p + l + ".weight" for l in lins if p + l + ".weight" in weights]
            if not names:
                continue
            x = torch.cat(taps[names[0]]).float() if names[0] in taps else None
            s = None
            if algo == "awq" and x is not None and norm is not None:
                _, s, _ = awq(torch.cat([weights[n].float() for n in names]), x, fmt)
                nw = p + norm + ".weight"
                result[nw] = (weights[nw].float() / s).to(weights[nw].dtype)
            for n in names:
                w = weights[n].float()
                if s is not None:
                    stored = w * s[None, :]
                    eff = FORMATS[fmt](stored) / s[None, :]
                elif algo == "gptq" and x is not None:
                    stored = eff = gptq(w, x, fmt).float()
                else:
                    stored, eff = w, FORMATS[fmt](w)
                report[n] = output_error(w, eff, x) if x is not None else None
                result.update({n: stored.to(weights[n].dtype)} if gguf_kind else pack(n, stored, fmt))
    for name, w in weights.items():
        if name not in result and not any(name.endswith(l + ".weight") for l in LINEARS):
            result[name] = w
    os.makedirs(out, exist_ok=True)
    if gguf_kind is not None:
        # GGUF sink: the (AWQ-scaled) weights quantised to a ggml block format in one .gguf file
        from ..weights.gguf import save_gguf
        save_gguf(os.path.join(out, f"model-{gguf_kind}.gguf"), result, cfg, kind=gguf_kind)
        return report
    save_file(result, os.path.join(out, "model.safetensors"))
    hf = cfg.to_hf_dict()
    hf["quantization_config"] = {"quant_method": fmt, "algorithm": algo,
                                 "group_size": {"mxfp4": 32, "nvfp4": 16, "fp8": -1, "int4": 128, "int8": 128,
                                                "bitnet": -1}[fmt]}
    with open(os.path.join(out, "config.json"), "w") as f:
        json.dump(hf, f, indent=1)
    return report


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--algo", default="gptq", choices=["rtn", "awq", "gptq"])
    ap.add_argument("--format", default="mxfp4",
                    help="mxfp4 | nvfp4 | fp8 | int4 | int8 | bitnet | gguf:<ggml type, e.g. Q4_K, Q8_0, Q6_K>")
    ap.add_argument("--calib-tokens", type=int, default=2048)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    cfg = DecoderConfig.from_file(a.model)
    g = torch.Generator().manual_seed(a.seed)
    calib = [torch.randint(0, cfg.vocab_size, (min(512, a.calib_tokens),), generator=g)
             for _ in range(max(1, a.calib_tokens // 512))]
    rep = quantize_checkpoint(a.model, a.out, a.algo, a.format, calib)
    errs = [v for v in rep.values() if v is not None]
    print(json.dumps({"linears": len(rep), "mean_output_error": sum(errs) / len(errs) if errs else None}))


if __name__ == "__main__":
    main()
