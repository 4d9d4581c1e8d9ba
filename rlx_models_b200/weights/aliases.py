"""Checkpoint tensor names of model families that differ only in naming from
the canonical layout the builders read (Qwen3-MoE style MoE names).

Mixtral and MiniMax-M2: ``block_sparse_moe.gate`` is the router, ``block_sparse_moe.experts.{e}.w1 / w3 / w2``
are gate / up / down. ``canonical_name`` maps a checkpoint name to the
canonical one; ``CanonicalView`` presents a weight source under canonical names.
"""
from __future__ import annotations

import re

_MIXTRAL = [(re.compile(r"\.block_sparse_moe\.gate\."), ".mlp.gate."),
            (re.compile(r"\.block_sparse_moe\.experts\.(\d+)\.w1\."), r".mlp.experts.\1.gate_proj."),
            (re.compile(r"\.block_sparse_moe\.experts\.(\d+)\.w3\."), r".mlp.experts.\1.up_proj."),
            (re.compile(r"\.block_sparse_moe\.experts\.(\d+)\.w2\."), r".mlp.experts.\1.down_proj.")]


# MiniMax-M2: Mixtral's expert names plus the routing correction bias, which
# sits on the MoE block (``block_sparse_moe.`` in the release, ``mlp.`` in transformers)
_MINIMAX = _MIXTRAL + [(re.compile(r"\.(?:block_sparse_moe|mlp)\.e_score_correction_bias$"),
                        ".mlp.gate.e_score_correction_bias")]


def canonical_name(model_type: str, name: str) -> str:
    for pat, rep in {"mixtral": _MIXTRAL, "minimax_m2": _MINIMAX}.get(model_type, ()):
        name = pat.sub(rep, name)
    return name


class CanonicalView:
    """Weight source (dict or WeightMap-like) seen under canonical names."""

    def __init__(self, weights, model_type: str):
        self.w = weights
        names = list(weights.keys())
        self.to_ckpt = {canonical_name(model_type, n): n for n in names}

    def keys(self):
        return list(self.to_ckpt)

    def __contains__(self, name):
        return name in self.to_ckpt

    def take(self, name, **kw):
        n = self.to_ckpt[name]
        return self.w.take(n, **kw) if hasattr(self.w, "take") else self.w[n]

    def __getitem__(self, name):
        return self.take(name)


def split_fused_experts(sd: dict, gate_up_order: str = "gate_first") -> dict:
    """transformers' in-memory MoE layout (``mlp.experts.gate_up_proj`` [E, 2I, H],
    ``mlp.experts.down_proj`` [E, H, I]) -> the released checkpoints' per-expert
    names (``mlp.experts.{e}.gate_proj / up_proj / down_proj.weight``). Other
    tensors pass through; 3-D tensors whose layout differs (gpt-oss's
    [E, H, 2I] interleaved gate/up) are left to their own loaders."""
    out = {}
    for k, v in sd.items():
        if k.endswith("mlp.experts.gate_up_proj") and v.dim() == 3 and v.shape[1] % 2 == 0:
            pre = k[: -len("gate_up_proj")]
            inter = v.shape[1] // 2
            for e in range(v.shape[0]):
                out[pre + f"{e}.gate_proj.weight"] = v[e, :inter]
                out[pre + f"{e}.up_proj.weight"] = v[e, inter:]
        elif k.endswith("mlp.experts.down_proj") and v.dim() == 3:
            pre = k[: -len("down_proj")]
            for e in range(v.shape[0]):
                out[pre + f"{e}.down_proj.weight"] = v[e]
        else:
            out[k] = v
    return out


class FusedSplitView:
    """Weight source with fused dense projections presented as the separate
    ones the builders read: ``self_attn.qkv_proj`` -> q / k / v rows and
    ``mlp.gate_up_proj`` -> gate / up rows (Phi-3 layout)."""

    def __init__(self, weights, q_size: int, kv_size: int, intermediate: int):
        self.w = weights
        self.map: dict[str, tuple[str, int | None, int | None]] = {}
        for n in list(weights.keys()):
            if n.endswith("self_attn.qkv_proj.weight") or n.endswith("self_attn.qkv_proj.bias"):
                pre, suf = n.rsplit("qkv_proj.", 1)
                for part, (a, ln) in zip("qkv", ((0, q_size), (q_size, kv_size), (q_size + kv_size, kv_size))):
                    self.map[f"{pre}{part}_proj.{suf}"] = (n, a, ln)
            elif n.endswith("mlp.gate_up_proj.weight"):
                pre = n[: -len("gate_up_proj.weight")]
                self.map[pre + "gate_proj.weight"] = (n, 0, intermediate)
                self.map[pre + "up_proj.weight"] = (n, intermediate, intermediate)
            else:
                self.map[n] = (n, None, None)

    @staticmethod
    def needed(weights) -> bool:
        return any(n.endswith("qkv_proj.weight") or n.endswith("mlp.gate_up_proj.weight") for n in weights.keys())

    def keys(self):
        return list(self.map)

    def __contains__(self, name):
        return name in self.map

    def take(self, name, **kw):
        n, a, ln = self.map[name]
        t = self.w.take(n) if hasattr(self.w, "take") else self.w[n]
        return t if a is None else t.narrow(0, a, ln)

    def __getitem__(self, name):
        return self.take(name)


class ModelPrefixView:
    """Weights of a bare base model (``embed_tokens.weight``, ``layers.N...``,
    ``norm.weight``) seen under the ``model.``-prefixed names the decoder
    builders read; names that already carry the prefix pass through."""

    def __init__(self, weights):
        self.w = weights
        self.map = {}
        for n in list(weights.keys()):
            self.map[n if n.startswith(("model.", "lm_head.")) else "model." + n] = n

    def keys(self):
        return list(self.map)

    def __contains__(self, name):
        return name in self.map

    def take(self, name, **kw):
        n = self.map[name]
        return self.w.take(n, **kw) if hasattr(self.w, "take") else self.w[n]

    def __getitem__(self, name):
        return self.take(name)
