"""Checkpoint tensor names of model families that differ only in naming from
the canonical layout the builders read (Qwen3-MoE style MoE names).

Mixtral and MiniMax-M2: ``block_sparse_moe.gate`` is the router, ``block_sparse_moe.experts.{e}.w1 / w3 / w2``
are gate / up / down. ``canonical_name`` maps a checkpoint name to the
canonical one; ``CanonicalView`` presents a weight source under canonical names.
Llama-4 (``Llama4View``) also changes tensor layouts: fused expert banks are
split into per-expert matrices.
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


class Llama4View:
    """Llama-4 text weights under the canonical MoE names.

    ``feed_forward.`` -> ``mlp.``; the router ``feed_forward.router`` ->
    ``mlp.gate``; the always-on shared expert ``feed_forward.shared_expert`` ->
    ``mlp.shared_experts`` (ungated); the fused expert banks
    ``feed_forward.experts.gate_up_proj`` [E, H, 2I] (gate = the first I
    columns) and ``feed_forward.experts.down_proj`` [E, I, H] -> per-expert
    ``mlp.experts.{e}.gate_proj / up_proj / down_proj.weight`` ([I, H], [I, H],
    [H, I]). The multimodal release's ``language_model.`` prefix is dropped
    (its vision tower is not part of the text model)."""

    def __init__(self, weights):
        self.w = weights
        # peek: a fused bank is read once per expert
        self.get = (lambda k: weights.peek(k)) if hasattr(weights, "peek") else (lambda k: weights[k])
        self.map: dict[str, tuple] = {}
        for n in list(weights.keys()):
            c = n
            for pre in ("language_model.", "model.language_model."):
                if c.startswith(pre):
                    c = c[len(pre):]
                    if not c.startswith(("model.", "lm_head")):
                        c = "model." + c
            if c.startswith(("vision_model.", "multi_modal_projector.", "model.vision_model.",
                             "model.multi_modal_projector.")):
                continue
            c = c.replace(".feed_forward.router.", ".mlp.gate.").replace(".feed_forward.shared_expert.",
                                                                         ".mlp.shared_experts.")
            c = c.replace(".feed_forward.", ".mlp.")
            if c.endswith(".mlp.experts.gate_up_proj"):
                pre = c[: -len("gate_up_proj")]
                for e in range(self._n_experts(n)):
                    self.map[pre + f"{e}.gate_proj.weight"] = (n, e, "gate")
                    self.map[pre + f"{e}.up_proj.weight"] = (n, e, "up")
            elif c.endswith(".mlp.experts.down_proj"):
                pre = c[: -len("down_proj")]
                for e in range(self._n_experts(n)):
                    self.map[pre + f"{e}.down_proj.weight"] = (n, e, "down")
            else:
                self.map[c] = (n, None, None)
        self._bank: dict[str, object] = {}

    def _n_experts(self, n) -> int:
        return int(self.w.shape(n)[0]) if hasattr(self.w, "shape") else int(self.w[n].shape[0])

    def keys(self):
        return list(self.map)

    def __contains__(self, name):
        return name in self.map

    def _bank_of(self, n):
        if n not in self._bank:
            self._bank = {n: self.get(n)}  # one fused bank resident at a time
        return self._bank[n]

    def take(self, name, **kw):
        n, e, part = self.map[name]
        if e is None:
            t = self.get(n)
        else:
            b = self._bank_of(n)[e]
            if part == "down":
                t = b.t()
            else:
                inter = b.shape[1] // 2
                t = (b[:, :inter] if part == "gate" else b[:, inter:]).t()
        dt, dev = kw.get("dtype"), kw.get("device")
        return t if dt is None and dev is None else t.to(device=dev, dtype=dt)

    def __getitem__(self, name):
        return self.take(name)

    def as_dict(self) -> dict:
        return {k: self.take(k).contiguous() for k in self.map}


class LanguageModelView:
    """The text model inside a multimodal checkpoint, under the decoder's names:
    ``model.language_model.X`` -> ``model.X`` (the vision tower ``model.visual.*``
    and any projector are left out; ``lm_head`` stays), and transformers'
    fused expert banks ``mlp.experts.gate_up_proj`` [E, 2I, H] /
    ``mlp.experts.down_proj`` [E, H, I] seen as per-expert matrices."""

    _DROP = ("model.visual.", "visual.", "model.vision_tower.", "vision_tower.", "model.multi_modal_projector.",
             "multi_modal_projector.", "mtp.")

    def __init__(self, weights):
        self.w = weights
        self.get = (lambda k: weights.peek(k)) if hasattr(weights, "peek") else (lambda k: weights[k])
        self.map: dict[str, tuple] = {}
        for n in list(weights.keys()):
            if n.startswith(self._DROP):
                continue
            c = n.replace("model.language_model.", "model.", 1)
            if c.endswith("mlp.experts.gate_up_proj"):
                pre = c[: -len("gate_up_proj")]
                for e in range(self._dim0(n)):
                    self.map[pre + f"{e}.gate_proj.weight"] = (n, e, "gate")
                    self.map[pre + f"{e}.up_proj.weight"] = (n, e, "up")
            elif c.endswith("mlp.experts.down_proj"):
                pre = c[: -len("down_proj")]
                for e in range(self._dim0(n)):
                    self.map[pre + f"{e}.down_proj.weight"] = (n, e, "down")
            else:
                self.map[c] = (n, None, None)

    def _dim0(self, n) -> int:
        return int(self.w.shape(n)[0]) if hasattr(self.w, "shape") else int(self.w[n].shape[0])

    @staticmethod
    def applies(weights) -> bool:
        return any(k.startswith("model.language_model.") for k in weights.keys())

    def keys(self):
        return list(self.map)

    def __contains__(self, name):
        return name in self.map

    def take(self, name, **kw):
        n, e, part = self.map[name]
        t = self.get(n) if e is None else self.get(n)[e]
        if part in ("gate", "up"):
            inter = t.shape[0] // 2
            t = t[:inter] if part == "gate" else t[inter:]
        dt, dev = kw.get("dtype"), kw.get("device")
        return t if dt is None and dev is None else t.to(device=dev, dtype=dt)

    def __getitem__(self, name):
        return self.take(name)

    def as_dict(self) -> dict:
        return {k: self.take(k).contiguous() for k in self.map}
