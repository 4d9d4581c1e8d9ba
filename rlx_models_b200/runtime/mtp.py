"""Multi-token-prediction (MTP) heads shipped inside checkpoints, as draft
proposers for speculative decoding.

Qwen3.5 / Qwen3-Next checkpoints carry an ``mtp.*`` module next to the model:

    e  = RMSNorm_e(embed(token_{t+1}))            pre_fc_norm_embedding
    h  = RMSNorm_h(feature_t)                     pre_fc_norm_hidden (feature = the
                                                  target's final-normed hidden state)
    x  = fc([e ; h])                              2H -> H
    x  = decoder layer j (full attention with the output gate, QK-norm, partial
         RoPE at position t + 1; MoE or dense MLP, as the target's layers)
    y  = RMSNorm(x)                               mtp.norm
    p  = softmax(lm_head(y))                      -> token_{t+2} (embedding and head shared)

Drafting k tokens chains the head on its own output: the normalised ``y`` of
one step is the feature of the next. ``MTPHead.propose`` has the interface of
the learned ``DraftHead`` (``runtime/draft_head.py``), so ``SpeculativeDecoder``
verifies its proposals against the target exactly as for the other proposers
(the output equals the target's greedy decoding whatever the head proposes).
The head runs the layer with the fp32 oracle's attention / MoE code over a
window of the last positions (no KV cache of its own).

Reference: the reference's MTP drafting for Qwen3.5 (crates/rlx-qwen35/src/cache.rs:167-179);
the layout of the ``mtp.*`` tensors is the released checkpoints'.
"""
from __future__ import annotations

import torch

from ..models.qwen35 import Qwen35Config, Qwen35Oracle


class _MTPLayerSource:
    """The ``mtp.*`` tensors under the names the oracle's layer code reads:
    ``model.layers.{N + j}.X`` -> ``mtp.layers.{j}.X`` (N = target layers)."""

    def __init__(self, weights, n_layers: int):
        self.w, self.n = weights, n_layers
        self.get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])

    def _map(self, name: str) -> str:
        if name.startswith("model.layers."):
            rest = name[len("model.layers."):]
            i, tail = rest.split(".", 1)
            if int(i) >= self.n:
                return f"mtp.layers.{int(i) - self.n}.{tail}"
        return name

    def keys(self):
        out = []
        for k in self.w.keys():
            if k.startswith("mtp.layers."):
                j, tail = k[len("mtp.layers."):].split(".", 1)
                out.append(f"model.layers.{self.n + int(j)}.{tail}")
            elif not k.startswith("mtp."):
                out.append(k)
        return out

    def __contains__(self, name):
        return self._map(name) in self.w

    def __getitem__(self, name):
        return self.get(self._map(name))


def has_mtp(weights) -> bool:
    return any(k.startswith("mtp.") for k in weights.keys())


class MTPHead:
    uses_positions = True

    def __init__(self, cfg: Qwen35Config, weights, device="cpu", layer: int = 0):
        if not has_mtp(weights):
            raise ValueError("checkpoint has no mtp.* tensors")
        self.cfg, self.device = cfg, torch.device(device)
        self.j = layer
        self.L = cfg.num_hidden_layers + layer  # virtual index of the MTP layer
        src = _MTPLayerSource(weights, cfg.num_hidden_layers)
        self.oracle = Qwen35Oracle(cfg, src, device=device)
        t = lambda n: src[n].to(self.device, torch.float32)  # noqa: E731
        self.fc = t("mtp.fc.weight")
        self.n_e = t("mtp.pre_fc_norm_embedding.weight") + 1.0   # (1 + w) RMSNorms, as the model's
        self.n_h = t("mtp.pre_fc_norm_hidden.weight") + 1.0
        self.n_out = t("mtp.norm.weight") + 1.0
        self.embed = self.oracle._t("model.embed_tokens.weight")  # shared with the target
        self.head = self.embed if cfg.tie_word_embeddings else self.oracle._t("lm_head.weight")

    def _rms(self, x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.cfg.rms_norm_eps) * w

    def layer(self, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        o, p = self.oracle, f"model.layers.{self.L}."
        h = x + o.attention(self.L, o._rms(x, p + "input_layernorm.weight"), pos)
        xn = o._rms(h, p + "post_attention_layernorm.weight")
        return h + (o.moe(self.L, xn) if self.cfg.num_experts else o._swiglu(xn, p + "mlp."))

    @torch.no_grad()
    def features(self, h: torch.Tensor, next_tokens: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """h [W, H] features of positions pos - 1, next_tokens [W] the tokens at
        ``pos`` -> normalised MTP outputs [W, H] (features of positions ``pos``)."""
        e = self._rms(self.embed[next_tokens.long()], self.n_e)
        x = torch.cat([e, self._rms(h.float(), self.n_h)], -1) @ self.fc.t()
        return self._rms(self.layer(x, pos), self.n_out)

    def logits(self, y: torch.Tensor) -> torch.Tensor:
        return y @ self.head.t()

    @torch.no_grad()
    def propose(self, h_ctx: torch.Tensor, tok_ctx: list[int], k: int, pos0: int = 0) -> list[int]:
        """``h_ctx`` [W, H]: target features of W consecutive positions; ``tok_ctx``:
        the W tokens that followed them, the first at position ``pos0``. Returns
        k greedy draft tokens."""
        h = h_ctx.float().to(self.device)
        toks = torch.tensor(tok_ctx, device=self.device)
        out = []
        for _ in range(k):
            pos = torch.arange(pos0, pos0 + toks.shape[0], device=self.device)
            y = self.features(h, toks, pos)
            nxt = int(self.logits(y[-1:]).argmax(-1))
            out.append(nxt)
            h = torch.cat([h, y[-1:]], 0)
            toks = torch.cat([toks, torch.tensor([nxt], device=self.device)])
        return out


def random_mtp_weights(cfg: Qwen35Config, seed: int = 1, device="cpu", dtype=torch.bfloat16) -> dict:
    """Seeded ``mtp.*`` tensors of one MTP layer (full attention + the target's MLP kind)."""
    from ..models.qwen35 import random_weights
    one = Qwen35Config(**{**cfg.__dict__, "num_hidden_layers": 1, "layer_types": ["full_attention"],
                          "tie_word_embeddings": True})
    w = random_weights(one, seed, device, dtype)
    out = {}
    for k, v in w.items():
        if k.startswith("model.layers.0."):
            out["mtp.layers.0." + k[len("model.layers.0."):]] = v
    H = cfg.hidden_size
    g = torch.Generator(device=device).manual_seed(seed + 1)
    out["mtp.fc.weight"] = (torch.randn(H, 2 * H, generator=g, device=device) / (2 * H) ** 0.5).to(dtype)
    for n in ("pre_fc_norm_embedding", "pre_fc_norm_hidden", "norm"):
        out[f"mtp.{n}.weight"] = (0.1 * torch.randn(H, generator=g, device=device)).to(dtype)
    return out
