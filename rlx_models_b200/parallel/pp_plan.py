"""Pipeline stage planner: contiguous layer ranges per device.

Input: per-layer resident bytes (weights + KV cache at the planned context)
and state kind (attention KV / recurrent), per-node memory budgets (plus
optional network RTT and bytes already cached on the node), and the bytes of
the first stage's embedding and the last stage's final norm + LM head. Output:
one stage per node in pipeline order, each with its layer range, roles
(driver + embedding first, readout last), state affinity, migration policy
and reason codes, plus the activation boundaries between stages.

Placement: nodes are ordered best first (memory, then cached bytes, minus an
RTT penalty), then layers are cut into contiguous ranges that MINIMISE THE
LARGEST STAGE LOAD RELATIVE TO ITS NODE'S MEMORY (an exact dynamic program
over cut points, embedding / head bytes included in the end stages). A
pipeline runs at the pace of its slowest stage, and on one NVSwitch node all
links cost the same, so balancing bytes (which track both the weight stream of
decode and the FLOPs of prefill for a uniform decoder) is the objective; a
proportional split would give the head stage the same layers as the others
although it also holds the vocabulary projection.

Reference: crates/rlx-protocol/src/topology.rs (`plan` :246, roles,
StateAffinity, MigrationPolicy, reason codes); the reference splits layers in
proportion to node VRAM.
"""
from __future__ import annotations

from dataclasses import dataclass, field

ROLE_DRIVER, ROLE_EMBEDDING, ROLE_INTERMEDIATE, ROLE_READOUT = "driver", "embedding", "intermediate", "readout"


@dataclass
class LayerSpec:
    index: int
    param_bytes: int
    has_attention: bool = True
    has_recurrent: bool = False
    kv_bytes: int = 0  # KV cache bytes this layer holds at the planned context / batch


@dataclass
class NodeSpec:
    id: str
    mem_bytes: int
    rtt_ms: float | None = None
    cached_bytes: int = 0


@dataclass
class StagePlan:
    stage_index: int
    node_id: str
    layer_start: int
    layer_end: int
    roles: list[str]
    bytes: int
    utilisation: float
    state_affinity: str
    migration_policy: str
    reasons: list[str] = field(default_factory=list)

    @property
    def layer_count(self) -> int:
        return self.layer_end - self.layer_start


@dataclass
class Boundary:
    src_stage: int
    dst_stage: int
    after_layer: int
    carries: str = "activations"  # hidden states only; KV / recurrent state stays on its stage


@dataclass
class TopologyPlan:
    stages: list[StagePlan]
    boundaries: list[Boundary]
    max_utilisation: float
    diagnostics: list[str] = field(default_factory=list)

    def ranges(self) -> list[tuple[int, int]]:
        return [(s.layer_start, s.layer_end) for s in self.stages]


class PlanError(ValueError):
    pass


def classify(layers: list[LayerSpec]) -> str:
    a = any(l.has_attention for l in layers)
    r = any(l.has_recurrent for l in layers)
    return {(False, False): "stateless", (True, False): "attention_kv", (False, True): "recurrent",
            (True, True): "mixed"}[(a, r)]


def migration(affinity: str, allow_state_transfer: bool) -> str:
    if affinity == "stateless":
        return "freely_movable"
    if affinity == "attention_kv":
        return "costed_kv"
    return "recurrent_state_transfer_allowed" if allow_state_transfer else "sticky_recurrent_owner"


def _node_score(n: NodeSpec) -> float:
    return n.mem_bytes + 2 * n.cached_bytes - (n.rtt_ms or 0.0) * (16 << 20)


def plan(layers: list[LayerSpec], nodes: list[NodeSpec], *, embed_bytes: int = 0, head_bytes: int = 0,
         allow_state_transfer: bool = False, reserve_frac: float = 0.0) -> TopologyPlan:
    if not layers:
        raise PlanError("no layers")
    if not nodes:
        raise PlanError("no nodes")
    idx = [l.index for l in layers]
    if idx != list(range(idx[0], idx[0] + len(idx))):
        raise PlanError("layer indices must be contiguous and ascending")
    S = min(len(nodes), len(layers))
    order = sorted(range(len(nodes)), key=lambda i: (-_node_score(nodes[i]), i))[:S]
    ns = [nodes[i] for i in order]
    cap = [max(1.0, n.mem_bytes * (1.0 - reserve_frac)) for n in ns]
    L = len(layers)
    cost = [l.param_bytes + l.kv_bytes for l in layers]
    pre = [0]
    for c in cost:
        pre.append(pre[-1] + c)

    def load(s, a, b):  # stage s holds layers [a, b)
        x = pre[b] - pre[a]
        if s == 0:
            x += embed_bytes
        if s == S - 1:
            x += head_bytes
        return x / cap[s]

    INF = float("inf")
    # best[s][b]: min over cuts of the max utilisation of stages 0..s covering layers [0, b)
    best = [[INF] * (L + 1) for _ in range(S)]
    cut = [[0] * (L + 1) for _ in range(S)]
    for b in range(1, L - S + 2):
        best[0][b] = load(0, 0, b)
    for s in range(1, S):
        for b in range(s + 1, L - (S - 1 - s) + 1):
            for a in range(s, b):
                v = max(best[s - 1][a], load(s, a, b))
                if v < best[s][b]:
                    best[s][b], cut[s][b] = v, a
    bounds = [L]
    for s in range(S - 1, 0, -1):
        bounds.append(cut[s][bounds[-1]])
    bounds.append(0)
    bounds.reverse()
    stages, diags = [], []
    for s in range(S):
        a, b = bounds[s], bounds[s + 1]
        lay = layers[a:b]
        aff = classify(lay)
        mig = migration(aff, allow_state_transfer)
        roles = ([ROLE_DRIVER, ROLE_EMBEDDING] if s == 0 else []) + ([ROLE_READOUT] if s == S - 1 else [])
        roles = roles or [ROLE_INTERMEDIATE]
        reasons = {"costed_kv": ["attention_kv_costed"], "sticky_recurrent_owner": ["recurrent_owner_sticky"],
                   "recurrent_state_transfer_allowed": ["recurrent_state_transfer_allowed"]}.get(mig, [])
        if ns[s].cached_bytes > 0:
            reasons.append("cache_locality_preferred")
        if ns[s].rtt_ms:
            reasons.append("network_pipeline_cost")
        nbytes = pre[b] - pre[a] + (embed_bytes if s == 0 else 0) + (head_bytes if s == S - 1 else 0)
        u = load(s, a, b)
        if u > 1.0:
            diags.append(f"stage {s} on {ns[s].id} needs {nbytes} bytes, above its budget ({u:.2f}x)")
        if aff in ("recurrent", "mixed") and not allow_state_transfer:
            diags.append(f"stage {s} holds recurrent state: pinned to {ns[s].id}")
        stages.append(StagePlan(s, ns[s].id, lay[0].index, lay[-1].index + 1, roles, nbytes, u, aff, mig, reasons))
    bnds = [Boundary(s, s + 1, stages[s].layer_end - 1) for s in range(S - 1)]
    if len(nodes) > len(layers):
        diags.append(f"{len(nodes) - len(layers)} node(s) left idle: fewer layers than nodes")
    return TopologyPlan(stages, bnds, max(st.utilisation for st in stages), diags)


def plan_decoder(cfg, nodes: list[NodeSpec], *, context_tokens: int = 0, dtype_bytes: int = 2,
                 kv_dtype_bytes: int = 2) -> TopologyPlan:
    """Plan a :class:`DecoderConfig` model: per-layer weight bytes and the KV
    bytes of ``context_tokens`` cached tokens (all sequences together)."""
    H, I = cfg.hidden_size, cfg.intermediate_size
    attn = H * (cfg.q_size + 2 * cfg.kv_size) + cfg.q_size * H
    mlp = (cfg.num_experts * 3 * H * cfg.moe_intermediate_size + H * cfg.num_experts) if cfg.is_moe else 3 * H * I
    per_layer = (attn + mlp + 2 * H) * dtype_bytes
    kv = 2 * cfg.kv_size * context_tokens * kv_dtype_bytes
    layers = [LayerSpec(i, per_layer, True, False, kv) for i in range(cfg.num_hidden_layers)]
    emb = cfg.vocab_size * H * dtype_bytes
    head = emb + H * dtype_bytes  # the last stage holds its own LM head (a copy when tied)
    return plan(layers, nodes, embed_bytes=emb, head_bytes=head)
