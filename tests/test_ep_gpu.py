"""Expert-parallel combine kernel (parallel/ep.py, csrc/comm/ep_combine.cu).

The multi-rank kernel is checked on one GPU by emulating W ranks inside ONE
launch: every rank's rows / inverse-permutation slots are local buffers in the
peer tables, and the other ranks' barrier flags are set beforehand, so no
kernel ever waits on another launch. The cross-GPU run is
parallel/ep_check.py (tests/test_multigpu.py)."""
import pytest
import torch

from rlx_models_b200 import config as C
from rlx_models_b200 import ops
from rlx_models_b200.ops import ext, scratch
from rlx_models_b200.weights.init import random_weights

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,E,k,W,H", [(1, 8, 2, 2, 256), (37, 16, 4, 4, 2880), (128, 32, 4, 8, 2880),
                                       (5, 8, 4, 1, 4096)])
def test_ep_combine_emulated_ranks(cuda, T, E, k, W, H):
    g = torch.Generator().manual_seed(T + E)
    e_local = E // W
    logits = torch.randn(T, E, generator=g).to(cuda)
    experts = logits.topk(k, -1).indices.int().contiguous()
    n = T * k
    R = (torch.randn(n, H, generator=g) * 0.5).to(cuda, torch.bfloat16)  # row of assignment t*k+s
    rows, invs = [], []
    for q in range(W):
        meta = torch.empty(2 * e_local + 2, dtype=torch.int32, device=cuda)
        tiles = torch.empty(4 * (n // 32 + e_local + 1), dtype=torch.int32, device=cuda)
        perm = torch.empty(n, dtype=torch.int32, device=cuda)
        inv = torch.empty(n, dtype=torch.int32, device=cuda)
        cur = torch.empty(e_local, dtype=torch.int32, device=cuda)
        ext().moe_align(experts, e_local, q * e_local, e_local, 32, meta, tiles, perm, inv, cur)
        cnt = int(meta[1:e_local + 1].sum())
        rq = torch.zeros(n, H, dtype=torch.bfloat16, device=cuda)
        rq[:cnt] = R[perm[:cnt].long()]
        rows.append(rq)
        invs.append(inv)
    h = (torch.randn(T, H, generator=g)).to(cuda, torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(H, generator=g)).to(cuda, torch.bfloat16)
    flags = torch.ones(W, dtype=torch.int32, device=cuda)
    flags[0] = 0
    tab = lambda ts: torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=cuda)  # noqa: E731
    peer_flags = tab([flags] * W)
    ctr = torch.zeros(2, dtype=torch.int32, device=cuda)
    st = scratch(cuda).status
    h_fused = h.clone()
    out = torch.empty_like(h)
    ext().ep_combine_norm(tab(rows), tab(invs), peer_flags, flags, experts, e_local, h_fused, nw, out,
                          ctr[0:1], ctr[1:2], 0, W, 1e-6, st)
    torch.cuda.synchronize()
    assert int(st[0]) == 0
    assert int(ctr[0]) == 1 and int(ctr[1]) == 0 and int(flags[0]) == 1
    # existing kernels on the single-GPU arrangement: combine, then add + rmsnorm
    inv_all = torch.arange(n, dtype=torch.int32, device=cuda)
    moe = torch.empty(T, H, dtype=torch.bfloat16, device=cuda)
    ext().moe_combine(R, inv_all, k, moe, False)
    h_ref = h.clone()
    ref = ops.rmsnorm(moe, nw, 1e-6, residual=h_ref, residual_out=h_ref)
    torch.cuda.synchronize()
    assert torch.equal(h_fused, h_ref)
    assert torch.equal(out, ref)
    # and against plain fp32 PyTorch
    m32 = R.float().view(T, k, H).sum(1)
    h32 = h.float() + m32
    o32 = h32 * torch.rsqrt(h32.pow(2).mean(-1, keepdim=True) + 1e-6) * nw.float()
    assert ((out.float() - o32).norm() / o32.norm()).item() < 1e-2


@pytest.mark.parametrize("family", ["gpt_oss", "qwen3_moe"])
def test_moe_fused_combine_matches_unfused(cuda, family):
    """The single-GPU MoE block through ep_combine_norm (combine + add + norm in
    one kernel) gives the same logits, bit for bit, as combine -> rmsnorm."""
    from rlx_models_b200.models.decoder import ForwardBatch
    from rlx_models_b200.models.moe import MoEDecoderLM
    kw = dict(hidden_size=256, num_attention_heads=4, num_key_value_heads=2, head_dim=64, num_experts=8,
              num_experts_per_tok=2, moe_intermediate_size=256, intermediate_size=256, vocab_size=512)
    if family == "gpt_oss":
        kw["sliding_window"] = 16
    cfg = C.tiny(family, **kw)
    w = random_weights(cfg, seed=7, dtype=torch.bfloat16)
    fused = MoEDecoderLM(cfg, w, device=cuda, ep_combine="fused")
    plain = MoEDecoderLM(cfg, w, device=cuda, ep_combine="nccl")
    assert fused.combiner is not None and plain.combiner is None
    T = 29
    ids = torch.randint(0, cfg.vocab_size, (T,), generator=torch.Generator().manual_seed(3))
    nb = (T + 15) // 16

    def fb():
        return ForwardBatch(input_ids=ids.int().to(cuda), positions=torch.arange(T, dtype=torch.int32, device=cuda),
                            slots=torch.arange(T, dtype=torch.int64, device=cuda), num_decode=0,
                            pre_block_tables=torch.arange(nb, dtype=torch.int32, device=cuda).view(1, -1),
                            pre_ctx_lens=torch.tensor([T], dtype=torch.int32, device=cuda),
                            pre_cu_q=torch.tensor([0, T], dtype=torch.int32, device=cuda), pre_max_q=T)

    a = fused.forward(fb(), fused.make_kv_cache(nb))
    b = plain.forward(fb(), plain.make_kv_cache(nb))
    torch.cuda.synchronize()
    ops.check_errors(cuda)
    assert torch.equal(a, b)
