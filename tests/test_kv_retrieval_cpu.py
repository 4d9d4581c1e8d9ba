"""KV-block retrieval for long-context decode (CPU): block summaries, the
selection (sinks + recent window + top-k by query . summary, kept in block
order) and the equivalence of attention over the selection with full
attention when the context fits the budget or the mass sits in retrieved
blocks."""
import math

import torch

from rlx_models_b200.ops import reference as R
from rlx_models_b200.runtime.kv_retrieval import KVRetrieval


def _attend(q, kc, vc, table, ctx, scale):
    k = R.gather_paged(kc, table, ctx)
    v = R.gather_paged(vc, table, ctx)
    pos = torch.arange(ctx)
    return R.attention(q[None], k, v, pos[-1:], pos, scale)[0]


def test_selection_budget_order_and_ctx():
    g = torch.Generator().manual_seed(0)
    Hkv, G, D, nb = 2, 2, 16, 40
    kc = torch.randn(nb, Hkv, 16, D, generator=g).bfloat16()
    r = KVRetrieval(1, nb, Hkv, D, "cpu", topk_blocks=2, window_blocks=2, sink_blocks=1)
    r.update(0, kc, torch.arange(nb * 16))
    assert torch.allclose(r.summ[0].float(), kc.float().mean(2), atol=1e-2)
    table = torch.randperm(nb, generator=g)[:30].int()[None]
    ctx = torch.tensor([29 * 16 + 5])  # 30 blocks, the last one holding 5 tokens
    q = torch.zeros(1, Hkv * G, D)
    hot = [7, 12]  # make two old blocks score highest
    for w in hot:
        q += r.summ[0, table[0, w].long()].float().repeat_interleave(G, 0) * 3
    sel, sctx = r.select(0, q, table, ctx)
    expect = sorted([0] + hot + [28, 29])
    assert sel[0].tolist() == table[0, expect].tolist()
    assert int(sctx[0]) == 4 * 16 + 5
    # short context: the budget covers everything, selection is the identity
    short = torch.tensor([3 * 16 + 1])
    sel, sctx = r.select(0, q, table[:, :5], short)
    assert sel[0].tolist() == table[0, :5].tolist() and int(sctx[0]) == 3 * 16 + 1


def test_retrieved_attention_matches_full_when_mass_is_retrieved():
    g = torch.Generator().manual_seed(1)
    Hkv, G, D, nb = 2, 4, 32, 80
    kc = (0.1 * torch.randn(nb, Hkv, 16, D, generator=g)).bfloat16()
    vc = torch.randn(nb, Hkv, 16, D, generator=g).bfloat16()
    # query heads of a group look the same way (the regime where one block holds the attention mass)
    q = torch.randn(Hkv, 1, D, generator=g).expand(Hkv, G, D).reshape(Hkv * G, D) \
        + 0.05 * torch.randn(Hkv * G, D, generator=g)
    needle = 33  # one old block whose keys align with the query
    kc[needle] = (q.view(Hkv, G, D).mean(1)[:, None, :] * 8).bfloat16()  # holds nearly all the mass
    table = torch.arange(nb).int()[None]
    ctx = torch.tensor([nb * 16 - 3])
    r = KVRetrieval(1, nb, Hkv, D, "cpu", topk_blocks=4, window_blocks=4, sink_blocks=1)
    r.update(0, kc, torch.arange(nb * 16))
    sel, sctx = r.select(0, q[None], table, ctx)
    assert needle in sel[0].tolist()
    scale = 1 / math.sqrt(D)
    full = _attend(q, kc, vc, table[0], int(ctx[0]), scale)
    part = _attend(q, kc, vc, sel[0], int(sctx[0]), scale)
    assert ((part - full).norm() / full.norm()) < 0.05
