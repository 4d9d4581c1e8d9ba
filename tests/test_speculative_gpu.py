"""Speculative decoding on the GPU: output equals the target's greedy
continuation (draft = same model, draft = another model, prompt lookup)."""
import pytest
import torch

from rlx_models_b200 import config as C
from rlx_models_b200.registry import build_model
from rlx_models_b200.runtime.speculative import SpeculativeDecoder, _Seq

pytestmark = pytest.mark.gpu


def _greedy(model, prompt, n):
    s = _Seq(model, 512)
    lg = s.run(prompt, 0)
    out = [int(lg[-1].argmax())]
    while len(out) < n:
        lg = s.run([out[-1]], s.pos)
        out.append(int(lg[-1].argmax()))
    return out


def _agree(a, b):
    n = 0
    while n < min(len(a), len(b)) and a[n] == b[n]:
        n += 1
    return n


@pytest.mark.parametrize("mode", ["self", "other", "lookup"])
def test_speculative_matches_greedy(cuda, mode):
    cfg = C.tiny()
    target = build_model(cfg, device=cuda, seed=0)
    draft = {"self": target, "other": build_model(cfg, device=cuda, seed=7), "lookup": None}[mode]
    g = torch.Generator().manual_seed(3)
    base = torch.randint(0, cfg.vocab_size, (12,), generator=g).tolist()
    prompt = base * 3  # repetitive, so prompt lookup has matches
    ref = _greedy(target, prompt, 40)
    sd = SpeculativeDecoder(target, draft, k=4, max_len=512)
    out = sd.generate(prompt, 40)
    assert len(out) == 40
    # verification runs k+1-token chunks: allow a late near-tie divergence from single-token decode
    assert _agree(out, ref) >= 30, (out, ref)
    if mode == "self":
        assert sd.stats.acceptance > 0.8 and sd.stats.tokens_per_pass > 3


def test_speculative_with_learned_draft_head(cuda):
    """EAGLE-style draft head distilled on the target's own GPU features for
    this prompt's continuation: speculative output follows the target's greedy
    decode and the head's drafts are accepted."""
    from rlx_models_b200.models.decoder import ForwardBatch
    from rlx_models_b200.runtime.draft_head import DraftHead, train_draft_head
    from rlx_models_b200.weights.init import random_weights
    cfg = C.tiny(tie_word_embeddings=False)
    w = random_weights(cfg, 0)
    w["lm_head.weight"] = (w["lm_head.weight"].float() * 60).bfloat16()  # a confident target
    target = build_model(cfg, w, device=cuda)
    g = torch.Generator().manual_seed(5)
    prompt = torch.randint(0, cfg.vocab_size, (16,), generator=g).tolist()
    ref = _greedy(target, prompt, 48)

    def feats(ids):
        T = len(ids)
        nb = (T + 15) // 16
        fb = ForwardBatch(input_ids=torch.tensor(ids, dtype=torch.int32, device=cuda),
                          positions=torch.arange(T, dtype=torch.int32, device=cuda),
                          slots=torch.arange(T, dtype=torch.int64, device=cuda), num_decode=0,
                          pre_block_tables=torch.arange(nb, dtype=torch.int32, device=cuda).view(1, -1),
                          pre_ctx_lens=torch.tensor([T], dtype=torch.int32, device=cuda),
                          pre_cu_q=torch.tensor([0, T], dtype=torch.int32, device=cuda), pre_max_q=T)
        h = target.forward_hidden(fb, target.make_kv_cache(nb))
        return h.float(), target.logits(h).float()

    head = DraftHead(cfg.hidden_size, target.embed, target.lm_head, heads=4).to(cuda)
    losses = train_draft_head(head, feats, [prompt + ref], steps=400, lr=3e-3, window=48)
    assert losses[-1] < losses[0]
    sd = SpeculativeDecoder(target, draft_head=head, k=3, max_len=512)
    out = sd.generate(prompt, 48)
    assert _agree(out, ref) >= 36, (out, ref)
    assert sd.stats.acceptance > 0.3 and sd.stats.tokens_per_pass > 1.5, sd.stats
