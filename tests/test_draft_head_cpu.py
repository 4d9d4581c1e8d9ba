"""Learned draft head (EAGLE-style) on CPU: self-distillation on the fp32
oracle's features. The target is random, so there is no structure to
generalise to unseen text; the test checks that the pipeline (feature /
token alignment, KL to the target's next position, greedy recurrence) fits
the target on the sequences it was distilled on."""
import torch

from rlx_models_b200 import config as C
from rlx_models_b200.models.oracle import DecoderOracle
from rlx_models_b200.runtime.draft_head import DraftHead, train_draft_head
from rlx_models_b200.weights.init import random_weights


def test_draft_head_distills_the_target():
    cfg = C.tiny(num_hidden_layers=2, hidden_size=64, intermediate_size=128, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=16, vocab_size=64, tie_word_embeddings=False)
    w = {k: v.float() for k, v in random_weights(cfg, 0).items()}
    for k in w:
        if k.endswith("proj.weight"):
            w[k] = w[k] * 8
    w["lm_head.weight"] = w["lm_head.weight"] * 150  # a confident target, as trained LMs are
    oracle = DecoderOracle(cfg, w)

    def target(ids):
        h, _ = oracle.forward_hidden(torch.tensor(ids))
        return h, h @ w["lm_head.weight"].T

    g = torch.Generator().manual_seed(0)
    seqs = []
    for _ in range(8):  # the target's own greedy continuations of random prompts
        ids = torch.randint(0, 64, (8,), generator=g).tolist()
        toks, _ = oracle.generate(torch.tensor(ids), 56)
        seqs.append(ids + toks)
    head = DraftHead(64, w["model.embed_tokens.weight"], w["lm_head.weight"], heads=4)
    losses = train_draft_head(head, target, seqs, steps=500, lr=3e-3, window=48)
    assert sum(losses[-20:]) / 20 < 0.2 * sum(losses[:20]) / 20
    agree = total = 0
    for seq in seqs[:4]:
        h, _ = target(seq)
        for p in range(10, len(seq) - 2):
            d = head.propose(h[p - 7:p + 1], seq[p - 6:p + 2], 1)[0]
            agree += int(d == seq[p + 2])
            total += 1
    assert agree / total > 0.6, agree / total
    assert len(head.propose(h[:8], seq[1:9], 4)) == 4
