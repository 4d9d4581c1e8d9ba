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
