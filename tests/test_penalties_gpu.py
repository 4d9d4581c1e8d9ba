"""Sampling penalties and logit bias on the GPU (csrc/sampling/sampling.cu
penalties_kernel) against a plain PyTorch fp32 reference, and through the
engine (penalised rows take the eager path)."""
import pytest
import torch

from rlx_models_b200 import ops

pytestmark = pytest.mark.gpu


def reference(x, rows):
    x = x.clone()
    for r, row in enumerate(rows):
        if row is None:
            continue
        counts, rep, freq, pres, bias = row
        for t, n in counts.items():
            v = x[r, t]
            if rep != 1.0:
                v = v / rep if v > 0 else v * rep
            if n > 0:
                v = v - freq * n - pres
            x[r, t] = v
        for t, b in (bias or {}).items():
            x[r, t] += b
    return x


def test_penalties_kernel(cuda):
    g = torch.Generator().manual_seed(0)
    V = 1000
    x = torch.randn(4, V, generator=g) * 3
    rows = [({5: 2, 7: 0, 999: 1}, 1.3, 0.5, 0.25, {1: 4.0, 5: -1.0}), None,
            ({0: 3}, 1.0, 1.0, 0.0, None), ({v: 1 for v in range(0, V, 3)}, 0.8, 0.0, 0.7, {2: -100.0})]
    got = ops.apply_penalties(x.to(cuda), rows).cpu()
    ref = reference(x, rows)
    assert torch.allclose(got, ref, rtol=1e-6, atol=1e-6)
    assert torch.equal(got[1], x[1])


def test_engine_penalties(cuda):
    from rlx_models_b200 import config as C
    from rlx_models_b200.models.decoder import DecoderLM
    from rlx_models_b200.runtime.engine import EngineConfig, LLMEngine, SamplingParams
    from rlx_models_b200.weights.init import random_weights
    cfg = C.tiny(num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=64, vocab_size=512)
    m = DecoderLM(cfg, random_weights(cfg, 0), device=cuda)
    eng = LLMEngine(m, EngineConfig(max_num_seqs=8, max_model_len=256, num_blocks=64))
    prompt = list(range(10, 30))
    no_rep = eng.generate([prompt], SamplingParams(max_new_tokens=40, ignore_eos=True,
                                                   frequency_penalty=1e4))[0].token_ids
    assert len(set(no_rep)) == len(no_rep)  # a huge frequency penalty never repeats a token
    forced = eng.generate([prompt], SamplingParams(max_new_tokens=5, ignore_eos=True,
                                                   logit_bias={123: 1e4}))[0].token_ids
    assert forced == [123] * 5
    mixed = eng.generate([prompt, prompt], [SamplingParams(max_new_tokens=40, ignore_eos=True),
                                            SamplingParams(max_new_tokens=5, ignore_eos=True,
                                                           logit_bias={7: 1e4})])
    # the unpenalised row of a penalised step is untouched (its batch shape differs from a solo run,
    # so only its length and the forced row are compared)
    assert len(mixed[0].token_ids) == 40
    assert mixed[1].token_ids == [7] * 5
    rep = eng.generate([prompt], SamplingParams(max_new_tokens=20, ignore_eos=True,
                                                repetition_penalty=1e6))[0].token_ids
    assert not (set(rep) & set(prompt))  # prompt tokens pushed below every unseen token
    ops.check_errors(cuda)


def test_engine_logit_processors(cuda):
    from rlx_models_b200 import config as C
    from rlx_models_b200.models.decoder import DecoderLM
    from rlx_models_b200.runtime.engine import EngineConfig, LLMEngine, SamplingParams
    from rlx_models_b200.weights.init import random_weights
    cfg = C.tiny(num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=64, vocab_size=512)
    m = DecoderLM(cfg, random_weights(cfg, 0), device=cuda)
    eng = LLMEngine(m, EngineConfig(max_num_seqs=8, max_model_len=256, num_blocks=64))
    prompt = list(range(40, 60))
    sp = dict(max_new_tokens=48, ignore_eos=True)
    dry = eng.generate([prompt], SamplingParams(**sp, dry_multiplier=1e3, dry_allowed_length=2))[0].token_ids
    seq = prompt + dry
    trigrams = [tuple(seq[i:i + 3]) for i in range(len(prompt) - 2, len(seq) - 2)]
    assert len(set(trigrams)) == len(trigrams)  # no repeated 3-gram is ever extended
    typ = eng.generate([prompt], SamplingParams(**sp, temperature=1.0, typical_p=0.2, seed=1))[0].token_ids
    miro = eng.generate([prompt], SamplingParams(**sp, temperature=1.0, mirostat=2, mirostat_tau=3.0,
                                                 seed=2))[0].token_ids
    xtc = eng.generate([prompt], SamplingParams(**sp, temperature=1.0, xtc_probability=1.0, xtc_threshold=0.0,
                                                seed=3))[0].token_ids
    assert len(typ) == len(miro) == len(xtc) == 48
    ops.check_errors(cuda)
