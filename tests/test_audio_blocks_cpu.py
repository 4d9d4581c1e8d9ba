"""Shared audio blocks on CPU: the codebook delay pattern against transformers'
MusicGen (mono and stereo, with and without a prompt), delay undo, flow-matching
integration against closed-form ODE solutions and the sway grid, and greedy
RNN-T / TDT decoding on scripted networks."""
import math

import pytest
import torch

from rlx_models_b200.models.audio_blocks import (apply_delay_pattern, build_delay_pattern, flow_sample,
                                                 sway_schedule, transducer_greedy, undo_delay_pattern)

transformers = pytest.importorskip("transformers")


def _musicgen(channels):
    dec = transformers.MusicgenDecoderConfig(vocab_size=32, hidden_size=16, num_hidden_layers=1,
                                             num_attention_heads=2, ffn_dim=32, num_codebooks=4 * channels,
                                             audio_channels=channels)
    return transformers.MusicgenForCausalLM(dec)


@pytest.mark.parametrize("channels", [1, 2])
@pytest.mark.parametrize("S,max_len", [(1, 12), (3, 12), (5, 9), (2, 5)])
def test_delay_pattern_matches_musicgen(channels, S, max_len):
    m = _musicgen(channels)
    K = 4 * channels
    g = torch.Generator().manual_seed(S + max_len)
    ids = torch.randint(0, 30, (2, K, S), generator=g)
    ref_ids, ref_mask = m.build_delay_pattern_mask(ids.reshape(2 * K, S), pad_token_id=31, max_length=max_len)
    got_ids, got_mask = build_delay_pattern(ids, 31, max_len, audio_channels=channels)
    assert torch.equal(got_mask, ref_mask) and torch.equal(got_ids, ref_ids)
    gen = torch.randint(0, 30, (2 * K, max_len), generator=g)
    assert torch.equal(apply_delay_pattern(gen, got_mask), m.apply_delay_pattern_mask(gen, ref_mask))


def test_undo_delay_pattern():
    frames = torch.arange(3 * 5).view(3, 5)
    delayed = torch.full((3, 7), -1)
    for k in range(3):
        delayed[k, k:k + 5] = frames[k]
    assert torch.equal(undo_delay_pattern(delayed), frames)


def test_flow_sample_exact_for_linear_paths():
    # rectified flow between x0 and x1: v = x1 - x0 is constant, so any grid is exact
    x0, x1 = torch.randn(4, 3), torch.randn(4, 3)
    out = flow_sample(lambda x, t: x1 - x0, x0, sway_schedule(7, -1.0))
    torch.testing.assert_close(out, x1)
    # dx/dt = x from 1 at t=0: midpoint converges to e faster than Euler
    ts = torch.linspace(0, 1, 65)
    eu = flow_sample(lambda x, t: x, torch.ones(1), ts, "euler")
    mid = flow_sample(lambda x, t: x, torch.ones(1), ts, "midpoint")
    assert abs(float(mid) - math.e) < abs(float(eu) - math.e) and abs(float(mid) - math.e) < 5e-4


def test_sway_schedule_endpoints():
    t = sway_schedule(16, -1.0)
    assert float(t[0]) == 0.0 and abs(float(t[-1]) - 1.0) < 1e-6 and bool((t[1:] >= t[:-1]).all())
    assert torch.allclose(sway_schedule(8, None), torch.linspace(0, 1, 9))


def _scripted(script, vocab=6):
    """A joint that emits script[(frame, n)] where n counts tokens on that frame."""
    state = {"n": 0, "t": None}

    def pred(tok, st):
        return (tok, st)

    def joint(f, g):
        t = int(f[0])
        if state["t"] != t:
            state["t"], state["n"] = t, 0
        tok, dur = script.get((t, state["n"]), (0, 1))
        state["n"] += 1
        lg = torch.full((vocab,), -5.0)
        lg[tok] = 5.0
        dl = torch.full((4,), -5.0)
        dl[dur] = 5.0
        return lg, dl

    return pred, joint


def test_tdt_greedy_durations():
    enc = torch.arange(8.0)[:, None]
    # frame 0: token 3 with duration 0 (stay), then token 4 with duration 2 -> frame 2;
    # frame 2: blank duration 0 (must still advance) -> 3; frame 3: token 5 duration 3 -> 6; then blanks
    script = {(0, 0): (3, 0), (0, 1): (4, 2), (2, 0): (0, 0), (3, 0): (5, 3)}
    pred, joint = _scripted(script)
    out = transducer_greedy(enc, pred, joint, blank=0, durations=[0, 1, 2, 3])
    assert out == [3, 4, 5]


def test_rnnt_greedy_max_symbols():
    enc = torch.arange(3.0)[:, None]

    def pred(tok, st):
        return tok, st

    def joint(f, g):          # always emits token 2: capped at max_symbols per frame
        lg = torch.zeros(4)
        lg[2] = 1.0
        return lg

    assert transducer_greedy(enc, pred, joint, blank=0, max_symbols=2) == [2] * 6
