"""Blocks shared by the speech / music families: the codebook delay pattern of
multi-codebook codec language models, flow-matching ODE sampling, and greedy
transducer (RNN-T / TDT) decoding.

delay pattern (MusicGen / Parler-TTS / Dia-style codec LMs): codebook k of a
    frame is predicted k steps after codebook 0, so the LM sees one token per
    codebook per step without conditioning codebook k on later codebooks of the
    same frame. ``build_delay_pattern`` lays the prompt out that way and returns
    the mask of positions left to predict (-1) and fixed pad positions;
    ``apply_delay_pattern`` keeps the fixed entries of a generated sequence;
    ``undo_delay_pattern`` realigns a delayed [K, T] sequence to frames.

flow matching (F5-TTS, Stable Audio, FLUX-style samplers): Euler / midpoint
    integration of dx/dt = v(x, t) from noise at t = 0 to data at t = 1 over a
    time grid; ``sway_schedule`` is the F5-TTS sway sampling grid
    t' = t + s (cos(pi t / 2) - 1 + t).

transducers (Parakeet-TDT / RNN-T ASR): greedy decoding over encoder frames
    with a prediction network (``pred(token, state) -> (g, state)``) and a joint
    network (``joint(f, g) -> (token logits, duration logits)``). A non-blank
    token updates the prediction network; TDT models advance by the predicted
    duration (a blank with duration 0 still advances one frame), RNN-T models
    (no duration head) advance one frame on blank and stay on the frame after
    a token, up to ``max_symbols`` tokens per frame.

Reference: the reference's shared audio blocks (crates/rlx-audio-blocks: TDT /
transducer decoders, flow schedulers, codec delay patterns).
"""
from __future__ import annotations

import math
from typing import Callable

import torch


# ---------------------------------------------------------------------------
# codebook delay pattern
# ---------------------------------------------------------------------------

def build_delay_pattern(ids: torch.Tensor, pad_id: int, max_length: int, audio_channels: int = 1):
    """ids [B, K, S] (prompt codes, the start token included) -> (ids with the
    pattern applied [B * K, S'], pattern mask [B * K, max_length]: -1 where a
    token is still to be predicted, otherwise the fixed value).

    Codebook k (per channel, channels interleaved for stereo) is shifted right
    by k; positions before the shift and the last K - 1 - k positions are the
    pad id. Sequences shorter than 2K - 1 get no pattern (all -1)."""
    B, K, S = ids.shape
    shifted = torch.full((B, K, max_length), -1, dtype=torch.long, device=ids.device)
    ch = K // 2 if audio_channels == 2 else K
    if max_length < 2 * ch - 1:
        return ids.reshape(B * K, -1), shifted.reshape(B * K, -1)
    for k in range(ch):
        rows = [2 * k, 2 * k + 1] if audio_channels == 2 else [k]
        for r in rows:
            shifted[:, r, k:S + k] = ids[:, r]
    t = torch.arange(max_length)
    kk = torch.arange(ch)[:, None]
    fixed = (t[None, :] <= kk) | (t[None, :] >= max_length - ch + 1 + kk)     # BOS / EOS pad triangles
    if audio_channels == 2:
        fixed = fixed.repeat_interleave(2, 0)
    fixed = fixed.to(ids.device)
    pattern = torch.where(fixed[None], torch.full_like(shifted, pad_id), shifted)
    # the prompt part: up to the first position still to predict
    todo = pattern[:, 0] == -1                     # codebook 0 has no offset: it starts first
    has = todo.any(-1)
    start = int(todo.int().argmax(-1)[has].min()) if bool(has.any()) else S
    return pattern[..., :start].reshape(B * K, -1), pattern.reshape(B * K, -1)


def apply_delay_pattern(ids: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    """Keep predictions where the mask is -1 and the mask's fixed value elsewhere."""
    m = mask[..., :ids.shape[-1]]
    return torch.where(m == -1, ids, m)


def undo_delay_pattern(codes: torch.Tensor, delays: list[int] | None = None) -> torch.Tensor:
    """Delayed codes [K, T] (codebook k shifted right by delays[k], default k)
    -> aligned frames [K, T - max(delays)]."""
    K, T = codes.shape
    delays = list(range(K)) if delays is None else list(delays)
    n = T - max(delays)
    return torch.stack([codes[k, delays[k]:delays[k] + n] for k in range(K)])


# ---------------------------------------------------------------------------
# flow matching
# ---------------------------------------------------------------------------

def sway_schedule(steps: int, sway: float | None = -1.0) -> torch.Tensor:
    """Time grid [steps + 1] on [0, 1]; with ``sway`` the F5-TTS sway sampling
    t' = t + s (cos(pi t / 2) - 1 + t) (s < 0 puts more steps early)."""
    t = torch.linspace(0, 1, steps + 1)
    if sway is not None:
        t = t + sway * (torch.cos(math.pi / 2 * t) - 1 + t)
    return t


@torch.no_grad()
def flow_sample(velocity: Callable[[torch.Tensor, float], torch.Tensor], x0: torch.Tensor, ts: torch.Tensor,
                method: str = "euler") -> torch.Tensor:
    """Integrate dx/dt = velocity(x, t) over the grid ``ts`` from x0 (Euler, or
    the explicit midpoint rule)."""
    x = x0
    for i in range(len(ts) - 1):
        t, dt = float(ts[i]), float(ts[i + 1] - ts[i])
        if method == "euler":
            x = x + dt * velocity(x, t)
        elif method == "midpoint":
            xm = x + 0.5 * dt * velocity(x, t)
            x = x + dt * velocity(xm, t + 0.5 * dt)
        else:
            raise ValueError(f"method {method!r}: euler or midpoint")
    return x


# ---------------------------------------------------------------------------
# transducers
# ---------------------------------------------------------------------------

@torch.no_grad()
def transducer_greedy(enc: torch.Tensor, pred: Callable, joint: Callable, blank: int, state=None,
                      durations: list[int] | None = None, max_symbols: int = 10, start_token: int | None = None
                      ) -> list[int]:
    """Greedy RNN-T / TDT decoding of one utterance.

    enc [T, D] encoder frames; pred(token or None, state) -> (g, new state)
    (``None``: the start of the sequence); joint(f [D], g) -> token logits, or
    (token logits, duration logits) for TDT with ``durations`` the duration of
    each duration class. Returns the emitted token ids."""
    T = enc.shape[0]
    g, st = pred(start_token, state)
    out: list[int] = []
    t, emitted = 0, 0
    while t < T:
        res = joint(enc[t], g)
        if durations is not None:
            tok_logits, dur_logits = res
            d = durations[int(dur_logits.argmax())]
        else:
            tok_logits, d = res, None
        k = int(tok_logits.argmax())
        if k != blank:
            out.append(k)
            g, st = pred(k, st)
            emitted += 1
        if durations is not None:
            step = d if d > 0 else (1 if k == blank else 0)
            if step == 0 and emitted >= max_symbols:
                step = 1
        else:
            step = 1 if (k == blank or emitted >= max_symbols) else 0
        if step > 0:
            emitted = 0
        t += step
    return out
