"""Self-supervised pretraining objectives and their baselines (differentiable
torch, any device): masked-position selection, InfoNCE over a candidate set,
masked MSE, candidate sampling, sinusoidal positions, k-means targets and the
best-constant-predictor floors.

Reference: rlx-models-core src/pretrain.rs (``selection_matrix`` :137,
``l2_normalize`` :165, ``infonce_loss`` :183-255, ``masked_mse_loss`` :259,
``infonce_candidates`` :278, ``add_sinusoidal_positions`` :314,
``kmeans_labels`` / ``kmeans_centroids`` :1126-1235,
``prior_predictor_ce`` / ``constant_predictor_mse`` / ``constant_predictor_mae``
:1236-1300). There they are graph-building helpers of the reference's own
autodiff; here they are torch functions over tensors.
"""
from __future__ import annotations

import math

import torch


def selection_matrix(positions, n_pos: int, dtype=torch.float32) -> torch.Tensor:
    """[m, n_pos] one-hot rows: ``selection_matrix(p, n) @ x`` picks rows ``p`` of ``x``."""
    sel = torch.zeros(len(positions), n_pos, dtype=dtype)
    sel[torch.arange(len(positions)), torch.as_tensor(list(positions), dtype=torch.long)] = 1.0
    return sel


def select_rows(x: torch.Tensor, positions) -> torch.Tensor:
    """Rows ``positions`` of ``x`` viewed as [n_pos, width] (differentiable gather)."""
    flat = x.reshape(-1, x.shape[-1])
    return flat.index_select(0, torch.as_tensor(list(positions), dtype=torch.long, device=x.device))


def l2_normalize(x: torch.Tensor, dim: int = -1, floor: float = 1e-12) -> torch.Tensor:
    """x / (||x|| + floor): an all-zero row stays zero instead of dividing by 0."""
    return x / (x.norm(dim=dim, keepdim=True) + floor)


def infonce_loss(query: torch.Tensor, cands: torch.Tensor, temperature: float = 0.1) -> torch.Tensor:
    """Mean negative log-softmax of the positive among ``cands``.

    query [m, w]; cands [m, k1, w] with index 0 the positive and the rest
    distractors; similarity = cosine / temperature. Chance level is ln(k1)."""
    m, w = query.shape
    if cands.dim() != 3 or cands.shape[0] != m or cands.shape[2] != w:
        raise ValueError(f"infonce candidates must be [m, k1, width] = [{m}, k1, {w}], got {list(cands.shape)}")
    sim = (l2_normalize(cands, 2) * l2_normalize(query, 1)[:, None, :]).sum(-1) / temperature
    return -torch.log_softmax(sim, dim=1)[:, 0].mean()


def masked_mse_loss(pred: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """Mean squared error over every element of the masked rows."""
    if pred.shape != target.shape:
        raise ValueError(f"masked MSE shapes differ: {list(pred.shape)} vs {list(target.shape)}")
    return (pred - target).pow(2).mean()


def infonce_candidates(bank: torch.Tensor, positions, n_distractors: int, seed: int = 0) -> torch.Tensor:
    """[m, n_distractors + 1, w]: for each masked position p the bank row p
    first, then rows of *other* positions drawn uniformly (the answer never
    appears twice in the denominator)."""
    n_pos, w = bank.shape
    pos = torch.as_tensor(list(positions), dtype=torch.long)
    g = torch.Generator().manual_seed(seed)
    if n_pos > 1:
        # draw from the n_pos - 1 others: shift draws at or past p by one
        d = torch.randint(0, n_pos - 1, (len(pos), n_distractors), generator=g)
        d = d + (d >= pos[:, None]).long()
    else:
        d = torch.zeros(len(pos), n_distractors, dtype=torch.long)
    idx = torch.cat([pos[:, None], d], 1).to(bank.device)
    return bank[idx]


def add_sinusoidal_positions(x: torch.Tensor, seq: int, scale: float = 1.0) -> torch.Tensor:
    """x [n_pos, w] + scale * [sin(t f_i) | sin(t f_i + pi/2)], t = position % seq,
    f_i = 10000^(-2i / w) over the first and second halves of the width."""
    n_pos, w = x.shape
    half = max(1, w // 2)
    t = (torch.arange(n_pos, dtype=torch.float32) % max(1, seq))[:, None]
    d = torch.arange(w)
    i = torch.where(d < half, d, d - half).float()
    phase = torch.where(d < half, 0.0, math.pi / 2)
    freq = 1.0 / (10000.0 ** (2.0 * i / w))
    return x + scale * torch.sin(t * freq + phase).to(x.device, x.dtype)


def _kmeans(data: torch.Tensor, k: int, iters: int, seed: int):
    data = data.float()
    n = data.shape[0]
    if n == 0 or k == 0:
        return torch.empty(0, dtype=torch.long), torch.empty(0, data.shape[1])
    k = min(k, n)
    # farthest-point seeding: random seeding can leave a centre without members
    centres = [data[seed % n]]
    dmin = ((data - centres[0]) ** 2).sum(1)
    while len(centres) < k:
        i = int(torch.argmax(dmin))
        centres.append(data[i])
        dmin = torch.minimum(dmin, ((data - data[i]) ** 2).sum(1))
    c = torch.stack(centres)
    ids = torch.full((n,), -1, dtype=torch.long)
    for _ in range(max(1, iters)):
        new = torch.cdist(data, c).argmin(1)
        moved = not torch.equal(new, ids)
        ids = new
        counts = torch.bincount(ids, minlength=k)
        sums = torch.zeros_like(c).index_add_(0, ids, data)
        keep = counts == 0  # an emptied cluster keeps its centre
        c = torch.where(keep[:, None], c, sums / counts.clamp(min=1)[:, None])
        if not moved:
            break
    return ids, c


def kmeans_labels(data: torch.Tensor, k: int, iters: int = 20, seed: int = 0) -> torch.Tensor:
    """Cluster index of every row of ``data`` [n, w] (targets for a masked
    classification objective)."""
    return _kmeans(data, k, iters, seed)[0]


def kmeans_centroids(data: torch.Tensor, k: int, iters: int = 20, seed: int = 0) -> torch.Tensor:
    return _kmeans(data, k, iters, seed)[1]


def prior_predictor_ce(labels, num_classes: int) -> float:
    """Entropy H(p) of the label distribution: the cross-entropy of the best
    constant predictor (not -ln p_majority, whose cross-entropy is infinite)."""
    lab = torch.as_tensor(labels).reshape(-1)
    lab = lab[(lab >= 0) & (lab < num_classes)]
    if lab.numel() == 0:
        return float("nan")
    p = torch.bincount(lab, minlength=num_classes).double() / lab.numel()
    p = p[p > 0]
    return float(-(p * p.log()).sum())


def constant_predictor_mse(targets) -> float:
    """Variance: the MSE of predicting the mean."""
    t = torch.as_tensor(targets, dtype=torch.float64).reshape(-1)
    return float("nan") if t.numel() == 0 else float(((t - t.mean()) ** 2).mean())


def constant_predictor_mae(targets) -> float:
    """Mean absolute deviation from the median: the MAE of predicting the median."""
    t = torch.as_tensor(targets, dtype=torch.float64).reshape(-1)
    if t.numel() == 0:
        return float("nan")
    s = t.sort().values
    n = s.numel()
    med = s[n // 2] if n % 2 else 0.5 * (s[n // 2 - 1] + s[n // 2])
    return float((t - med).abs().mean())
