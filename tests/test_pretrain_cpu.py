"""Self-supervised objectives (train/pretrain.py): selection, InfoNCE chance level
and learnability, candidate sampling without the answer twice, sinusoidal
positions, k-means targets and the constant-predictor floors."""
import math

import pytest
import torch

from rlx_models_b200.train import pretrain as P


def test_selection_and_rows():
    assert P.selection_matrix([0, 2], 3).flatten().tolist() == [1, 0, 0, 0, 0, 1]
    x = torch.arange(12.0).view(4, 3)
    assert torch.equal(P.select_rows(x, [3, 1]), x[[3, 1]])
    assert torch.equal(P.selection_matrix([3, 1], 4) @ x, x[[3, 1]])


def test_infonce_chance_and_gradient():
    g = torch.Generator().manual_seed(0)
    q = torch.randn(64, 32, generator=g)
    cands = torch.randn(64, 8, 32, generator=g)
    loss = P.infonce_loss(q, cands, temperature=1e3)  # flat similarities -> chance
    assert abs(float(loss) - math.log(8)) < 1e-3
    cands[:, 0] = q * 5  # the positive is the query itself: loss near 0 at low temperature
    assert float(P.infonce_loss(q, cands, temperature=0.05)) < 1e-3
    qq = torch.randn(4, 16, requires_grad=True)
    P.infonce_loss(qq, torch.randn(4, 3, 16)).backward()
    assert qq.grad is not None and torch.isfinite(qq.grad).all()
    with pytest.raises(ValueError):
        P.infonce_loss(q, torch.randn(64, 32, 8))


def test_candidates_never_repeat_the_answer():
    bank = torch.arange(10.0)[:, None].repeat(1, 4)
    c = P.infonce_candidates(bank, [0, 5, 9], 50, seed=3)
    assert c.shape == (3, 51, 4)
    assert c[:, 0, 0].tolist() == [0, 5, 9]
    for row, p in zip(c, [0, 5, 9]):
        assert not (row[1:, 0] == p).any()


def test_masked_mse_and_positions():
    assert float(P.masked_mse_loss(torch.ones(2, 3), torch.zeros(2, 3))) == 1.0
    x = P.add_sinusoidal_positions(torch.zeros(6, 8), seq=3)
    assert torch.allclose(x[0], x[3]) and torch.allclose(x[0, 4:], torch.ones(4))  # cos(0) on the second half
    assert torch.allclose(x[:, 0], torch.sin(torch.tensor([0., 1., 2., 0., 1., 2.])))


def test_kmeans_and_floors():
    g = torch.Generator().manual_seed(1)
    blobs = torch.cat([torch.randn(50, 2, generator=g) * 0.1 + torch.tensor(c) for c in
                       ([0., 0.], [5., 0.], [0., 5.], [5., 5.])])
    ids = P.kmeans_labels(blobs, 4, 20, 7)
    assert len(set(ids.tolist())) == 4  # every cluster used
    for b in range(4):
        assert len(set(ids[b * 50:(b + 1) * 50].tolist())) == 1
    assert P.kmeans_centroids(blobs, 4).shape == (4, 2)
    assert abs(P.prior_predictor_ce([0, 0, 1, 1], 2) - math.log(2)) < 1e-9
    assert P.prior_predictor_ce([0, 0, 0, 3], 3) == 0.0  # out-of-range labels skipped
    assert abs(P.constant_predictor_mse([1.0, 3.0]) - 1.0) < 1e-9
    assert abs(P.constant_predictor_mae([1.0, 2.0, 10.0]) - 3.0) < 1e-9
