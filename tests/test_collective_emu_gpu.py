"""Peer-memory collective kernels as one emulated rank on one GPU: every peer
table entry points at a local buffer and the flags are preset, so each kernel's
arithmetic (the reduction order, the fused residual add and RMSNorm, the packed
argmax keys, the expert-row combine) is checked against a plain fp32 PyTorch
reference without a second GPU."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rms(x, w, eps=1e-6):
    x = x.float()
    return (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()).bfloat16()


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda", 0)


@pytest.mark.parametrize("world", [2, 8])
def test_ar_pull_norm_emulated(dev, world):
    from rlx_models_b200 import ops
    from rlx_models_b200.parallel.collective_emu import build
    M, H = 24, 4096
    launch, _, b = build("pull", world, M, H, dev)
    h0 = b["h"].clone()
    launch()
    torch.cuda.synchronize(dev)
    ops.check_errors(dev)
    part = torch.stack([a[:M] for a in b["accs"]]).sum(0).bfloat16().float()
    h_ref = (h0.float() + part).bfloat16()
    assert (b["h"].float() - h_ref.float()).abs().max() <= 2e-2
    ref = _rms(h_ref, b["nw"])
    assert (b["out"].float() - ref.float()).abs().max() <= 3e-2
    assert float(b["zero"].abs().max()) == 0.0


def test_ar2_norm_emulated_own_rows(dev):
    """Rank 0 reduces rows [0, rpr); the rows owned by other ranks come from
    their result buffers, which nothing fills in this emulation."""
    from rlx_models_b200 import ops
    from rlx_models_b200.parallel.collective_emu import build
    M, H, world = 64, 4096, 4
    launch, _, b = build("pull2", world, M, H, dev)
    h0 = b["h"].clone()
    launch()
    torch.cuda.synchronize(dev)
    ops.check_errors(dev)
    r = b["rpr"]
    part = torch.stack([a[:r] for a in b["accs"]]).sum(0).bfloat16().float()
    h_ref = (h0[:r].float() + part).bfloat16()
    ref = _rms(h_ref, b["nw"])
    assert (b["out"][:r].float() - ref.float()).abs().max() <= 3e-2


@pytest.mark.parametrize("world", [2, 8])
def test_tp_argmax_emulated(dev, world):
    """Peers' key buffers hold zero keys, which every real value beats: the
    winner is this rank's shard argmax, offset by the shard start (0)."""
    from rlx_models_b200 import ops
    from rlx_models_b200.parallel.collective_emu import build
    launch, _, b = build("argmax", world, 48, 4096, dev)
    b["logits"][5, 17] = 1e4  # a known winner
    launch()
    torch.cuda.synchronize(dev)
    ops.check_errors(dev)
    ref = b["logits"].argmax(1).to(torch.int32)
    assert torch.equal(b["picked"], ref)
    assert int(b["picked"][5]) == 17


def test_ep_combine_norm_emulated(dev):
    from rlx_models_b200 import ops
    from rlx_models_b200.parallel.collective_emu import build
    T, H, world, k = 40, 2880, 8, 4
    launch, _, b = build("combine", world, T, H, dev, k=k)
    h0 = b["h"].clone()
    launch()
    torch.cuda.synchronize(dev)
    ops.check_errors(dev)
    ex = b["experts"].long().cpu()
    owner = ex // b["e_local"]
    moe = torch.zeros(T, H, device=dev)
    for t in range(T):
        for s in range(k):
            moe[t] += b["rows"][int(owner[t, s])][t * k + s].float()
    h_ref = (h0.float() + moe.bfloat16().float()).bfloat16()
    assert (b["h"].float() - h_ref.float()).abs().max() <= 2e-2
    ref = _rms(h_ref, b["nw"])
    assert (b["out"].float() - ref.float()).abs().max() <= 3e-2
