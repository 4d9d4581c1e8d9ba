"""FSDP gradient reduce-scatter by push (csrc/comm/fsdp_comm.cu, the GEMM's
shard-push epilogue, train/fsdp.py GradPush).

Multi-rank addressing is checked on one GPU with W emulated ranks: the peer
table points at W local shard buffers, so one launch adds into all of them and
nothing waits on another launch. The cross-GPU run is train/fsdp_check.py
(tests/test_multigpu.py)."""
import pytest
import torch

from rlx_models_b200 import config as C
from rlx_models_b200.ops import check_errors, ext, scratch
from rlx_models_b200.train.trainer import TrainConfig, Trainer
from rlx_models_b200.weights.init import random_weights

pytestmark = pytest.mark.gpu


def _shards(W, shard_n, dev):
    bufs = [torch.zeros(shard_n, dtype=torch.float32, device=dev) for _ in range(W)]
    table = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=dev)
    return bufs, table


@pytest.mark.parametrize("M,N,K,base,W,shard_n", [(256, 384, 512, 0, 3, 33024), (200, 104, 192, 12, 4, 5248),
                                                  (1024, 2048, 4096, 4096, 2, 1050624), (128, 40, 64, 5, 2, 2688)])
def test_gemm_push_shards_emulated(cuda, M, N, K, base, W, shard_n):
    """dW = dY^T X pushed into W shards equals the dense GEMM; shard
    boundaries fall inside rows, ragged column tails and odd bases included."""
    assert base + M * N <= W * shard_n
    g = torch.Generator().manual_seed(M + N)
    dy = (torch.randn(K, M, generator=g) * 0.1).to(cuda, torch.bfloat16)  # [tokens, out]
    x = (torch.randn(K, N, generator=g) * 0.1).to(cuda, torch.bfloat16)   # [tokens, in]
    bufs, table = _shards(W, shard_n, cuda)
    s = scratch(cuda)
    for _ in range(2):  # pushes accumulate
        ext().gemm_push_shards(dy.t(), x, table, base, shard_n, 1.0, s.gemm_ws, s.gemm_sem, s.status)
    dense = torch.empty(M, N, dtype=torch.float32, device=cuda)
    ext().gemm(dy.t(), x, dense, False, 1.0, None, None, False, s.gemm_ws, s.gemm_sem, s.status)
    torch.cuda.synchronize()
    check_errors(cuda)
    flat = torch.cat(bufs)
    got = flat[base:base + M * N].view(M, N)
    assert torch.allclose(got, 2 * dense, rtol=1e-5, atol=1e-6)
    assert flat[:base].abs().sum() == 0 and flat[base + M * N:].abs().sum() == 0
    ref = 2 * (dy.float().t() @ x.float())
    assert ((got - ref).norm() / ref.norm()).item() < 1e-3


@pytest.mark.parametrize("dtype,n,base", [(torch.float32, 10000, 0), (torch.bfloat16, 777, 3),
                                          (torch.float32, 4096, 1020)])
def test_shard_push_add_emulated(cuda, dtype, n, base):
    W, shard_n = 3, 4096
    src = torch.randn(n, generator=torch.Generator().manual_seed(n)).to(cuda, dtype)
    bufs, table = _shards(W, shard_n, cuda)
    ext().shard_push_add(src, table, base, shard_n, 1.0)
    ext().shard_push_add(src, table, base, shard_n, 0.5)
    torch.cuda.synchronize()
    flat = torch.cat(bufs)
    assert torch.allclose(flat[base:base + n], 1.5 * src.float(), rtol=1e-6, atol=1e-6)
    assert flat[:base].abs().sum() == 0 and flat[base + n:].abs().sum() == 0


def test_peer_barrier_single_rank(cuda):
    flags = torch.zeros(1, dtype=torch.int32, device=cuda)
    table = torch.tensor([flags.data_ptr()], dtype=torch.int64, device=cuda)
    epoch = torch.zeros(1, dtype=torch.int32, device=cuda)
    for _ in range(3):
        ext().peer_barrier(table, flags, epoch, 0, 1, scratch(cuda).status)
    torch.cuda.synchronize()
    check_errors(cuda)
    assert int(epoch) == 3 and int(flags[0]) == 3


def test_trainer_push_matches_nccl_path(cuda):
    """World 1: pushing weight gradients from the wgrad GEMM (and the dense
    ones from the push kernel) gives the gradients of the materialise-then-
    reduce path. That path hands autograd a dW that is rounded to the weight's
    bf16 dtype; the push adds the GEMM's fp32 dW, so the two agree to bf16
    rounding, not bit for bit."""
    cfg = C.tiny(num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=64, vocab_size=512, tie_word_embeddings=True)
    w = random_weights(cfg, 0)
    batch = torch.randint(0, cfg.vocab_size, (4, 129), generator=torch.Generator().manual_seed(0))
    a = Trainer(cfg, TrainConfig(lr=1e-3, micro_batch=2, grad_reduce="push"), w, device=cuda)
    b = Trainer(cfg, TrainConfig(lr=1e-3, micro_batch=2, grad_reduce="nccl"), w, device=cuda)
    assert a.push is not None and b.push is None
    ids, tgt = batch[:, :-1].to(cuda), batch[:, 1:].to(cuda)
    for t in (a, b):
        t.model.loss(ids, tgt).backward()
    a.push.barrier()
    torch.cuda.synchronize()
    check_errors(cuda)
    for ga, gb in zip(a.model.groups, b.model.groups):
        rel = ((ga.grad - gb.grad).norm() / gb.grad.norm()).item()
        assert rel < 5e-3, (ga.name, rel)
        ga.grad.zero_()
        gb.grad.zero_()
    la = [a.step(batch) for _ in range(3)]
    lb = [b.step(batch) for _ in range(3)]
    check_errors(cuda)
    for x, y in zip(la, lb):
        assert abs(x.loss - y.loss) < 2e-3 * abs(y.loss) and abs(x.grad_norm - y.grad_norm) < 1e-2 * y.grad_norm
    assert la[-1].loss < la[0].loss
    a.push.close()
