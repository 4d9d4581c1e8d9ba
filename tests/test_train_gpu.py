"""Training path on the GPU: our GEMM fwd/dgrad/wgrad, fused CE and AdamW
against the fp32 CPU path of the same trainer."""
import pytest
import torch

from rlx_models_b200 import config as C
from rlx_models_b200.train.trainer import TrainConfig, Trainer
from rlx_models_b200.weights.init import random_weights

pytestmark = pytest.mark.gpu


def test_gpu_training_matches_cpu_reference(cuda):
    cfg = C.tiny(num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=64, vocab_size=512, tie_word_embeddings=True)
    w = random_weights(cfg, 0)
    batch = torch.randint(0, cfg.vocab_size, (4, 129), generator=torch.Generator().manual_seed(0))
    tc = dict(lr=1e-3, micro_batch=2)
    gpu = Trainer(cfg, TrainConfig(**tc), w, device=cuda)
    cpu = Trainer(cfg, TrainConfig(**tc, param_dtype="float32"), w, device="cpu")
    lg = [gpu.step(batch).loss for _ in range(3)]
    lc = [cpu.step(batch).loss for _ in range(3)]
    for a, b in zip(lg, lc):
        assert abs(a - b) / b < 2e-2, (lg, lc)
    assert lg[-1] < lg[0]


def test_fused_ce_matches_torch(cuda):
    from rlx_models_b200.train.functional import lm_head_ce
    T, H, V = 300, 256, 1000
    x = (torch.randn(T, H) * 0.5).to(cuda, torch.bfloat16).requires_grad_(True)
    w = (torch.randn(V, H) * 0.05).to(cuda, torch.bfloat16).requires_grad_(True)
    t = torch.randint(0, V, (T,), device=cuda)
    t[5] = -100
    loss = lm_head_ce(x, w, t, chunk=128)
    loss.backward()
    xr, wr = x.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    lr = torch.nn.functional.cross_entropy(xr @ wr.T, t, ignore_index=-100)
    lr.backward()
    assert abs(loss.item() - lr.item()) < 1e-2
    assert ((x.grad.float() - xr.grad).norm() / xr.grad.norm()) < 2e-2
    assert ((w.grad.float() - wr.grad).norm() / wr.grad.norm()) < 2e-2


def test_lora_on_gpu_trains_adapters(cuda):
    from rlx_models_b200 import config as C
    from rlx_models_b200.train.trainer import TrainConfig, Trainer
    from rlx_models_b200.weights.init import random_weights
    cfg = C.tiny(num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=64, vocab_size=512)
    t = Trainer(cfg, TrainConfig(lr=2e-2, micro_batch=2, lora_rank=16, lora_alpha=32.0),
                random_weights(cfg, 0), device=cuda)
    base = [g.master.clone() for g in t.model.groups]
    b = torch.randint(0, 512, (4, 129), generator=torch.Generator().manual_seed(0))
    losses = [t.step(b).loss for _ in range(5)]
    assert losses[-1] < losses[0]
    assert all(torch.equal(g.master, m) for g, m in zip(t.model.groups, base))
