"""Training host logic on CPU: FSDP (gloo, 2 ranks) == single process, LR
schedules, sharded checkpoint resume across world sizes, HF export."""
import os
import tempfile

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rlx_models_b200 import config as C
from rlx_models_b200.train.trainer import TrainConfig, Trainer
from rlx_models_b200.weights.init import random_weights


def _cfg():
    return C.tiny(num_hidden_layers=2, hidden_size=64, intermediate_size=128, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=16, vocab_size=96, tie_word_embeddings=True)


def _batch(seed=0, B=4, S=12, V=96):
    return torch.randint(0, V, (B, S + 1), generator=torch.Generator().manual_seed(seed))


def _single(steps=2, ckpt=False):
    cfg = _cfg()
    t = Trainer(cfg, TrainConfig(lr=1e-2, micro_batch=2, activation_checkpointing=ckpt, param_dtype="float32"), random_weights(cfg, 0),
                device="cpu")
    losses = [t.step(_batch(s)).loss for s in range(steps)]
    return losses, t.model.hf_state_dict(), t


def _worker(rank, world, port, out_dir, steps):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = _cfg()
    t = Trainer(cfg, TrainConfig(lr=1e-2, micro_batch=1, activation_checkpointing=True, param_dtype="float32"), random_weights(cfg, 0),
                rank=rank, world=world, device="cpu")
    losses = []
    for s in range(steps):
        b = _batch(s)
        per = b.shape[0] // world
        losses.append(t.step(b[rank * per:(rank + 1) * per]).loss)
    sd = t.model.hf_state_dict()
    t.save_checkpoint(os.path.join(out_dir, "ckpt"))
    if rank == 0:
        torch.save({"losses": losses, "sd": sd}, os.path.join(out_dir, "res.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_fsdp_two_ranks_matches_single_process():
    steps = 2
    ref_losses, ref_sd, _ = _single(steps)
    with tempfile.TemporaryDirectory() as d:
        port = 29600 + os.getpid() % 300
        mp.spawn(_worker, args=(2, port, d, steps), nprocs=2, join=True)
        res = torch.load(os.path.join(d, "res.pt"))
        for a, b in zip(res["losses"], ref_losses):
            assert abs(a - b) < 1e-4 * max(1.0, abs(b))
        for k, v in ref_sd.items():
            assert torch.allclose(res["sd"][k], v, atol=2e-5, rtol=1e-4), k
        # resume the 2-rank checkpoint in one process: identical state
        cfg = _cfg()
        t1 = Trainer(cfg, TrainConfig(lr=1e-2, param_dtype="float32"), random_weights(cfg, 7), device="cpu")
        t1.load_checkpoint(os.path.join(d, "ckpt"))
        assert t1.step_num == steps
        sd1 = t1.model.hf_state_dict()
        for k, v in ref_sd.items():
            assert torch.allclose(sd1[k], v, atol=2e-5, rtol=1e-4), k


def test_loss_decreases_and_ckpt_equivalence():
    losses, _, _ = _single(steps=1)
    cfg = _cfg()
    t = Trainer(cfg, TrainConfig(lr=3e-3), random_weights(cfg, 0), device="cpu")
    b = _batch(3)
    l0 = [t.step(b).loss for _ in range(6)]
    assert l0[-1] < l0[0]
    # activation checkpointing does not change the math
    a, _, _ = _single(steps=2, ckpt=False)
    c, _, _ = _single(steps=2, ckpt=True)
    assert all(abs(x - y) < 1e-5 for x, y in zip(a, c))


def test_lr_schedules():
    c = TrainConfig(lr=1.0, schedule="cosine", warmup_steps=2, total_steps=12, min_lr_ratio=0.0)
    assert c.lr_at(0) == 0.5 and c.lr_at(1) == 1.0
    assert abs(c.lr_at(7) - 0.5) < 1e-9 and c.lr_at(12) < 1e-9
    l = TrainConfig(lr=1.0, schedule="linear", total_steps=10, min_lr_ratio=0.0)
    assert abs(l.lr_at(5) - 0.5) < 1e-9


def test_hf_export_roundtrip(tmp_path):
    from rlx_models_b200.weights.weight_map import WeightMap
    _, sd, t = _single(steps=1)
    t.export_hf(str(tmp_path))
    wm = WeightMap.from_dir(str(tmp_path))
    assert set(wm.keys()) == set(sd)
    assert torch.allclose(wm.peek("model.layers.1.mlp.up_proj.weight").float(),
                          sd["model.layers.1.mlp.up_proj.weight"].bfloat16().float())


def test_newton_schulz_orthogonalizes():
    from rlx_models_b200.train.muon import newton_schulz5
    g = torch.randn(48, 96, generator=torch.Generator().manual_seed(0))
    o = newton_schulz5(g)
    sv = torch.linalg.svdvals(o)
    assert sv.min() > 0.5 and sv.max() < 1.3  # singular values pushed toward 1 (the method's band)
    # same left / right singular vectors as G: O is close to U V^T
    u, _, vh = torch.linalg.svd(g, full_matrices=False)
    assert ((o - u @ vh).norm() / (u @ vh).norm()) < 0.35


def _muon_worker(rank, world, port, out_dir, steps):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = _cfg()
    t = Trainer(cfg, TrainConfig(lr=1e-2, micro_batch=1, param_dtype="float32", optimizer="muon"),
                random_weights(cfg, 0), rank=rank, world=world, device="cpu")
    losses = []
    for s in range(steps):
        b = _batch(s)
        per = b.shape[0] // world
        losses.append(t.step(b[rank * per:(rank + 1) * per]).loss)
    sd = t.model.hf_state_dict()
    if rank == 0:
        torch.save({"losses": losses, "sd": sd}, os.path.join(out_dir, "res.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_muon_sharded_matches_single_process_and_learns():
    cfg = _cfg()
    t = Trainer(cfg, TrainConfig(lr=1e-2, micro_batch=2, param_dtype="float32", optimizer="muon"),
                random_weights(cfg, 0), device="cpu")
    losses = [t.step(_batch(s)).loss for s in range(3)]
    ref_sd = t.model.hf_state_dict()
    t2 = Trainer(cfg, TrainConfig(lr=1e-2, micro_batch=2, param_dtype="float32", optimizer="muon"),
                 random_weights(cfg, 0), device="cpu")
    fixed = _batch(5)
    l0 = t2.step(fixed).loss
    for _ in range(6):
        l1 = t2.step(fixed).loss
    assert l1 < l0  # overfits one batch
    with tempfile.TemporaryDirectory() as d:
        port = 29650 + os.getpid() % 300
        mp.spawn(_muon_worker, args=(2, port, d, 3), nprocs=2, join=True)
        res = torch.load(os.path.join(d, "res.pt"))
        for a, b in zip(res["losses"], losses):
            assert abs(a - b) < 1e-4 * max(1.0, abs(b))
        for k, v in ref_sd.items():
            assert torch.allclose(res["sd"][k], v, atol=5e-5, rtol=1e-4), k
