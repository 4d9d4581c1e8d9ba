"""LoRA / DoRA fine-tuning, JSONL datasets and DPO on CPU (fp32, gloo)."""
import os
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rlx_models_b200 import config as C
from rlx_models_b200.tokenizer import ByteTokenizer
from rlx_models_b200.train.data import PreferencePairs, SFTDataset
from rlx_models_b200.train.losses import dpo_loss
from rlx_models_b200.train.trainer import TrainConfig, Trainer
from rlx_models_b200.weights.init import random_weights


def _cfg():
    return C.tiny(num_hidden_layers=2, hidden_size=64, intermediate_size=128, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=16, vocab_size=256, tie_word_embeddings=True)


def _trainer(dora=False, **kw):
    cfg = _cfg()
    tc = TrainConfig(lr=5e-2, micro_batch=2, param_dtype="float32", lora_rank=4, lora_alpha=8.0, dora=dora,
                     activation_checkpointing=False)
    return Trainer(cfg, tc, random_weights(cfg, 0), device="cpu", **kw)


@pytest.mark.parametrize("dora", [False, True])
def test_lora_trains_adapters_only_and_merges(dora):
    t = _trainer(dora)
    base = [g.master.clone() for g in t.model.groups]
    b = torch.randint(0, 256, (4, 17), generator=torch.Generator().manual_seed(0))
    losses = [t.step(b).loss for _ in range(6)]
    assert losses[-1] < losses[0]
    for g, m in zip(t.model.groups, base):
        assert torch.equal(g.master, m), "base weights must stay frozen"
    # the export folds the adapters in: merged model == adapter model on the same input
    ids, tgt = b[:, :-1], b[:, 1:]
    with torch.no_grad():
        l_adapt = float(t.model.loss(ids, tgt))
    with tempfile.TemporaryDirectory() as d:
        t.export_hf(d)
        from rlx_models_b200.weights.weight_map import WeightMap
        cfg = _cfg()
        t2 = Trainer(cfg, TrainConfig(param_dtype="float32", activation_checkpointing=False), WeightMap.from_dir(d),
                     device="cpu")
        with torch.no_grad():
            l_merged = float(t2.model.loss(ids, tgt))
    assert abs(l_adapt - l_merged) < 1e-4 * max(1.0, abs(l_adapt))


def test_sft_dataset_masks_prompt_and_packs_text():
    tok = ByteTokenizer()
    recs = [{"prompt": "ab", "completion": "cd"}, {"text": "hello world"}, {"input_ids": [5, 6, 7]}]
    ds = SFTDataset(recs, tok, seq_len=8, eos_id=0)
    x, y = ds.rows[0]
    # ids a b c d eos -> inputs a b c d, targets b c d eos; prompt target (b) masked
    assert x[:4] == [97, 98, 99, 100] and y[:4] == [-1, 99, 100, 0] and y[4:] == [-1] * 4
    assert ds.rows[1][0][:3] == [5, 6, 0] and ds.rows[1][1][:2] == [6, 7]
    assert any(r[0][:5] == list(b"hello") for r in ds.rows)
    xb, yb = next(ds.batches(2, rank=0, world=1))
    assert xb.shape == (2, 8) and yb.dtype == torch.int64


def test_dpo_loss_and_step():
    import math
    z = torch.zeros(3)
    assert abs(float(dpo_loss(z, z, z, z)) - math.log(2)) < 1e-6
    t = _trainer()
    pairs = PreferencePairs([{"prompt": "q", "chosen": "good", "rejected": "bad!"}] * 2, ByteTokenizer(), 8)
    ch, rj = pairs.batch([0, 1])
    m0 = t.dpo_step(ch, rj, beta=0.5)
    assert abs(m0.loss - math.log(2)) < 1e-3  # adapters start at zero: policy == reference
    for _ in range(4):
        m = t.dpo_step(ch, rj, beta=0.5)
    assert m.loss < m0.loss


def _lora_worker(rank, world, port, d):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    t = _trainer(rank=rank, world=world)
    b = torch.randint(0, 256, (4, 17), generator=torch.Generator().manual_seed(rank))
    for _ in range(2):
        t.step(b)
    torch.save(t.lora.group_flat.master, os.path.join(d, f"a{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_lora_two_ranks_keep_adapters_in_sync():
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_lora_worker, args=(2, 29900 + os.getpid() % 40, d), nprocs=2, join=True)
        a0, a1 = torch.load(os.path.join(d, "a0.pt")), torch.load(os.path.join(d, "a1.pt"))
        assert torch.equal(a0, a1) and a0.abs().sum() > 0
