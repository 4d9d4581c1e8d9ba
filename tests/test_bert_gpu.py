"""BERT encoder on the GPU (bf16 GEMMs on the tcgen05 linear) against the fp32 CPU path."""
import pytest
import torch

from rlx_models_b200.models.bert import BertConfig, BertEncoder

pytestmark = pytest.mark.gpu


def test_bert_gpu_matches_cpu(cuda):
    cfg = BertConfig(vocab_size=300, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                     intermediate_size=512, max_position_embeddings=64)
    g = torch.Generator().manual_seed(0)
    H, I = cfg.hidden_size, cfg.intermediate_size
    w = {"embeddings.word_embeddings.weight": torch.randn(300, H, generator=g) * 0.05,
         "embeddings.position_embeddings.weight": torch.randn(64, H, generator=g) * 0.05,
         "embeddings.token_type_embeddings.weight": torch.randn(2, H, generator=g) * 0.05,
         "embeddings.LayerNorm.weight": torch.ones(H), "embeddings.LayerNorm.bias": torch.zeros(H)}
    for i in range(cfg.num_hidden_layers):
        p = f"encoder.layer.{i}."
        for n in ("query", "key", "value"):
            w[p + f"attention.self.{n}.weight"] = torch.randn(H, H, generator=g) * 0.05
            w[p + f"attention.self.{n}.bias"] = torch.randn(H, generator=g) * 0.02
        w[p + "attention.output.dense.weight"] = torch.randn(H, H, generator=g) * 0.05
        w[p + "attention.output.dense.bias"] = torch.zeros(H)
        w[p + "attention.output.LayerNorm.weight"], w[p + "attention.output.LayerNorm.bias"] = torch.ones(H), torch.zeros(H)
        w[p + "intermediate.dense.weight"], w[p + "intermediate.dense.bias"] = torch.randn(I, H, generator=g) * 0.05, torch.zeros(I)
        w[p + "output.dense.weight"], w[p + "output.dense.bias"] = torch.randn(H, I, generator=g) * 0.05, torch.zeros(H)
        w[p + "output.LayerNorm.weight"], w[p + "output.LayerNorm.bias"] = torch.ones(H), torch.zeros(H)
    ids = torch.randint(1, 300, (4, 48), generator=g)
    mask = torch.ones(4, 48, dtype=torch.long)
    mask[3, 30:] = 0
    a = BertEncoder(cfg, w).embed(ids, mask)
    b = BertEncoder(cfg, w, device=cuda).embed(ids, mask).cpu()
    assert torch.nn.functional.cosine_similarity(a, b, dim=-1).min() > 0.999
