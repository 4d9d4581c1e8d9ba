"""NLLB / M2M-100 on the GPU (bf16 linears on the tcgen05 GEMM) against the
fp32 CPU model: encoder states and teacher-forced decoder logits."""
import pytest
import torch

from rlx_models_b200.models.nllb import NllbConfig, NllbTranslator

pytestmark = pytest.mark.gpu


def test_nllb_gpu_matches_cpu():
    transformers = pytest.importorskip("transformers")
    torch.manual_seed(0)
    hc = transformers.M2M100Config(vocab_size=256, d_model=128, encoder_layers=2, decoder_layers=2,
                                   encoder_attention_heads=4, decoder_attention_heads=4, encoder_ffn_dim=256,
                                   decoder_ffn_dim=256, max_position_embeddings=64)
    hm = transformers.M2M100ForConditionalGeneration(hc)
    sd = {k: (v + 0.02 * torch.randn_like(v)) if v.dtype.is_floating_point else v for k, v in hm.state_dict().items()
          if "embed_positions" not in k}
    sd["lm_head.weight"] = sd["model.shared.weight"]
    cfg = NllbConfig.from_dict(hc.to_dict())
    cpu, gpu = NllbTranslator(cfg, sd), NllbTranslator(cfg, sd, device="cuda")
    src = torch.tensor([[5, 17, 33, 40, 2], [9, 12, 2, 1, 1]])
    tgt = torch.tensor([[2, 50, 7, 8], [2, 50, 11, 12]])
    e_ref, m_ref = cpu.encode(src)
    e, m = gpu.encode(src)
    for b, n in ((0, 5), (1, 3)):
        assert (e[b, :n].cpu() - e_ref[b, :n]).norm() / e_ref[b, :n].norm() < 3e-2
    ref = cpu.decode_step(tgt, 0, [], cpu.cross_kv(e_ref), m_ref)
    got = gpu.decode_step(tgt, 0, [], gpu.cross_kv(e), m).cpu()
    assert (got - ref).norm() / ref.norm() < 3e-2
