"""Mimi on the GPU (SEANet convs on the codec blocks, Transformer linears on
the tcgen05 GEMM, bf16) against the fp32 CPU model."""
import pytest
import torch

from rlx_models_b200.models.mimi import MimiConfig, MimiModel

pytestmark = pytest.mark.gpu


def test_mimi_gpu_matches_cpu():
    transformers = pytest.importorskip("transformers")
    torch.manual_seed(0)
    hc = transformers.MimiConfig(hidden_size=64, num_filters=16, upsampling_ratios=[4, 2], codebook_size=32,
                                 codebook_dim=32, num_quantizers=4, vector_quantization_hidden_dimension=32,
                                 upsample_groups=64, num_hidden_layers=2, intermediate_size=128,
                                 num_attention_heads=4, num_key_value_heads=4, head_dim=16, sliding_window=8,
                                 sampling_rate=1600)
    hm = transformers.MimiModel(hc)
    sd = {}
    for k, v in hm.state_dict().items():
        if v.dtype.is_floating_point:
            v = v + 0.05 * torch.randn_like(v)
            if k.endswith("cluster_usage"):
                v = v.abs() + 0.5
        sd[k] = v
    cfg = MimiConfig.from_dict(hc.to_dict())
    cpu, gpu = MimiModel(cfg, sd), MimiModel(cfg, sd, device="cuda")
    x = 0.3 * torch.randn(2, 1, 1600)
    z_ref, z = cpu.encode_latents(x), gpu.encode_latents(x).cpu()
    assert (z - z_ref).norm() / z_ref.norm() < 3e-2
    codes = cpu.encode(x)
    assert (gpu.encode(x).cpu()[:, 0] == codes[:, 0]).float().mean() > 0.8
    a_ref, a = cpu.decode(codes), gpu.decode(codes.cuda()).cpu()
    assert a.shape == a_ref.shape and (a - a_ref).norm() / a_ref.norm() < 5e-2
