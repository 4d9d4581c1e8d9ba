"""TimesFM on the GPU (bf16 linears on the tcgen05 GEMM) against the fp32 CPU model."""
import pytest
import torch

from rlx_models_b200.models.timesfm import TimesFm, TimesFmConfig

pytestmark = pytest.mark.gpu


def test_timesfm_gpu_matches_cpu():
    transformers = pytest.importorskip("transformers")
    torch.manual_seed(0)
    hc = transformers.TimesFmConfig(patch_length=16, context_length=128, horizon_length=32, num_hidden_layers=2,
                                    hidden_size=64, intermediate_size=64, head_dim=16, num_attention_heads=4)
    hm = transformers.TimesFmModelForPrediction(hc)
    sd = {k: v if "inv_timescales" in k else v + 0.05 * torch.randn_like(v) for k, v in hm.state_dict().items()}
    cfg = TimesFmConfig.from_dict(hc.to_dict())
    cpu, gpu = TimesFm(cfg, sd), TimesFm(cfg, sd, device="cuda")
    series = [torch.randn(100).cumsum(0), torch.sin(torch.arange(60.0) / 4) * 3]
    ref, _ = cpu.forecast(series, freq=[0, 1])
    got, _ = gpu.forecast(series, freq=[0, 1])
    assert (got - ref).norm() / ref.norm() < 3e-2
