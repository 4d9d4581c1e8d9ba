"""TimesFM forecasting on CPU against transformers' TimesFmModelForPrediction
(the fp32 oracle): series shorter and longer than the context, per-series
frequencies, with and without positional embeddings, the moving-average
trend / residual decomposition, and a forecast longer than one model step."""
import pytest
import torch

from rlx_models_b200.models.timesfm import TimesFm, TimesFmConfig

transformers = pytest.importorskip("transformers")


def _pair(pe: bool, seed=0):
    torch.manual_seed(seed)
    hc = transformers.TimesFmConfig(patch_length=8, context_length=64, horizon_length=16, num_hidden_layers=2,
                                    hidden_size=32, intermediate_size=32, head_dim=8, num_attention_heads=4,
                                    use_positional_embedding=pe)
    hm = transformers.TimesFmModelForPrediction(hc).eval()
    sd = {k: v if "inv_timescales" in k else v + 0.1 * torch.randn_like(v) for k, v in hm.state_dict().items()}
    hm.load_state_dict(sd)
    return hm, TimesFm(TimesFmConfig.from_dict(hc.to_dict()), sd)


SERIES = [torch.randn(50).cumsum(0), torch.randn(80).cumsum(0) + 5, torch.sin(torch.arange(30.0) / 3)]


@pytest.mark.parametrize("pe", [False, True])
@pytest.mark.parametrize("window", [None, 5])
def test_forecast_matches_transformers(pe, window):
    hm, m = _pair(pe)
    with torch.no_grad():
        ref = hm(past_values=SERIES, freq=[0, 1, 2], window_size=window)
    mean, full = m.forecast(SERIES, freq=[0, 1, 2], window_size=window)
    torch.testing.assert_close(full, ref.full_predictions, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(mean, ref.mean_predictions, atol=1e-4, rtol=1e-4)


def test_long_horizon_chains_model_steps():
    hm, m = _pair(False, seed=1)
    mean, full = m.forecast(SERIES[:2], horizon=40)
    assert mean.shape == (2, 40) and full.shape == (2, 40, 10)
    first, _ = m.forecast(SERIES[:2], horizon=16)
    torch.testing.assert_close(mean[:, :16], first)
    # the second step sees the first step's mean forecast appended to the context
    ext = [torch.cat([s[-64:], first[i]]) for i, s in enumerate(SERIES[:2])]
    nxt, _ = m.forecast(ext, horizon=16)
    torch.testing.assert_close(mean[:, 16:32], nxt, atol=1e-4, rtol=1e-4)


def test_load_forecaster(tmp_path):
    import json

    from rlx_models_b200.api import load_forecaster
    from rlx_models_b200.weights.safetensors_io import save_file
    hm, m = _pair(False, seed=2)
    d = tmp_path / "tfm"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(hm.config.to_dict()))
    save_file({k: v.contiguous() for k, v in hm.state_dict().items()}, str(d / "model.safetensors"))
    f = load_forecaster(str(d), device="cpu")
    torch.testing.assert_close(f.forecast(SERIES)[0], m.forecast(SERIES)[0])
