"""V-JEPA 2 on CPU against transformers (the fp32 oracle): encoder tokens
(tubelet embedding, 3-D rotary attention incl. head dims with a pass-through
remainder) and the attentive-probe classifier's logits."""
import pytest
import torch

from rlx_models_b200.models.vjepa2 import VJEPA2, VJEPA2Config

transformers = pytest.importorskip("transformers")


@pytest.mark.parametrize("hidden,heads", [(48, 2), (64, 2)])
def test_features_and_classifier_match_transformers(hidden, heads):
    torch.manual_seed(0)
    hc = transformers.VJEPA2Config(patch_size=4, crop_size=16, frames_per_clip=4, tubelet_size=2,
                                   hidden_size=hidden, num_attention_heads=heads, num_hidden_layers=2,
                                   num_pooler_layers=1, pred_hidden_size=24, pred_num_attention_heads=2,
                                   pred_num_hidden_layers=1, num_labels=5)
    hm = transformers.VJEPA2ForVideoClassification(hc).eval()
    sd = {k: v + 0.05 * torch.randn_like(v) for k, v in hm.state_dict().items()}
    hm.load_state_dict(sd)
    m = VJEPA2(VJEPA2Config.from_dict(hc.to_dict()), sd)
    vid = torch.randn(2, 4, 3, 16, 16)
    with torch.no_grad():
        feats = hm.vjepa2(vid, skip_predictor=True).last_hidden_state
        logits = hm(vid).logits
    torch.testing.assert_close(m.features(vid), feats, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(m.classify(vid), logits, atol=1e-5, rtol=1e-4)


def test_encoder_only_checkpoint():
    torch.manual_seed(1)
    hc = transformers.VJEPA2Config(patch_size=4, crop_size=16, frames_per_clip=4, tubelet_size=2, hidden_size=48,
                                   num_attention_heads=2, num_hidden_layers=1, pred_hidden_size=24,
                                   pred_num_attention_heads=2, pred_num_hidden_layers=1)
    hm = transformers.VJEPA2Model(hc).eval()
    m = VJEPA2(VJEPA2Config.from_dict(hc.to_dict()), hm.state_dict())
    vid = torch.randn(1, 4, 3, 16, 16)
    with torch.no_grad():
        ref = hm(vid, skip_predictor=True).last_hidden_state
    torch.testing.assert_close(m.features(vid), ref, atol=1e-4, rtol=1e-4)
    with pytest.raises(ValueError):
        m.pooled(vid)
