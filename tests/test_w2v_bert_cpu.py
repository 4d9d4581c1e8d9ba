"""w2v-BERT 2.0 Conformer CTC on CPU against transformers Wav2Vec2BertForCTC:
encoder output and CTC logits with the clipped relative-key distance bias
(sequences longer than both clip distances) and without position bias; the
greedy CTC decode of those logits."""
import math

import pytest
import torch


def _rand(m):
    torch.manual_seed(0)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 1 / math.sqrt(p[0].numel()))
            else:
                p.normal_(1.0 if ("norm" in n and n.endswith("weight")) else 0.0, 0.1)
    return m.eval()


@pytest.mark.parametrize("pos", ["relative_key", None])
def test_w2v_bert_ctc_matches_transformers(pos):
    import transformers as T
    from rlx_models_b200.models.w2v_bert import W2vBertConfig, W2vBertCTC
    hcfg = T.Wav2Vec2BertConfig(hidden_size=32, num_hidden_layers=2, num_attention_heads=4, intermediate_size=48,
                                feature_projection_input_dim=20, conv_depthwise_kernel_size=5,
                                position_embeddings_type=pos, left_max_position_embeddings=6,
                                right_max_position_embeddings=3, vocab_size=24, pad_token_id=0, add_adapter=False)
    m = _rand(T.Wav2Vec2BertForCTC(hcfg))
    feats = torch.randn(1, 29, 20, generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        out = m(input_features=feats, output_hidden_states=True)
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    model = W2vBertCTC(W2vBertConfig.from_dict(hcfg.to_dict()), sd)
    lg = model.logits(feats[0])
    assert (lg - out.logits[0]).abs().max() < 1e-4, (lg - out.logits[0]).abs().max()
    ids = model.transcribe_ids(feats[0])
    best = out.logits[0].argmax(-1).tolist()
    ref = [t for i, t in enumerate(best) if t != 0 and (i == 0 or t != best[i - 1])]
    assert ids == ref


def test_fbank_features_match_seamless_extractor():
    import numpy as np
    import transformers as T
    from rlx_models_b200.models.w2v_bert import fbank_features
    fe = T.SeamlessM4TFeatureExtractor()
    a = (0.1 * torch.randn(16000 + 1234, generator=torch.Generator().manual_seed(4))).numpy().astype(np.float32)
    ref = torch.from_numpy(fe(a, sampling_rate=16000, return_tensors="np")["input_features"][0])
    got = fbank_features(a)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert (got - ref).abs().max() < 2e-3, (got - ref).abs().max()


def test_transcriber_runs_end_to_end():
    from rlx_models_b200.models.w2v_bert import W2vBertConfig, W2vBertCTC, W2vBertTranscriber
    import transformers as T
    hcfg = T.Wav2Vec2BertConfig(hidden_size=32, num_hidden_layers=1, num_attention_heads=4, intermediate_size=48,
                                feature_projection_input_dim=160, conv_depthwise_kernel_size=5, vocab_size=24,
                                pad_token_id=0, add_adapter=False)
    m = _rand(T.Wav2Vec2BertForCTC(hcfg))
    sd = {k: v.detach() for k, v in m.state_dict().items()}
    tr = W2vBertTranscriber(W2vBertCTC(W2vBertConfig.from_dict(hcfg.to_dict()), sd))
    ids = tr.transcribe(0.1 * torch.randn(8000, generator=torch.Generator().manual_seed(5)), sample_rate=8000)
    assert isinstance(ids, list) and all(0 < t < 24 for t in ids)
