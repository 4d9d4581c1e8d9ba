"""CSM on the GPU (both decoders' linears on the tcgen05 GEMM, bf16) against
the fp32 CPU model: backbone hidden state, depth-decoder codes for one backbone
state, and the codebook-0 logits of a prompt."""
import pytest
import torch

from rlx_models_b200.models.csm import CsmConfig, CsmModel

pytestmark = pytest.mark.gpu


def test_csm_gpu_matches_cpu():
    transformers = pytest.importorskip("transformers")
    torch.manual_seed(0)
    depth = dict(model_type="csm_depth_decoder_model", num_codebooks=4, backbone_hidden_size=128, vocab_size=32,
                 hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=16, max_position_embeddings=5)
    hc = transformers.CsmConfig(num_codebooks=4, vocab_size=32, text_vocab_size=64, hidden_size=128,
                                intermediate_size=256, num_hidden_layers=2, num_attention_heads=4,
                                num_key_value_heads=2, head_dim=32, codebook_pad_token_id=31, audio_token_id=62,
                                audio_eos_token_id=63, pad_token_id=62, bos_token_id=1, depth_decoder_config=depth,
                                codec_config=dict(model_type="mimi"))
    hm = transformers.CsmForConditionalGeneration(hc)
    sd = {k: (v + 0.05 * torch.randn_like(v)) if v.dtype.is_floating_point else v for k, v in hm.state_dict().items()
          if not k.startswith("codec_model.")}
    cfg = CsmConfig.from_dict(hc.to_dict())
    cpu, gpu = CsmModel(cfg, sd, codec=False), CsmModel(cfg, sd, device="cuda", codec=False)
    ids = torch.tensor([[1, 5, 7, 9, 11, 13]])
    h_ref = cpu.backbone.forward(cpu.text_prompt(ids), 0, [])[:, -1]
    h = gpu.backbone.forward(gpu.text_prompt(ids), 0, [])[:, -1].cpu()
    assert (h - h_ref).norm() / h_ref.norm() < 3e-2
    lg_ref = cpu._lin(h_ref, cpu.head0)
    lg = gpu._lin(h.cuda(), gpu.head0).cpu()
    assert (lg - lg_ref).norm() / lg_ref.norm() < 3e-2
    c0 = lg_ref.argmax(-1)
    codes_ref = cpu.depth_codes(h_ref, c0)
    codes = gpu.depth_codes(h_ref.cuda(), c0.cuda()).cpu()
    assert codes.shape == codes_ref.shape and (codes == codes_ref).float().mean() >= 0.5
