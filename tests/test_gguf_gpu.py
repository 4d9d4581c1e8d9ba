"""GGUF on the GPU: the device dequantisation kernel against the CPU block
formulas (bit for bit, every block type), and a decoder loaded from a
quantised GGUF file through ``api.load`` against the fp32 oracle on the same
dequantised weights."""
import pytest
import torch

from rlx_models_b200 import ops
from rlx_models_b200.weights import gguf as G

from test_gguf_cpu import random_blocks

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", ["Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K",
                                  "Q8_K"])
def test_gguf_dequant_kernel(cuda, kind):
    raw, be = random_blocks(kind, 37, seed=5)
    ref = G.dequantize_blocks(raw, kind)
    got32 = ops.gguf_dequant(raw.to(cuda), kind, (37 * be,), torch.float32)
    got16 = ops.gguf_dequant(raw.to(cuda), kind, (37 * be,), torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.equal(got32.cpu(), ref)
    assert torch.equal(got16.cpu(), ref.bfloat16())


def test_load_gguf_model_on_gpu(cuda, tmp_path):
    from rlx_models_b200 import config as C
    from rlx_models_b200.api import load
    from rlx_models_b200.models.oracle import DecoderOracle
    from rlx_models_b200.weights.init import random_weights
    cfg = C.tiny("qwen3", num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=64, vocab_size=512, tie_word_embeddings=False)
    w = random_weights(cfg, 0)
    p = G.save_gguf(str(tmp_path / "m-Q8_0.gguf"), w, cfg, kind="Q8_0")
    llm = load(str(tmp_path), device=cuda)  # directory without config.json: picks the GGUF file
    ids = torch.randint(0, 512, (20,), generator=torch.Generator().manual_seed(1))
    lg = llm.logits(ids.tolist()).float().cpu()
    gw = G.GGUFWeights(p, dtype=torch.float32)
    ref, _ = DecoderOracle(gw.config, {k: gw.take(k) for k in gw.keys()}).forward(ids)
    assert ((lg - ref).norm() / ref.norm()).item() < 2e-2
    out = llm.generate([ids.tolist()])[0]
    assert len(out.token_ids) > 0
