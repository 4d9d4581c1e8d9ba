"""GPU decoder + engine against the fp32 oracle.

Synthetic seeded weights (distinct per layer), bf16 on the GPU vs fp32 on the
CPU oracle with the same bf16-rounded weights. Checks logits (teacher forced)
and greedy tokens through the engine: chunked prefill, decode CUDA graphs,
prefix caching and eager/graph equivalence.
"""
import pytest
import torch

from rlx_models_b200 import config as C
from rlx_models_b200.models.decoder import DecoderLM
from rlx_models_b200.models.oracle import DecoderOracle
from rlx_models_b200.runtime.engine import EngineConfig, LLMEngine, SamplingParams
from rlx_models_b200.weights.init import random_weights

pytestmark = pytest.mark.gpu


def rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def _setup(cfg, seed=0):
    w = random_weights(cfg, seed=seed, dtype=torch.bfloat16)
    oracle = DecoderOracle(cfg, {k: v.float() for k, v in w.items()})
    model = DecoderLM(cfg, w, device="cuda")
    return model, oracle


@pytest.fixture(scope="module")
def tiny_model():
    cfg = C.tiny(num_hidden_layers=3, hidden_size=512, intermediate_size=1024, num_attention_heads=8,
                 num_key_value_heads=2, head_dim=128, vocab_size=1024)
    return (cfg,) + _setup(cfg, seed=11)


def test_teacher_forced_logits(tiny_model):
    cfg, model, oracle = tiny_model
    eng = LLMEngine(model, EngineConfig(max_num_seqs=8, max_batched_tokens=512, max_model_len=512,
                                        num_blocks=64, cuda_graphs=False, prefix_caching=False))
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg.vocab_size, (100,), generator=g)
    out = eng.generate([prompt.tolist()], SamplingParams(max_new_tokens=12, ignore_eos=True))[0]
    # oracle on the same token sequence
    ref_logits, _ = oracle.forward(torch.tensor(prompt.tolist() + out.token_ids[:-1]))
    ref_tokens = ref_logits[len(prompt) - 1:].argmax(-1).tolist()
    assert ref_tokens[0] == out.token_ids[0]
    agree = sum(int(a == b) for a, b in zip(ref_tokens, out.token_ids))
    assert agree >= len(out.token_ids) - 1
    # direct logits check through the model forward (prefill of the prompt)
    from rlx_models_b200.models.decoder import ForwardBatch
    kv = model.make_kv_cache(16)
    T = len(prompt)
    nb = (T + 15) // 16
    fb = ForwardBatch(input_ids=prompt.int().cuda(), positions=torch.arange(T, dtype=torch.int32).cuda(),
                      slots=torch.arange(T, dtype=torch.int64).cuda(), num_decode=0,
                      pre_block_tables=torch.arange(nb, dtype=torch.int32).view(1, -1).cuda(),
                      pre_ctx_lens=torch.tensor([T], dtype=torch.int32).cuda(),
                      pre_cu_q=torch.tensor([0, T], dtype=torch.int32).cuda(), pre_max_q=T,
                      logit_rows=None)
    lg = model.forward(fb, kv)
    ref_prefill, _ = oracle.forward(prompt)
    assert rel(lg.cpu(), ref_prefill) < 3e-2


def test_engine_graphs_chunking_prefix(tiny_model):
    cfg, model, _ = tiny_model
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 40, 77, 130, 16, 1)]
    sp = SamplingParams(max_new_tokens=20, ignore_eos=True)

    def run(**kw):
        e = LLMEngine(model, EngineConfig(max_num_seqs=8, max_model_len=512, num_blocks=128, **kw))
        return [o.token_ids for o in e.generate(prompts, sp)], e

    base, e0 = run(max_batched_tokens=1024, cuda_graphs=False, prefix_caching=False)
    graphs, e1 = run(max_batched_tokens=1024, cuda_graphs=True, prefix_caching=False)
    assert e1.stats["graph_steps"] > 0
    assert graphs == base
    chunked, _ = run(max_batched_tokens=48, cuda_graphs=True, prefix_caching=False)
    # chunking changes GEMM shapes (and so bf16 rounding) upstream of attention;
    # a tiny random model's greedy continuations may then part at a near-tie
    # (chunked-prefill logits are checked directly in test_chunked_prefill_logits)

    def common_prefix(a, b):
        n = 0
        while n < min(len(a), len(b)) and a[n] == b[n]:
            n += 1
        return n / max(1, len(b))

    cp = [common_prefix(a, b) for a, b in zip(chunked, base)]
    assert sum(cp) / len(base) >= 0.5, cp
    # prefix cache: same prompts twice through one engine
    e = LLMEngine(model, EngineConfig(max_num_seqs=8, max_model_len=512, num_blocks=128, prefix_caching=True))
    first = [o.token_ids for o in e.generate(prompts, sp)]
    second = e.generate(prompts, sp)
    assert sum(o.cached_prompt_tokens for o in second) > 0
    pc = [common_prefix(o.token_ids, a) for a, o in zip(first, second)]
    assert sum(pc) / len(pc) >= 0.5, pc


def test_sampling_through_engine(tiny_model):
    cfg, model, _ = tiny_model
    e = LLMEngine(model, EngineConfig(max_num_seqs=8, max_model_len=256, num_blocks=64))
    p = [[1, 2, 3, 4, 5]] * 4
    sp = SamplingParams(max_new_tokens=16, temperature=0.8, top_k=50, top_p=0.9, seed=7, ignore_eos=True,
                        logprobs=True)
    a = e.generate(p, sp)
    assert all(len(o.token_ids) == 16 for o in a)
    assert all(o.logprobs is not None and all(lp <= 0 for lp in o.logprobs) for o in a)
    # different sequences (different seq ids in the seed) should not all coincide
    assert len({tuple(o.token_ids) for o in a}) > 1


def test_qwen3_0_6b_shape_vs_cpu_oracle():
    """Config 1 shape (28 layers, 1024 hidden, 16/8 heads, vocab 151936, tied):
    128-token prompt, GPU bf16 greedy vs fp32 CPU oracle, teacher-forced."""
    cfg = C.qwen3_0_6b()
    w = random_weights(cfg, seed=0, dtype=torch.bfloat16)
    model = DecoderLM(cfg, w, device="cuda")
    e = LLMEngine(model, EngineConfig(max_num_seqs=4, max_model_len=512, num_blocks=64))
    prompt = torch.randint(0, cfg.vocab_size, (128,), generator=torch.Generator().manual_seed(1)).tolist()
    out = e.generate([prompt], SamplingParams(max_new_tokens=8, ignore_eos=True))[0]
    oracle = DecoderOracle(cfg, {k: v.float() for k, v in w.items()})
    ref_logits, _ = oracle.forward(torch.tensor(prompt + out.token_ids[:-1]))
    ref_tok = ref_logits[127:].argmax(-1).tolist()
    assert ref_tok[0] == out.token_ids[0]
    assert sum(int(a == b) for a, b in zip(ref_tok, out.token_ids)) >= 7



def test_chunked_prefill_logits(tiny_model):
    """Prefill in chunks over the cached pages == one-shot prefill (logits of every position)."""
    from rlx_models_b200.models.decoder import ForwardBatch
    cfg, model, _ = tiny_model
    T = 130
    ids = torch.randint(0, cfg.vocab_size, (T,), generator=torch.Generator().manual_seed(5)).int().cuda()
    nb = (T + 15) // 16
    table = torch.arange(nb, dtype=torch.int32).view(1, -1).cuda()

    def run(kv, lo, hi):
        n = hi - lo
        fb = ForwardBatch(input_ids=ids[lo:hi], positions=torch.arange(lo, hi, dtype=torch.int32).cuda(),
                          slots=torch.arange(lo, hi, dtype=torch.int64).cuda(), num_decode=0,
                          pre_block_tables=table, pre_ctx_lens=torch.tensor([hi], dtype=torch.int32).cuda(),
                          pre_cu_q=torch.tensor([0, n], dtype=torch.int32).cuda(), pre_max_q=n)
        return model.forward(fb, kv)

    full = run(model.make_kv_cache(nb), 0, T)
    kv = model.make_kv_cache(nb)
    parts = [run(kv, lo, min(T, lo + 48)) for lo in range(0, T, 48)]
    chunked = torch.cat(parts)
    assert rel(chunked.cpu(), full.cpu()) < 2e-2


def test_prompt_cache_save_load_roundtrip(cuda, tmp_path):
    """A prompt's cached KV saved by one engine and loaded into a fresh one is
    reused (no recompute of those tokens) and gives the same greedy output; a
    file from another model is refused."""
    from rlx_models_b200 import config as C
    from rlx_models_b200.models.decoder import DecoderLM
    from rlx_models_b200.runtime.engine import EngineConfig, LLMEngine, SamplingParams
    from rlx_models_b200.weights.init import random_weights
    cfg = C.tiny(num_hidden_layers=2, hidden_size=2048, intermediate_size=2048, num_attention_heads=16,
                 num_key_value_heads=8, head_dim=128, vocab_size=4096)
    m = DecoderLM(cfg, random_weights(cfg, seed=1, device=cuda), device=cuda)
    prompt = torch.randint(0, cfg.vocab_size, (70,), generator=torch.Generator().manual_seed(0)).tolist()
    sp = SamplingParams(max_new_tokens=6, ignore_eos=True)
    ecfg = EngineConfig(max_num_seqs=8, max_batched_tokens=256, max_model_len=256, num_blocks=64)
    e1 = LLMEngine(m, ecfg)
    ref = e1.generate([prompt], sp)[0].token_ids
    path = str(tmp_path / "p.safetensors")
    assert e1.save_prompt_cache(path, prompt) == 64
    e2 = LLMEngine(m, ecfg)
    assert e2.load_prompt_cache(path) == 64
    out = e2.generate([prompt], sp)[0]
    assert out.cached_prompt_tokens == 64 and out.token_ids == ref
    other = DecoderLM(cfg, random_weights(cfg, seed=2, device=cuda), device=cuda)
    assert LLMEngine(other, ecfg).load_prompt_cache(path) == 0
