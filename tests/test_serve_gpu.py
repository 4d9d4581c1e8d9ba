"""OpenAI server over the real engine and a tiny Qwen3 model on the GPU."""
import json

import pytest

pytestmark = pytest.mark.gpu


def test_openai_server_real_engine(cuda):
    from fastapi.testclient import TestClient

    from rlx_models_b200 import config as C
    from rlx_models_b200.api import LLM
    from rlx_models_b200.registry import build_model
    from rlx_models_b200.runtime.engine import EngineConfig
    from rlx_models_b200.serve.openai_server import create_app
    from rlx_models_b200.serve.runner import EngineRunner
    from rlx_models_b200.tokenizer import ByteTokenizer

    cfg = C.tiny()
    llm = LLM(build_model(cfg, device=cuda, seed=0), EngineConfig(max_num_seqs=8, max_model_len=256, num_blocks=64))
    tok = ByteTokenizer()
    runner = EngineRunner(llm.engine, tok)
    try:
        with TestClient(create_app(runner, tok, "tiny")) as c:
            r = c.post("/v1/completions", json={"prompt": [1, 2, 3, 4], "max_tokens": 8, "temperature": 0,
                                               "ignore_eos": True})
            j = r.json()
            ref = llm.generate([[1, 2, 3, 4]], __import__("rlx_models_b200.runtime.engine", fromlist=["x"])
                               .SamplingParams(max_new_tokens=8, ignore_eos=True))[0].token_ids
            assert j["choices"][0]["token_ids"] == ref
            with c.stream("POST", "/v1/chat/completions",
                          json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 6,
                                "stream": True, "temperature": 0.7, "seed": 3}) as s:
                lines = [ln for ln in s.iter_lines() if ln]
            assert lines[-1] == "data: [DONE]"
            assert json.loads(lines[-2][6:])["usage"]["completion_tokens"] == 6
    finally:
        runner.shutdown()
