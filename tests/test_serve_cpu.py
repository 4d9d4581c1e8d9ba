"""OpenAI server + engine thread against a fake engine (no GPU): routes,
token-id and text prompts, SSE framing, stop strings aborting in the engine,
concurrent requests sharing one batch, metrics."""
import json
import threading
from dataclasses import dataclass, field

import pytest

fastapi = pytest.importorskip("fastapi")
from fastapi.testclient import TestClient  # noqa: E402

from rlx_models_b200.serve.openai_server import create_app  # noqa: E402
from rlx_models_b200.serve.runner import EngineRunner  # noqa: E402
from rlx_models_b200.tokenizer import ByteTokenizer  # noqa: E402


@dataclass
class _St:
    tokens: list = field(default_factory=list)
    logprobs: list = field(default_factory=list)


@dataclass
class _Out:
    seq_id: int
    token_ids: list
    finish_reason: str
    logprobs: list | None = None


class FakeEngine:
    """Emits prompt[-1] + 1, + 2, ... (bytes) one token per step for every live request."""

    def __init__(self):
        self.requests, self.params, self.max_batch, self.aborted = {}, {}, 0, []
        self._n = 0
        self.lock = threading.Lock()

    def add_request(self, ids, params):
        self._n += 1
        self.requests[self._n] = _St()
        self.params[self._n] = (ids, params)
        return self._n

    def abort(self, sid):
        self.aborted.append(sid)
        self.requests.pop(sid, None)

    def has_unfinished(self):
        return bool(self.requests)

    def step(self):
        import time
        time.sleep(0.002)  # a device step takes time; lets concurrent clients join the batch
        self.max_batch = max(self.max_batch, len(self.requests))
        done = []
        for sid, st in list(self.requests.items()):
            ids, p = self.params[sid]
            t = (ids[-1] + len(st.tokens) + 1) % 256
            st.tokens.append(t)
            if p.logprobs:
                st.logprobs.append(-0.5 * len(st.tokens))
            if t in p.stop_token_ids or len(st.tokens) >= p.max_new_tokens:
                done.append(_Out(sid, list(st.tokens), "stop" if t in p.stop_token_ids else "length",
                                 list(st.logprobs) if p.logprobs else None))
                del self.requests[sid]
        return done


@pytest.fixture()
def client():
    eng = FakeEngine()
    tok = ByteTokenizer()
    runner = EngineRunner(eng, tok)
    app = create_app(runner, tok, "fake")
    with TestClient(app) as c:
        yield c, eng
    runner.shutdown()


def test_completion_token_ids(client):
    c, _ = client
    r = c.post("/v1/completions", json={"prompt": [10, 20], "max_tokens": 4, "temperature": 0})
    assert r.status_code == 200
    j = r.json()
    assert j["choices"][0]["token_ids"] == [21, 22, 23, 24]
    assert j["choices"][0]["finish_reason"] == "length"
    assert j["usage"] == {"prompt_tokens": 2, "completion_tokens": 4, "total_tokens": 6}


def test_text_prompt_stop_string_and_stream(client):
    c, eng = client
    # "a" = 97 -> generates "bcdef..." ; stop at "de"
    r = c.post("/v1/completions", json={"prompt": "a", "max_tokens": 20, "stop": ["de"]})
    assert r.json()["choices"][0]["text"] == "bc"
    assert eng.aborted, "stop string must abort the request in the engine"
    with c.stream("POST", "/v1/completions", json={"prompt": "a", "max_tokens": 5, "stream": True}) as s:
        lines = [ln for ln in s.iter_lines() if ln]
    assert lines[-1] == "data: [DONE]"
    chunks = [json.loads(ln[6:]) for ln in lines[:-1]]
    assert "".join(ch["choices"][0]["text"] for ch in chunks) == "bcdef"
    assert chunks[-1]["choices"][0]["finish_reason"] == "length"


def test_chat_and_models_and_metrics(client):
    c, _ = client
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 3})
    j = r.json()
    assert j["object"] == "chat.completion" and j["choices"][0]["message"]["role"] == "assistant"
    assert c.get("/v1/models").json()["data"][0]["id"] == "fake"
    m = c.get("/metrics").text
    assert "b200_requests_total" in m and "b200_generated_tokens_total" in m


def test_concurrent_requests_share_a_batch(client):
    c, eng = client
    res = {}

    def go(i):
        res[i] = c.post("/v1/completions", json={"prompt": [i], "max_tokens": 30}).json()

    th = [threading.Thread(target=go, args=(i,)) for i in range(6)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    assert all(len(res[i]["choices"][0]["token_ids"]) == 30 for i in range(6))
    assert eng.max_batch >= 2


class ScriptedEngine(FakeEngine):
    """Emits the bytes of a fixed reply, one per step."""

    def __init__(self, reply: str):
        super().__init__()
        self.reply = list(reply.encode())

    def step(self):
        done = []
        for sid, st in list(self.requests.items()):
            ids, p = self.params[sid]
            st.tokens.append(self.reply[len(st.tokens)])
            if len(st.tokens) >= min(len(self.reply), p.max_new_tokens):
                done.append(_Out(sid, list(st.tokens), "stop"))
                del self.requests[sid]
        return done


TOOLS = [{"type": "function", "function": {"name": "get_weather", "parameters": {
    "type": "object", "properties": {"city": {"type": "string"}}, "required": ["city"]}}}]


@pytest.mark.parametrize("reply,expect", [
    ('Checking.<tool_call>{"name": "get_weather", "arguments": {"city": "Oslo", "junk": 1}}</tool_call>', "call"),
    ('<tool_call>{"name": "launch_rocket", "arguments": {}}</tool_call>', "rejected"),
    ("It is sunny.", "text")])
def test_chat_tool_calls_validated(reply, expect):
    eng = ScriptedEngine(reply)
    tok = ByteTokenizer()
    runner = EngineRunner(eng, tok)
    app = create_app(runner, tok, "fake")
    with TestClient(app) as c:
        r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "weather?"}],
                                                 "tools": TOOLS, "max_tokens": 500, "ignore_eos": True})
    runner.shutdown()
    ch = r.json()["choices"][0]
    if expect == "call":
        assert ch["finish_reason"] == "tool_calls" and ch["message"]["content"] == "Checking."
        fn = ch["message"]["tool_calls"][0]["function"]
        assert fn["name"] == "get_weather" and json.loads(fn["arguments"]) == {"city": "Oslo"}
    elif expect == "rejected":
        assert "tool_calls" not in ch["message"] and "unknown tool" in ch["guardrail_errors"][0]
    else:
        assert ch["message"]["content"] == "It is sunny." and "tool_calls" not in ch["message"]
    # the tool catalog reached the prompt
    ids, _ = eng.params[1]
    assert b"get_weather" in bytes(ids)


def test_chat_compaction_budget(client):
    c, eng = client
    msgs = [{"role": "system", "content": "SYS"}] + [{"role": "user", "content": "x" * 400}] * 5 + \
           [{"role": "user", "content": "last"}]
    r = c.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 2, "max_context_tokens": 120})
    assert r.status_code == 200
    ids, _ = eng.params[1]
    assert len(ids) < 300 and b"SYS" in bytes(ids) and b"last" in bytes(ids)


class _FakeEmbedder:
    def embed(self, inputs):
        import torch
        return torch.stack([torch.tensor([float(len(x)), 1.0, 0.5]) for x in inputs])


def test_embeddings_endpoint():
    eng = FakeEngine()
    tok = ByteTokenizer()
    runner = EngineRunner(eng, tok)
    with TestClient(create_app(runner, tok, "fake", embedder=_FakeEmbedder())) as c:
        r = c.post("/v1/embeddings", json={"input": ["abc", "hello"]}).json()
        assert [d["index"] for d in r["data"]] == [0, 1]
        assert r["data"][1]["embedding"] == [5.0, 1.0, 0.5]
        assert r["usage"]["prompt_tokens"] == 8
        r = c.post("/v1/embeddings", json={"input": [1, 2, 3, 4]}).json()
        assert len(r["data"]) == 1 and r["data"][0]["embedding"][0] == 4.0
        assert c.post("/v1/embeddings", json={"input": []}).status_code == 400
    runner.shutdown()
    runner = EngineRunner(FakeEngine(), tok)
    with TestClient(create_app(runner, tok, "fake")) as c:
        assert c.post("/v1/embeddings", json={"input": "x"}).status_code == 404
    runner.shutdown()


class _FakeTranscriber:
    def transcribe(self, audio, sr):
        return f"{audio.numel()} samples at {sr} Hz, peak {float(audio.abs().max()):.2f}"


def test_transcriptions_endpoint():
    import io
    import struct
    import wave
    buf = io.BytesIO()
    with wave.open(buf, "wb") as w:  # stereo 16-bit, 8 kHz
        w.setnchannels(2)
        w.setsampwidth(2)
        w.setframerate(8000)
        w.writeframes(b"".join(struct.pack("<hh", 16384, 16384) for _ in range(400)))
    tok = ByteTokenizer()
    runner = EngineRunner(FakeEngine(), tok)
    with TestClient(create_app(runner, tok, "fake", transcriber=_FakeTranscriber())) as c:
        r = c.post("/v1/audio/transcriptions", files={"file": ("a.wav", buf.getvalue(), "audio/wav")})
        assert r.status_code == 200 and r.json()["text"] == "400 samples at 8000 Hz, peak 0.50"
        bad = c.post("/v1/audio/transcriptions", files={"file": ("a.wav", b"not audio", "audio/wav")})
        assert bad.status_code == 400
    runner.shutdown()


def test_logprobs_completion_chat_and_stream(client):
    c, _ = client
    r = c.post("/v1/completions", json={"prompt": "a", "max_tokens": 3, "logprobs": 1})
    lp = r.json()["choices"][0]["logprobs"]
    assert lp["tokens"] == ["b", "c", "d"] and lp["token_logprobs"] == [-0.5, -1.0, -1.5]
    assert lp["text_offset"] == [0, 1, 2]
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "a"}], "max_tokens": 2,
                                             "logprobs": True})
    content = r.json()["choices"][0]["logprobs"]["content"]
    assert [e["logprob"] for e in content] == [-0.5, -1.0]
    with c.stream("POST", "/v1/completions", json={"prompt": "a", "max_tokens": 3, "stream": True,
                                                    "logprobs": 1}) as s:
        lines = [ln for ln in s.iter_lines() if ln]
    chunks = [json.loads(ln[6:]) for ln in lines[:-1]]
    got = [ch["choices"][0]["logprobs"]["token_logprobs"][0] for ch in chunks if ch["choices"][0]["logprobs"]]
    assert len(got) == 3 and got[-1] == -1.5
    r = c.post("/v1/completions", json={"prompt": "a", "max_tokens": 2})
    assert r.json()["choices"][0]["logprobs"] is None
