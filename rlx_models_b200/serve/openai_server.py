"""OpenAI-compatible HTTP server with continuous batching and SSE streaming.

    python -m rlx_models_b200 serve --model qwen3-0.6b --port 8000

Endpoints: ``GET /health``, ``GET /v1/models``, ``GET /metrics``
(Prometheus text), ``POST /v1/completions``, ``POST /v1/chat/completions``,
``POST /v1/embeddings`` (when the server was given an embedder),
``POST /v1/audio/transcriptions`` (multipart WAV upload, when it was given a
transcriber).
Prompts may be text (tokenised with the checkpoint's tokenizer, or bytes
for random-weight shapes) or token-id arrays. Sampling fields: ``max_tokens``,
``temperature``, ``top_p``, ``top_k``, ``min_p``, ``seed``, ``stop`` (strings),
``stop_token_ids``, ``ignore_eos``, ``logprobs``; ``stream: true`` answers
with ``text/event-stream`` chunks and a final ``data: [DONE]``. Every request
joins the same continuous batch (``serve.runner.EngineRunner``).

Reference: rlx-openai (OpenAI route shapes, SSE framing) and rlx-serve
src/engine.rs, src/backend.rs:116-167 (stop strings).
"""
from __future__ import annotations

import torch

import json
import time
import uuid

from ..runtime.engine import SamplingParams
from .runner import EngineRunner


# llama.cpp-style sampler fields accepted on the request body
_EXTRA_SAMPLING = ("typical_p", "xtc_threshold", "xtc_probability", "dry_multiplier", "dry_base",
                   "dry_allowed_length", "dry_penalty_last_n", "mirostat", "mirostat_tau", "mirostat_eta")


def _params(body: dict, eos: int | None) -> tuple[SamplingParams, list[str]]:
    stop = body.get("stop") or []
    if isinstance(stop, str):
        stop = [stop]
    stop_ids = list(body.get("stop_token_ids") or [])
    if eos is not None and not body.get("ignore_eos", False):
        stop_ids.append(int(eos))
    sp = SamplingParams(max_new_tokens=int(body.get("max_tokens") or 16),
                        temperature=float(body.get("temperature", 1.0) if body.get("temperature") is not None else 1.0),
                        top_k=int(body.get("top_k") or 0), top_p=float(body.get("top_p") or 1.0),
                        min_p=float(body.get("min_p") or 0.0), seed=int(body.get("seed") or 0),
                        ignore_eos=bool(body.get("ignore_eos", False)), stop_token_ids=stop_ids,
                        logprobs=bool(body.get("logprobs")),
                        repetition_penalty=float(body.get("repetition_penalty") or 1.0),
                        frequency_penalty=float(body.get("frequency_penalty") or 0.0),
                        presence_penalty=float(body.get("presence_penalty") or 0.0),
                        logit_bias={int(k): float(v) for k, v in (body.get("logit_bias") or {}).items()} or None,
                        **{k: type(getattr(SamplingParams, k))(body[k]) for k in _EXTRA_SAMPLING if k in body})
    return sp, list(stop)


def decode_wav(data: bytes) -> tuple[torch.Tensor, int]:
    """PCM WAV bytes (8 / 16 / 32-bit integer, any channel count) -> (mono fp32
    samples in [-1, 1], sample rate)."""
    import io
    import wave
    with wave.open(io.BytesIO(data)) as w:
        ch, width, sr, n = w.getnchannels(), w.getsampwidth(), w.getframerate(), w.getnframes()
        raw = w.readframes(n)
    if width == 1:
        x = torch.frombuffer(bytearray(raw), dtype=torch.uint8).float().sub_(128.0).div_(128.0)
    elif width == 2:
        x = torch.frombuffer(bytearray(raw), dtype=torch.int16).float().div_(32768.0)
    elif width == 4:
        x = torch.frombuffer(bytearray(raw), dtype=torch.int32).float().div_(2147483648.0)
    else:
        raise ValueError(f"unsupported WAV sample width {width}")
    return x.view(-1, ch).mean(1), sr


def create_app(runner: EngineRunner, tokenizer, model_name: str = "b200-model", embedder=None, transcriber=None):
    """``embedder``: any object with ``embed(inputs) -> [N, D]`` over a list of
    strings or of token-id lists (``api.load_embedder``, ``LLM.embed``);
    ``transcriber``: any object with ``transcribe(samples, sample_rate) -> str``
    (``api.load_transcriber``)."""
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse
    from prometheus_client import CollectorRegistry, Counter, Histogram, generate_latest

    app = FastAPI(title="rlx_models_b200 OpenAI server")
    reg = CollectorRegistry()
    m_req = Counter("b200_requests_total", "requests", ["route"], registry=reg)
    m_tok = Counter("b200_generated_tokens_total", "generated tokens", registry=reg)
    m_ttft = Histogram("b200_ttft_seconds", "time to first token", registry=reg,
                       buckets=(0.01, 0.05, 0.1, 0.25, 0.5, 1, 2, 5, 10, 30))
    eos = getattr(tokenizer, "eos_token_id", None)

    def encode_prompt(p):
        if isinstance(p, list) and p and isinstance(p[0], int):
            return list(p)
        if isinstance(p, list):
            p = p[0] if p else ""
        if not isinstance(p, str):
            raise HTTPException(400, "prompt must be a string or an array of token ids")
        return tokenizer.encode(p)

    def run(ids, body, kind, route_id, created):
        sp, stop = _params(body, eos)
        t0 = time.perf_counter()
        h = runner.submit(ids, sp, stop)
        first = [None]

        def events():
            toks, lps = [], []
            for ev in h.events():
                if ev[0] == "token":
                    if first[0] is None:
                        first[0] = time.perf_counter()
                        m_ttft.observe(first[0] - t0)
                    toks.append(ev[1])
                    lps.append(ev[2] if len(ev) > 2 else None)
                    m_tok.inc()
                    yield "token", ev[1], toks, lps
                elif ev[0] == "error":
                    raise HTTPException(500, ev[1])
                else:
                    out = ev[1]
                    reason = h.finish_reason or (out.finish_reason if out is not None else "stop")
                    final = getattr(out, "logprobs", None) if out is not None else None
                    if final:
                        lps[:] = list(final[:len(toks)])
                    yield "done", reason, toks, lps
        return events()

    def logprobs_of(kind, toks, lps):
        """OpenAI ``logprobs`` object of the sampled tokens (no alternatives):
        completions: tokens / token_logprobs / text_offset; chat: content[]."""
        pieces = [tokenizer.decode([t]) for t in toks]
        vals = [None if v is None else float(v) for v in lps[:len(toks)]]
        if kind == "chat":
            return {"content": [{"token": p, "logprob": v, "bytes": list(p.encode("utf-8")), "top_logprobs": []}
                                for p, v in zip(pieces, vals)]}
        offs, o = [], 0
        for p in pieces:
            offs.append(o)
            o += len(p)
        return {"tokens": pieces, "token_logprobs": vals, "top_logprobs": None, "text_offset": offs}

    def text_of(toks, stop):
        s = tokenizer.decode(toks)
        for st in stop:
            if st and st in s:
                s = s[:s.index(st)]
        return s

    def choice(kind, text, reason, idx=0, delta=False, logprobs=None):
        if kind == "chat":
            key = "delta" if delta else "message"
            ch = {"index": idx, key: ({"role": "assistant", "content": text}), "finish_reason": reason}
            if logprobs is not None:
                ch["logprobs"] = logprobs
            return ch
        return {"index": idx, "text": text, "finish_reason": reason, "logprobs": logprobs}

    def respond(body, ids, kind):
        rid = ("chatcmpl-" if kind == "chat" else "cmpl-") + uuid.uuid4().hex[:24]
        created = int(time.time())
        obj = "chat.completion" if kind == "chat" else "text_completion"
        stop = body.get("stop") or []
        stop = [stop] if isinstance(stop, str) else list(stop)
        evs = run(ids, body, kind, rid, created)
        want_lp = bool(body.get("logprobs"))
        if body.get("stream"):
            def sse():
                sent = ""
                for typ, val, toks, lps in evs:
                    if typ == "token":
                        cur = text_of(toks, stop)
                        piece, sent = cur[len(sent):], cur
                        if piece or want_lp:
                            lp = logprobs_of(kind, toks[-1:], lps[-1:]) if want_lp else None
                            chunk = {"id": rid, "object": obj + ".chunk", "created": created, "model": model_name,
                                     "choices": [choice(kind, piece, None, delta=True, logprobs=lp)]}
                            yield f"data: {json.dumps(chunk)}\n\n"
                    else:
                        chunk = {"id": rid, "object": obj + ".chunk", "created": created, "model": model_name,
                                 "choices": [choice(kind, "", val, delta=True)],
                                 "usage": {"prompt_tokens": len(ids), "completion_tokens": len(toks),
                                           "total_tokens": len(ids) + len(toks)}}
                        yield f"data: {json.dumps(chunk)}\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(sse(), media_type="text/event-stream")
        toks, lps, reason = [], [], "stop"
        for typ, val, tk, lp in evs:
            toks, lps = tk, lp
            if typ == "done":
                reason = val
        text = text_of(toks, stop)
        ch = choice(kind, text, reason, logprobs=logprobs_of(kind, toks, lps) if want_lp else None)
        tools = body.get("tools") or []
        if kind == "chat" and tools:
            # tool calls in the text: validated and sanitised against the request's tools
            from .tool_calls import parse, to_openai
            calls, rest = parse(text)
            if calls:
                good, errors = to_openai(calls, tools)
                if good:
                    ch["message"] = {"role": "assistant", "content": rest or None, "tool_calls": good}
                    ch["finish_reason"] = "tool_calls"
                if errors:
                    ch["guardrail_errors"] = errors
        res = {"id": rid, "object": obj, "created": created, "model": model_name,
               "choices": [ch],
               "usage": {"prompt_tokens": len(ids), "completion_tokens": len(toks),
                         "total_tokens": len(ids) + len(toks)}}
        if kind != "chat":
            res["choices"][0]["token_ids"] = toks
        return JSONResponse(res)

    @app.get("/health")
    def health():
        return {"status": "ok"}

    @app.get("/v1/models")
    def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "rlx_models_b200"}]}

    @app.get("/metrics")
    def metrics():
        return PlainTextResponse(generate_latest(reg).decode())

    @app.post("/v1/completions")
    def completions(body: dict):
        m_req.labels("completions").inc()
        if int(body.get("n", 1)) != 1:
            raise HTTPException(400, "n > 1 is not supported")
        return respond(body, encode_prompt(body.get("prompt", "")), "text")

    @app.post("/v1/embeddings")
    def embeddings(body: dict):
        m_req.labels("embeddings").inc()
        if embedder is None:
            raise HTTPException(404, "this server has no embedding model")
        inp = body.get("input")
        if inp is None or inp == [] or inp == "":
            raise HTTPException(400, "input required")
        if isinstance(inp, str) or (isinstance(inp, list) and inp and isinstance(inp[0], int)):
            inp = [inp]  # one text or one token-id list
        vecs = embedder.embed(list(inp))
        n_tok = sum(len(x) if isinstance(x, list) else len(tokenizer.encode(x)) for x in inp)
        data = [{"object": "embedding", "index": i, "embedding": [float(v) for v in vec]}
                for i, vec in enumerate(vecs.float().cpu())]
        return {"object": "list", "data": data, "model": body.get("model", model_name),
                "usage": {"prompt_tokens": n_tok, "total_tokens": n_tok}}

    if transcriber is not None:
        from fastapi import File, UploadFile

        async def transcriptions(file=File(...)):
            m_req.labels("transcriptions").inc()
            try:
                audio, sr = decode_wav(await file.read())
            except Exception as e:  # not a PCM WAV file
                raise HTTPException(400, f"could not read the audio: {e}")
            return {"text": transcriber.transcribe(audio, sr)}

        # a real type object (not a postponed string) so that FastAPI reads it as an upload
        transcriptions.__annotations__ = {"file": UploadFile}
        app.post("/v1/audio/transcriptions")(transcriptions)

    @app.post("/v1/chat/completions")
    def chat(body: dict):
        m_req.labels("chat").inc()
        msgs = body.get("messages") or []
        if not msgs:
            raise HTTPException(400, "messages required")
        budget = body.get("max_context_tokens")
        if budget:  # keep the conversation inside a token budget (system messages stay)
            from .guardrails import compact_messages
            msgs = compact_messages(msgs, int(budget), tokenizer)
        tools = body.get("tools") or None
        try:
            text = tokenizer.apply_chat_template(msgs, add_generation_prompt=True, tokenize=False, tools=tools)
        except TypeError:  # a template helper without tool support
            text = tokenizer.apply_chat_template(msgs, add_generation_prompt=True, tokenize=False)
        return respond(body, tokenizer.encode(text), "chat")

    return app


def serve(llm, host: str = "127.0.0.1", port: int = 8000, model_name: str = "b200-model", embedder=None,
          transcriber=None):
    import uvicorn

    from ..tokenizer import ByteTokenizer
    tok = llm.tokenizer or ByteTokenizer()
    runner = EngineRunner(llm.engine, tok)
    app = create_app(runner, tok, model_name, embedder=embedder, transcriber=transcriber)
    try:
        uvicorn.run(app, host=host, port=port, log_level="info")
    finally:
        runner.shutdown()
