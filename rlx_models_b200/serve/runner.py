"""Engine thread for concurrent clients.

``EngineRunner`` owns an engine (anything with ``add_request`` / ``step`` /
``has_unfinished`` / ``abort`` / ``requests``, i.e. ``runtime.engine.LLMEngine``)
on one background thread, so every client's request joins the same
continuous batch. ``submit`` returns a ``RequestHandle`` whose ``events()``
yields ``("token", id, logprob)`` as tokens appear (logprob None unless the
request asked for log-probabilities) and finally ``("done", output)``.
Stop strings are matched on the incrementally decoded text; a match aborts
the request in the engine.

Reference: rlx-serve src/engine.rs (request queue feeding the batching
loop, per-request channels), src/backend.rs (stop handling).
"""
from __future__ import annotations

import queue
import threading
import time
from dataclasses import dataclass, field


@dataclass
class RequestHandle:
    rid: int
    q: "queue.Queue" = field(default_factory=queue.Queue)
    stop: list = field(default_factory=list)
    text: str = ""
    finish_reason: str | None = None

    def events(self, timeout: float = 600.0):
        while True:
            ev = self.q.get(timeout=timeout)
            yield ev
            if ev[0] == "done":
                return


class EngineRunner:
    def __init__(self, engine, tokenizer=None, idle_sleep: float = 0.002):
        self.engine, self.tok = engine, tokenizer
        self._in: "queue.Queue" = queue.Queue()
        self._live: dict[int, tuple[RequestHandle, int]] = {}  # engine sid -> (handle, tokens sent)
        self._stop = threading.Event()
        self._wake = threading.Event()
        self._next = 0
        self._lock = threading.Lock()
        self.stats = dict(requests=0, tokens=0, aborted_by_stop=0)
        self._t = threading.Thread(target=self._loop, name="b200-engine", daemon=True)
        self._t.start()

    def submit(self, prompt_ids: list[int], params, stop: list[str] | None = None) -> RequestHandle:
        with self._lock:
            self._next += 1
            h = RequestHandle(self._next, stop=list(stop or []))
        self._in.put((h, prompt_ids, params))
        self._wake.set()
        return h

    def shutdown(self):
        self._stop.set()
        self._wake.set()
        self._t.join(timeout=10)

    # -- engine thread ---------------------------------------------------------
    def _admit(self):
        while True:
            try:
                h, ids, params = self._in.get_nowait()
            except queue.Empty:
                return
            sid = self.engine.add_request(ids, params)
            self._live[sid] = (h, 0)
            self.stats["requests"] += 1

    def _emit(self, sid, toks, final=None, lps=None):
        h, sent = self._live[sid]
        for i, t in enumerate(toks[sent:], start=sent):
            h.q.put(("token", t, lps[i] if lps is not None and i < len(lps) else None))
            self.stats["tokens"] += 1
            if h.stop and self.tok is not None:
                h.text += self.tok.decode([t])
                if any(s and s in h.text for s in h.stop):
                    h.finish_reason = "stop"
        self._live[sid] = (h, len(toks))
        if final is not None:
            h.q.put(("done", final))
            del self._live[sid]
        elif h.finish_reason == "stop":
            self.engine.abort(sid)
            self.stats["aborted_by_stop"] += 1
            h.q.put(("done", None))
            del self._live[sid]

    def _loop(self):
        while not self._stop.is_set():
            self._admit()
            if not self.engine.has_unfinished():
                self._wake.wait(0.05)
                self._wake.clear()
                continue
            try:
                done = {o.seq_id: o for o in self.engine.step()}
            except Exception as e:  # surface to every waiting client, keep serving
                for sid in list(self._live):
                    h, _ = self._live.pop(sid)
                    h.q.put(("error", repr(e)))
                    h.q.put(("done", None))
                continue
            for sid in list(self._live):
                if sid in done:
                    self._emit(sid, done[sid].token_ids, final=done[sid],
                               lps=getattr(done[sid], "logprobs", None))
                else:
                    st = self.engine.requests.get(sid)
                    if st is not None:
                        self._emit(sid, st.tokens, lps=getattr(st, "logprobs", None) or None)
