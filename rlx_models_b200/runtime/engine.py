"""LLM engine: native scheduler + paged KV + model runner with CUDA graphs.

Step loop (the B200 counterpart of rlx-serve's `BatchedEngine` /
`scheduler_loop`, src/batch.rs:567-640, and `FusedBatchRunner::forward_batch`,
src/batch.rs:262-360):

1. the C++ scheduler (``_runtime.Scheduler``) picks decode tokens and prefill
   chunks under the token budget and writes the flat batch into pinned host
   staging buffers;
2. one non-blocking host->device copy per field;
3. decode-only steps replay a CUDA graph captured for the padded batch size
   (model forward + on-GPU sampling in one graph); mixed / prefill steps run
   eagerly;
4. only the sampled token ids come back to the host; the scheduler appends
   them and retires finished sequences.

Overlapped scheduling (``EngineConfig.async_scheduling``, the default): step
n+1 is scheduled and launched before step n's tokens are read back. The
scheduler appends a placeholder for every sampled row; decode rows fed by a
placeholder carry the previous step's logit row in ``tok_src`` and a small
kernel (``ops.forward_tokens``, the first launch of every step) copies the
sampled ids on the device. Host staging and the token read-back buffers are
double-buffered by step parity; the host waits for step n's event only after
step n+1 is queued, so scheduling, staging and Python bookkeeping run while
the GPU computes. Requests that need the host between steps (penalties,
host-side logit processors) and pipeline stages fall back to the synchronous
loop.

Every launch in a step is one of this package's kernels (GEMM, attention,
norm/RoPE, sampling) except for small torch copies/index ops.
"""
from __future__ import annotations

import collections
import dataclasses
import json

import time
from dataclasses import dataclass, field

import torch

from .. import ops
from ..utils.trace import nvtx
from ..models.decoder import ForwardBatch
from .kv_cache import BLOCK_SIZE

try:
    from .. import _runtime  # type: ignore
except Exception as e:  # pragma: no cover
    _runtime = None
    _RT_ERR = e


@dataclass
class SamplingParams:
    max_new_tokens: int = 16
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    min_p: float = 0.0
    seed: int = 0
    ignore_eos: bool = False
    stop_token_ids: list[int] = field(default_factory=list)
    logprobs: bool = False
    # penalties (applied on the GPU before selection; such rows take the eager path):
    # repetition (HF / CTRL: over prompt + output), frequency and presence (OpenAI: output only)
    repetition_penalty: float = 1.0
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0
    logit_bias: dict | None = None
    # host-side logit processors (runtime/samplers.py), also eager-path only
    typical_p: float = 1.0
    xtc_threshold: float = 0.1
    xtc_probability: float = 0.0
    dry_multiplier: float = 0.0
    dry_base: float = 1.75
    dry_allowed_length: int = 2
    dry_penalty_last_n: int = -1
    mirostat: int = 0          # 2: Mirostat v2
    mirostat_tau: float = 5.0
    mirostat_eta: float = 0.1

    @property
    def penalised(self) -> bool:
        return (self.repetition_penalty != 1.0 or self.frequency_penalty != 0.0 or self.presence_penalty != 0.0
                or bool(self.logit_bias))

    @property
    def processed(self) -> bool:
        from .samplers import needs_processing
        return needs_processing(self)


@dataclass
class EngineConfig:
    max_num_seqs: int = 256
    max_batched_tokens: int = 8192
    chunk_size: int = 0
    max_model_len: int = 4096
    num_blocks: int = 0            # 0: size from kv_memory_gb
    kv_memory_gb: float = 16.0
    prefix_caching: bool = True
    cuda_graphs: bool = True
    graph_batch_sizes: tuple = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 192, 256)
    eos_token_id: int = -1
    # long-context decode over retrieved KV blocks, e.g. {"topk_blocks": 64,
    # "window_blocks": 16, "sink_blocks": 1} (runtime/kv_retrieval.py); None = full attention
    kv_retrieval: dict | None = None
    # "bf16", or "fp8": float8 e4m3 pages holding value / scale with scales (k, v) (the
    # decode kernel reads them directly; prefill reads bf16 copies of its pages)
    kv_cache_dtype: str = "bf16"
    kv_cache_scales: tuple = (1.0, 1.0)
    # schedule / launch step n+1 before step n's tokens come back (see module docstring)
    async_scheduling: bool = True
    # per-step metrics as JSON lines (step kind, tokens, batch occupancy, KV blocks in use,
    # host launch / wait time, device time); None = off. ``LLMEngine.step_log`` keeps the last 4096.
    metrics_path: str | None = None


@dataclass
class RequestState:
    seq_id: int
    prompt_len: int
    params: SamplingParams
    arrival: float
    first_token: float | None = None
    finish: float | None = None
    token_times: list[float] = field(default_factory=list)
    tokens: list[int] = field(default_factory=list)
    logprobs: list[float] = field(default_factory=list)
    finish_reason: str | None = None
    prompt: list[int] | None = None     # kept for the repetition penalty and DRY
    out_counts: dict | None = None      # token -> count of generated tokens (penalised requests)
    rng: object = None                  # XTC coin flips
    mirostat_mu: float | None = None
    mirostat_lp2: object = None
    n_sched: int = 0                    # sampled rows scheduled so far (the sampler's stream offset)
    mm: list | None = None              # [(first prompt position, [n, H] input embeddings)] (images)


@dataclass
class RequestOutput:
    seq_id: int
    prompt_len: int
    token_ids: list[int]
    finish_reason: str
    ttft: float
    tpot: float
    latency: float
    cached_prompt_tokens: int = 0
    logprobs: list[float] | None = None


_REASONS = {1: "length", 2: "stop", 3: "abort"}


class LLMEngine:
    def __init__(self, model, config: EngineConfig | None = None):
        if _runtime is None:
            raise RuntimeError(f"rlx_models_b200._runtime not built: {_RT_ERR}")
        self.model = model
        self.cfg = cfg = config or EngineConfig()
        self.device = model.device
        mc = model.cfg
        lim = getattr(model, "max_context", None)
        if lim and cfg.max_model_len > lim:
            raise ValueError(f"{type(model).__name__}: max_model_len {cfg.max_model_len} > {lim}, the context this "
                             "model's kernels run exactly (e.g. Llama-4's chunked attention starts there)")
        self.max_blocks_per_seq = (cfg.max_model_len + BLOCK_SIZE - 1) // BLOCK_SIZE
        if cfg.kv_cache_dtype != "bf16" or hasattr(model, "set_kv_cache_dtype"):
            if not hasattr(model, "set_kv_cache_dtype"):
                raise NotImplementedError(f"{type(model).__name__}: kv_cache_dtype {cfg.kv_cache_dtype!r}")
            model.set_kv_cache_dtype(cfg.kv_cache_dtype, cfg.kv_cache_scales)
        nb = cfg.num_blocks
        if nb <= 0:
            per = (model.kv_bytes_per_block() if hasattr(model, "kv_bytes_per_block")
                   else 2 * mc.num_hidden_layers * model.hkv * BLOCK_SIZE * model.D * 2)
            nb = max(self.max_blocks_per_seq + 1, int(cfg.kv_memory_gb * (1 << 30)) // per)
        self.stateful = bool(getattr(model, "stateful", False))
        if self.stateful:
            # recurrent per-sequence state (hybrid linear-attention models): one slot per
            # running sequence; a cached KV prefix would not restore that state
            cfg = self.cfg = dataclasses.replace(cfg, prefix_caching=False)
            self.kv = model.make_kv_cache(nb + 1, num_slots=cfg.max_num_seqs)
            self.free_slots = list(range(cfg.max_num_seqs - 1, -1, -1))
            self.slot_of: dict[int, int] = {}
        else:
            self.kv = model.make_kv_cache(nb + 1)
        if cfg.kv_retrieval:
            if not hasattr(model, "enable_kv_retrieval"):
                raise NotImplementedError(f"{type(model).__name__} has no KV retrieval")
            model.enable_kv_retrieval(nb + 1, **cfg.kv_retrieval)
        self.dummy_block = nb  # never handed out by the scheduler; padding rows write here
        self.sched = _runtime.Scheduler(nb, cfg.max_num_seqs, cfg.max_batched_tokens, self.max_blocks_per_seq,
                                        cfg.prefix_caching, cfg.chunk_size)
        T, S, W = cfg.max_batched_tokens, cfg.max_num_seqs, self.max_blocks_per_seq
        pin = dict(pin_memory=True)
        i32, i64 = torch.int32, torch.int64

        def staging():
            return dict(
                input_ids=torch.zeros(T, dtype=i32, **pin), positions=torch.zeros(T, dtype=i32, **pin),
                slots=torch.zeros(T, dtype=i64, **pin), dec_tables=torch.zeros(S, W, dtype=i32, **pin),
                dec_ctx=torch.zeros(S, dtype=i32, **pin), pre_tables=torch.zeros(S, W, dtype=i32, **pin),
                pre_ctx=torch.zeros(S, dtype=i32, **pin), pre_cu=torch.zeros(S + 1, dtype=i32, **pin),
                logit_rows=torch.zeros(T, dtype=i64, **pin), sample_ids=torch.zeros(T, dtype=i64, **pin),
                seq_slots=torch.full((S,), -1, dtype=i32, **pin), tok_src=torch.full((T,), -1, dtype=i32, **pin))

        # host staging, double-buffered by step parity: step n+1 is written while
        # step n's host->device copies may still be queued
        self._hs = [staging(), staging()]
        self._hb = 0
        self.h = self._hs[0]
        dev = self.device
        self.d = {k: torch.zeros_like(v, device=dev) for k, v in self.h.items() if k != "sample_ids"}
        self.d["tok_src"].fill_(-1)
        # per-row sampling parameters (host pinned -> device)
        self.hp = dict(temp=torch.zeros(T, **pin), top_k=torch.zeros(T, dtype=i32, **pin),
                       top_p=torch.ones(T, **pin), min_p=torch.zeros(T, **pin),
                       seed=torch.zeros(T, dtype=i64, **pin), offset=torch.zeros(T, dtype=i64, **pin))
        self.dp = {k: torch.zeros_like(v, device=dev) for k, v in self.hp.items()}
        self.tok_out = torch.zeros(T, dtype=i32, device=dev)
        self.logprob_out = torch.zeros(T, dtype=torch.float32, device=dev)
        self._tok_hosts = [torch.zeros(T, dtype=i32, pin_memory=True) for _ in range(2)]
        self._lp_hosts = [torch.zeros(T, dtype=torch.float32, pin_memory=True) for _ in range(2)]
        self.tok_host = self._tok_hosts[0]
        self.requests: dict[int, RequestState] = {}
        self._n_nongreedy = 0   # active requests that sample or want logprobs
        self._n_host_rows = 0   # active requests that need the host between steps (penalties, processors)
        self._n_mm = 0          # active requests with input embeddings (images)
        self._inflight = None
        self.graphs: dict[int, tuple] = {}
        self._graph_pool = None
        self.stats = dict(steps=0, graph_steps=0, eager_steps=0, tokens=0, h2d_bytes=0, d2h_bytes=0,
                          overlapped_steps=0)
        self.copy_stream = torch.cuda.current_stream(dev)
        self.step_log = collections.deque(maxlen=4096)
        self._metrics_f = open(cfg.metrics_path, "a") if cfg.metrics_path else None
        self._nblocks = nb

    # -- requests --------------------------------------------------------------
    def add_request(self, prompt: list[int], params: SamplingParams | None = None, mm: list | None = None) -> int:
        """Queue a request. ``mm``: [(position, embeds [n, H])] input embeddings that
        replace the token embeddings of prompt positions position .. position + n - 1
        (image tokens of a vision-language model)."""
        params = params or SamplingParams()
        if mm:
            if self.cfg.prefix_caching:
                raise ValueError("requests with input embeddings need prefix_caching=False "
                                 "(equal placeholder ids would share cached KV across images)")
            for p0, e in mm:
                if p0 < 0 or p0 + e.shape[0] > len(prompt):
                    raise ValueError(f"embeddings at {p0}..{p0 + e.shape[0]} outside the {len(prompt)}-token prompt")
        sid = self.sched.add_request(list(map(int, prompt)), int(params.max_new_tokens), bool(params.ignore_eos),
                                     list(params.stop_token_ids))
        st = RequestState(sid, len(prompt), params, time.perf_counter())
        if mm:
            st.mm = [(int(p0), e.to(self.device)) for p0, e in mm]
            self._n_mm += 1
        if params.penalised or params.processed:
            st.out_counts = {}
            if params.repetition_penalty != 1.0 or params.dry_multiplier > 0:
                st.prompt = list(map(int, prompt))
        self.requests[sid] = st
        self._track(st, +1)
        return sid

    def _track(self, st: RequestState, d: int):
        p = st.params
        if p.temperature > 0 or p.logprobs:
            self._n_nongreedy += d
        if st.out_counts is not None:
            self._n_host_rows += d

    def _retire(self, sid: int) -> RequestState | None:
        st = self.requests.pop(sid, None)
        if st is not None:
            self._track(st, -1)
            if st.mm is not None:
                st.mm = None
                self._n_mm -= 1
        self._free_slot(sid)
        return st

    def abort(self, sid: int):
        self.sched.abort(sid)
        self._retire(sid)

    def _free_slot(self, sid: int):
        if self.stateful and sid in self.slot_of:
            self.free_slots.append(self.slot_of.pop(sid))

    def _assign_slots(self) -> int:
        """State slot of every sequence of the step (batch order) into the staging buffer."""
        ids = self.sched.step_seq_ids()
        hs = self.h["seq_slots"]
        for i, sid in enumerate(ids):
            slot = self.slot_of.get(sid)
            if slot is None:
                slot = self.slot_of[sid] = self.free_slots.pop()
            hs[i] = slot
        return len(ids)

    def has_unfinished(self) -> bool:
        return self.sched.has_work() or self._inflight is not None

    # -- model step ------------------------------------------------------------
    def _params_rows(self, sids: list[int]) -> bool:
        """Advance each row's sampler offset and, unless every active request is
        greedy without logprobs (returns True then), fill the per-row sampling
        parameters with one pinned write per field."""
        reqs = self.requests
        sts = [reqs[sid] for sid in sids]
        offs = [st.n_sched for st in sts]
        for st in sts:
            st.n_sched += 1
        if self._n_nongreedy == 0:
            return True
        ps = [st.params for st in sts]
        if not any(p.temperature > 0 or p.logprobs for p in ps):
            return True
        R = len(sids)
        hp = self.hp
        hp["temp"][:R] = torch.tensor([p.temperature for p in ps], dtype=torch.float32)
        hp["top_k"][:R] = torch.tensor([p.top_k for p in ps], dtype=torch.int32)
        hp["top_p"][:R] = torch.tensor([p.top_p for p in ps], dtype=torch.float32)
        hp["min_p"][:R] = torch.tensor([p.min_p for p in ps], dtype=torch.float32)
        hp["seed"][:R] = torch.tensor([p.seed * 1000003 + sid for p, sid in zip(ps, sids)], dtype=torch.int64)
        hp["offset"][:R] = torch.tensor(offs, dtype=torch.int64)
        return False

    def _penalty_rows(self, sids: list[int]):
        """Per-row penalty tables for ops.apply_penalties (None when no row of
        the step is penalised): output tokens with their counts, plus prompt
        tokens at count 0 when the repetition penalty is on."""
        rows, any_pen = [], False
        for sid in sids:
            st = self.requests[sid]
            p = st.params
            if st.out_counts is None:
                rows.append(None)
                continue
            any_pen = True
            if not p.penalised:
                rows.append(None)
                continue
            counts = st.out_counts
            if st.prompt and p.repetition_penalty != 1.0:
                counts = dict.fromkeys(st.prompt, 0)
                counts.update(st.out_counts)
            rows.append((counts, p.repetition_penalty, p.frequency_penalty, p.presence_penalty, p.logit_bias))
        return rows if any_pen else None

    def _sample(self, logits: torch.Tensor, R: int, greedy: bool, pen=None):
        out = self.tok_out[:R]
        comm = getattr(self.model, "comm", None)
        if comm is not None and getattr(self.model, "tp_size", 1) > 1:
            # vocab-parallel logits: every rank must pick the same tokens
            if greedy and pen is None:
                return comm.greedy(logits, out)
            logits = comm.gather_logits(logits)
        if pen is not None:
            logits = logits.float() if logits.dtype != torch.float32 else logits
            if any(r is not None for r in pen):
                ops.apply_penalties(logits, pen)
            from .samplers import process_row
            for r, sid in enumerate(self._step_sids[:R]):
                st = self.requests[sid]
                if st.params.processed:
                    process_row(logits[r], st.params, st, (st.prompt or []) + st.tokens)
        if greedy:
            ops.argmax(logits, out=out)
        else:
            for k in self.hp:
                self.dp[k][:R].copy_(self.hp[k][:R], non_blocking=True)
            ops.sample(logits, self.dp["temp"][:R], self.dp["top_k"][:R], self.dp["top_p"][:R],
                       self.dp["min_p"][:R], self.dp["seed"][:R], self.dp["offset"][:R], out=out,
                       logprob=self.logprob_out[:R])
        return out

    def _copy_in(self, keys_rows: dict[str, int]):
        for k, n in keys_rows.items():
            if n > 0:
                src = self.h[k][:n]
                self.d[k][:n].copy_(src, non_blocking=True)
                self.stats["h2d_bytes"] += src.numel() * src.element_size()

    def _eager_forward(self, T: int, nd: int, npf: int, max_q: int, R: int) -> torch.Tensor:
        d = self.d
        self._copy_in(dict(input_ids=T, positions=T, slots=T, dec_tables=nd, dec_ctx=nd, pre_tables=npf,
                           pre_ctx=npf, pre_cu=npf + 1 if npf else 0, logit_rows=R,
                           seq_slots=nd + npf if self.stateful else 0, tok_src=nd))
        if nd:  # decode inputs still being sampled by the previous step
            ops.forward_tokens(d["input_ids"][:nd], d["tok_src"][:nd], self.tok_out)
        fb = ForwardBatch(
            input_ids=d["input_ids"][:T], positions=d["positions"][:T], slots=d["slots"][:T], num_decode=nd,
            dec_block_tables=d["dec_tables"][:nd] if nd else None, dec_ctx_lens=d["dec_ctx"][:nd] if nd else None,
            pre_block_tables=d["pre_tables"][:npf] if npf else None,
            pre_ctx_lens=d["pre_ctx"][:npf] if npf else None, pre_cu_q=d["pre_cu"][:npf + 1] if npf else None,
            pre_max_q=max_q, logit_rows=d["logit_rows"][:R],
            seq_slots=d["seq_slots"][:nd + npf] if self.stateful else None,
            pre_cu_host=self.h["pre_cu"][:npf + 1].tolist() if npf else None)
        if npf and self._n_mm:
            fb.mm_rows, fb.mm_embeds = self._mm_rows(nd, npf)
        return self.model.forward(fb, self.kv)

    def _mm_rows(self, nd: int, npf: int):
        """Rows of this step's prefill tokens whose input embeddings a request
        supplies (images), and those embeddings; (None, None) when there are none."""
        sids = self.sched.step_seq_ids()[nd:nd + npf]
        cu, ctx = self.h["pre_cu"][:npf + 1].tolist(), self.h["pre_ctx"][:npf].tolist()
        rows, embs = [], []
        for j, sid in enumerate(sids):
            st = self.requests.get(sid)
            if st is None or st.mm is None:
                continue
            n = cu[j + 1] - cu[j]
            p_lo = ctx[j] - n  # prompt position of this chunk's first row
            for p0, e in st.mm:
                a, b = max(p0, p_lo), min(p0 + e.shape[0], ctx[j])
                if a < b:
                    rows.append(torch.arange(nd + cu[j] + a - p_lo, nd + cu[j] + b - p_lo))
                    embs.append(e[a - p0:b - p0])
        if not rows:
            return None, None
        return torch.cat(rows).to(self.device), torch.cat(embs)

    def _bucket(self, n: int) -> int | None:
        for b in self.cfg.graph_batch_sizes:
            if b >= n and b <= self.cfg.max_num_seqs:
                return b
        return None

    def _pad_decode_rows(self, nd: int, B: int):
        if nd == B:
            return
        h = self.h
        db = self.dummy_block
        h["input_ids"][nd:B] = 0
        h["positions"][nd:B] = 0
        h["slots"][nd:B] = db * BLOCK_SIZE
        h["dec_tables"][nd:B] = db
        h["dec_ctx"][nd:B] = 1
        h["tok_src"][nd:B] = -1
        h["seq_slots"][nd:B] = -1  # no state slot: the recurrent kernels skip these rows

    def _capture(self, B: int, greedy: bool):
        d = self.d
        fb = ForwardBatch(input_ids=d["input_ids"][:B], positions=d["positions"][:B], slots=d["slots"][:B],
                          num_decode=B, dec_block_tables=d["dec_tables"][:B], dec_ctx_lens=d["dec_ctx"][:B],
                          logit_rows=None, seq_slots=d["seq_slots"][:B] if self.stateful else None)
        # warm up (allocations, kernel attributes) outside the graph on dummy
        # rows written straight into the device buffers: the host staging
        # buffers may already hold the step being scheduled. A step may be in
        # flight (overlapped scheduling): wait for it so its device inputs are
        # not overwritten under it.
        torch.cuda.synchronize(self.device)
        saved = {k: d[k][:B].clone() for k in ("input_ids", "positions", "slots", "dec_tables", "dec_ctx",
                                               "seq_slots", "tok_src")}
        saved_tok = self.tok_out.clone()
        db = self.dummy_block
        d["input_ids"][:B].zero_()
        d["positions"][:B].zero_()
        d["slots"][:B].fill_(db * BLOCK_SIZE)
        d["dec_tables"][:B].fill_(db)
        d["dec_ctx"][:B].fill_(1)
        d["seq_slots"][:B].fill_(-1)
        d["tok_src"][:B].fill_(-1)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):
                ops.forward_tokens(d["input_ids"][:B], d["tok_src"][:B], self.tok_out)
                logits = self.model.forward(fb, self.kv)
                self._sample(logits, B, greedy)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        if self._graph_pool is None:
            self._graph_pool = torch.cuda.graph_pool_handle()
        n0 = ops.launch_count()
        with torch.cuda.graph(g, pool=self._graph_pool):
            ops.forward_tokens(d["input_ids"][:B], d["tok_src"][:B], self.tok_out)
            logits = self.model.forward(fb, self.kv)
            out = self._sample(logits, B, greedy)
        n_launch = ops.launch_count() - n0
        ops._count(-n_launch)  # capture does not execute; replays are counted
        for k, v in saved.items():
            d[k][:B].copy_(v)
        self.tok_out.copy_(saved_tok)
        torch.cuda.synchronize(self.device)
        self.graphs[(B, greedy)] = (g, out, n_launch)
        return g, out, n_launch

    def capture_graphs(self, sizes=None, greedy: bool = True):
        sizes = sizes or [b for b in self.cfg.graph_batch_sizes if b <= self.cfg.max_num_seqs]
        for B in sorted(sizes, reverse=True):
            if (B, greedy) not in self.graphs:
                self._capture(B, greedy)

    def step(self) -> list[RequestOutput]:
        """One engine iteration. With overlapped scheduling this launches the
        next step and returns the requests finished by the previous one."""
        with nvtx("engine.step"):
            if self._can_overlap():
                inf = self._launch(overlap=True)
                outs = self._finish(self._inflight) if self._inflight is not None else []
                self._inflight = inf
                return outs
            outs = []
            if self._inflight is not None:  # leave overlapped mode: drain the step in flight first
                outs = self._finish(self._inflight)
                self._inflight = None
            inf = self._launch(overlap=False)
            if inf is not None:
                outs += self._finish(inf)
            return outs

    def _can_overlap(self) -> bool:
        return (self.cfg.async_scheduling and self._n_host_rows == 0 and not hasattr(self.model, "share_tokens"))

    def _launch(self, overlap: bool):
        """Schedule one step and queue it on the GPU (tokens read back
        asynchronously into the pinned buffer of this step's parity)."""
        t0 = time.perf_counter()
        hb = self._hb
        h = self.h = self._hs[hb]
        info = self.sched.schedule(h["input_ids"], h["positions"], h["slots"], h["dec_tables"], h["dec_ctx"],
                                   h["pre_tables"], h["pre_ctx"], h["pre_cu"], h["logit_rows"], h["sample_ids"],
                                   h["tok_src"], overlap)
        T, nd, npf = info["num_tokens"], info["num_decode"], info["num_prefill"]
        R, max_q = info["num_logits"], info["max_q_len"]
        self.stats["steps"] += 1
        if T == 0:
            return None
        sids = h["sample_ids"][:R].tolist()
        self._step_sids = sids
        if self.stateful:
            self._assign_slots()
        greedy = self._params_rows(sids)
        pen = None if overlap else self._penalty_rows(sids)
        B = self._bucket(nd) if (npf == 0 and self.cfg.cuda_graphs and not hasattr(self.model, "share_tokens")
                                 and pen is None) else None
        stream = torch.cuda.current_stream(self.device)
        timing = self._metrics_f is not None
        ev0 = torch.cuda.Event(enable_timing=True) if timing else None
        if ev0 is not None:
            ev0.record(stream)
        if B is not None:
            key = (B, greedy)
            if key not in self.graphs:
                self._capture(B, greedy)
            g, out, n_launch = self.graphs[key]
            self._pad_decode_rows(nd, B)
            self._copy_in(dict(input_ids=B, positions=B, slots=B, dec_tables=B, dec_ctx=B, tok_src=B,
                               seq_slots=B if self.stateful else 0))
            g.replay()
            ops._count(n_launch)
            toks = out[:nd]
            self.stats["graph_steps"] += 1
            kind = "graph"
        else:
            logits = self._eager_forward(T, nd, npf, max_q, R)
            if logits is None:  # a non-final pipeline stage: tokens come from the last stage
                toks = self.tok_out[:R]
            else:
                toks = self._sample(logits, R, greedy, pen)
            if hasattr(self.model, "share_tokens"):
                self.model.share_tokens(self.tok_out[:R])
                toks = self.tok_out[:R]
            self.stats["eager_steps"] += 1
            kind = "eager"
        th = self._tok_hosts[hb]
        th[:R].copy_(toks[:R], non_blocking=True)
        self.stats["d2h_bytes"] += 4 * R
        if not greedy:
            self._lp_hosts[hb][:R].copy_(self.logprob_out[:R], non_blocking=True)
            self.stats["d2h_bytes"] += 4 * R
        ev = torch.cuda.Event(enable_timing=timing)
        ev.record(stream)
        if overlap:
            self.stats["overlapped_steps"] += 1
        self._hb ^= 1
        rec = None
        if timing:
            rec = dict(step=self.stats["steps"], kind=kind, tokens=T, decode=nd, prefill=npf, logits=R,
                       batch=B or T, running=self.sched.num_running(), waiting=self.sched.num_waiting(),
                       kv_blocks_used=self._nblocks - self.sched.num_free_blocks(), kv_blocks=self._nblocks,
                       overlap=overlap, host_launch_ms=round((time.perf_counter() - t0) * 1e3, 3))
        return dict(sids=sids, R=R, greedy=greedy, hb=hb, ev=ev, ev0=ev0, rec=rec)

    def _finish(self, inf) -> list[RequestOutput]:
        """Wait for a launched step's tokens and hand them to the scheduler and
        the request states; returns the requests that finished."""
        t0 = time.perf_counter()
        inf["ev"].synchronize()
        t1 = time.perf_counter()
        R, sids = inf["R"], inf["sids"]
        tl = self._tok_hosts[inf["hb"]][:R].tolist()
        lps = self._lp_hosts[inf["hb"]][:R].tolist() if not inf["greedy"] else None
        now = time.perf_counter()
        reqs = self.requests
        for r, sid in enumerate(sids):
            st = reqs.get(sid)
            if st is None:  # finished (stop token) while this row was in flight: discarded
                continue
            st.tokens.append(tl[r])
            if st.out_counts is not None:
                st.out_counts[tl[r]] = st.out_counts.get(tl[r], 0) + 1
                if st.params.mirostat == 2:
                    from .samplers import mirostat_update
                    mirostat_update(st.params, st, tl[r])
            st.token_times.append(now)
            if st.first_token is None:
                st.first_token = now
            if lps is not None and st.params.logprobs:
                st.logprobs.append(lps[r])
        self.stats["tokens"] += R
        done = self.sched.update(sids, tl, int(self.cfg.eos_token_id))
        outs = []
        for sid in done:
            st = self._retire(sid)
            if st is None:
                continue
            st.finish = now
            reason = _REASONS.get(self.sched.finish_reason(sid), "length")
            cached = self.sched.num_cached_prompt_tokens(sid)
            self.sched.release(sid)
            n = len(st.tokens)
            tpot = (st.finish - st.first_token) / max(1, n - 1)
            outs.append(RequestOutput(sid, st.prompt_len, st.tokens, reason, st.first_token - st.arrival, tpot,
                                      st.finish - st.arrival, cached, st.logprobs or None))
        rec = inf["rec"]
        if rec is not None:
            rec["device_ms"] = round(inf["ev0"].elapsed_time(inf["ev"]), 3)
            rec["host_wait_ms"] = round((t1 - t0) * 1e3, 3)
            rec["host_finish_ms"] = round((time.perf_counter() - t1) * 1e3, 3)
            rec["finished"] = len(outs)
            self.step_log.append(rec)
            self._metrics_f.write(json.dumps(rec) + "\n")
        return outs

    def save_prompt_cache(self, path: str, tokens: list[int]) -> int:
        """Persist the cached KV of ``tokens``' longest cached prefix (full 16-token
        blocks) with a model fingerprint; returns the tokens saved. See runtime/prompt_cache.py."""
        from .prompt_cache import save_prompt
        torch.cuda.synchronize(self.device)
        return save_prompt(self, path, tokens)

    def load_prompt_cache(self, path: str) -> int:
        """Restore a saved prompt prefix into the prefix cache (0 if the file is
        from another model); later requests starting with it skip those tokens."""
        from .prompt_cache import load_prompt
        return load_prompt(self, path)

    def generate(self, prompts: list[list[int]], params: SamplingParams | list[SamplingParams] | None = None,
                 mm: list | None = None) -> list[RequestOutput]:
        """Run requests to completion; ``mm[i]`` (optional) is request i's input
        embeddings (see ``add_request``)."""
        if not isinstance(params, list):
            params = [params or SamplingParams()] * len(prompts)
        mm = mm or [None] * len(prompts)
        ids = [self.add_request(p, sp, m) for p, sp, m in zip(prompts, params, mm)]
        order = {sid: i for i, sid in enumerate(ids)}
        results: list[RequestOutput | None] = [None] * len(ids)
        while self.has_unfinished():
            for o in self.step():
                if o.seq_id in order:
                    results[order[o.seq_id]] = o
        return results  # type: ignore
