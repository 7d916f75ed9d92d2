"""Continuous-batching generation engine.

Reference: BatchScheduler (runtime/src/batched_serving.rs:1-300) -- a worker
thread owns the GPU, admits up to ``max_concurrent`` requests, prefills each
new request, runs one multiplexed decode tick for every active slot, samples
per slot and retires finished sequences. Here the decode tick is one CUDA
graph replay of ``QwenModel.decode_step`` over all active slots (per-row
positions and cache slots), and prefill runs the whole prompt at once on the
tensor cores.
"""
from __future__ import annotations

import collections
import itertools
import queue
import threading
import time
from dataclasses import dataclass, field

import torch

from .sampling import SamplingParams, sample_rows


@dataclass
class Request:
    prompt_ids: list
    params: SamplingParams
    id: int = 0
    out: "queue.Queue" = field(default_factory=queue.Queue)  # token ids, then None
    tokens: list = field(default_factory=list)
    finish_reason: str | None = None
    t_submit: float = 0.0
    t_first: float | None = None
    t_done: float | None = None
    slot: int = -1
    text_so_far: str = ""

    @property
    def ttft(self) -> float | None:
        return None if self.t_first is None else self.t_first - self.t_submit


class Metrics:
    """Prometheus-style counters and a TTFT summary."""

    def __init__(self):
        self.lock = threading.Lock()
        self.counters = {"requests_total": 0, "requests_finished": 0, "tokens_generated": 0, "prompt_tokens": 0,
                         "decode_steps": 0}
        self.ttft = []
        self.queue_depth = 0
        self.active = 0

    def inc(self, key, n=1):
        with self.lock:
            self.counters[key] = self.counters.get(key, 0) + n

    def prometheus(self) -> str:
        with self.lock:
            lines = []
            for k, v in self.counters.items():
                lines.append(f"# TYPE aether_{k} counter\naether_{k} {v}")
            lines.append(f"# TYPE aether_queue_depth gauge\naether_queue_depth {self.queue_depth}")
            lines.append(f"# TYPE aether_active_sequences gauge\naether_active_sequences {self.active}")
            if self.ttft:
                s = sorted(self.ttft)
                for q in (0.5, 0.9, 0.99):
                    lines.append(f'aether_ttft_seconds{{quantile="{q}"}} {s[min(len(s) - 1, int(q * len(s)))]:.6f}')
            return "\n".join(lines) + "\n"


class Engine:
    def __init__(self, model, tokenizer, max_concurrent: int = 8, eos_ids=None, use_graph: bool = True):
        self.model = model
        self.tok = tokenizer
        self.max_concurrent = min(max_concurrent, model.max_batch)
        self.eos_ids = set(eos_ids or ([tokenizer.eos_id] if getattr(tokenizer, "eos_id", None) is not None else []))
        self.use_graph = use_graph
        self.pending: "queue.Queue[Request]" = queue.Queue()
        self.active: dict = {}  # slot -> Request
        self.free_slots = list(range(self.max_concurrent))
        self.metrics = Metrics()
        self._ids = itertools.count(1)
        self._stop = threading.Event()
        self._wake = threading.Condition()
        self._gens: dict = {}
        self.errors: list = []  # formatted tracebacks of worker-side failures
        self._deferred: collections.deque = collections.deque()  # admitted later, when KV pages free up
        self.paged = bool(getattr(model, "paged", False))
        self.worker = threading.Thread(target=self._loop, name="aether-engine", daemon=True)
        self.worker.start()

    # ------------------------------------------------------------------ API
    def submit(self, prompt_ids: list, params: SamplingParams | None = None) -> Request:
        params = params or SamplingParams()
        limit = self.model.max_seq - 1
        if len(prompt_ids) == 0:
            raise ValueError("empty prompt")
        if len(prompt_ids) + params.max_tokens > limit:
            params.max_tokens = max(1, limit - len(prompt_ids))
        if self.paged:
            c = self.model.cache
            if c.pages_for(len(prompt_ids) + params.max_tokens) > c.alloc.num_pages - 1:
                raise ValueError("request needs more KV pages than the pool holds")
        r = Request(list(prompt_ids), params, id=next(self._ids), t_submit=time.perf_counter())
        self.metrics.inc("requests_total")
        self.metrics.inc("prompt_tokens", len(prompt_ids))
        self.pending.put(r)
        with self._wake:
            self._wake.notify()
        return r

    def generate(self, prompt: str | list, params: SamplingParams | None = None, timeout: float = 600.0):
        """Blocking helper: returns (text, token_ids, request)."""
        ids = self.tok.encode(prompt) if isinstance(prompt, str) else list(prompt)
        r = self.submit(ids, params)
        toks = []
        deadline = time.time() + timeout
        while True:
            t = r.out.get(timeout=max(0.01, deadline - time.time()))
            if t is None:
                break
            toks.append(t)
        return self.tok.decode(toks), toks, r

    def stream(self, r: Request, timeout: float = 600.0):
        """Yields token ids of a submitted request as they are produced."""
        deadline = time.time() + timeout
        while True:
            t = r.out.get(timeout=max(0.01, deadline - time.time()))
            if t is None:
                return
            yield t

    def shutdown(self):
        self._stop.set()
        with self._wake:
            self._wake.notify()
        self.worker.join(timeout=10)

    # ------------------------------------------------------------------ worker
    def _gen(self, r: Request):
        if r.id not in self._gens:
            g = torch.Generator(device=self.model.device)
            g.manual_seed(int(r.params.seed) if r.params.seed is not None else (r.id * 7919 + 17))
            self._gens[r.id] = g
        return self._gens[r.id]

    def _emit(self, r: Request, tok: int) -> bool:
        """Records a token; returns True when the request is finished."""
        if r.t_first is None:
            r.t_first = time.perf_counter()
            with self.metrics.lock:
                self.metrics.ttft.append(r.ttft)
        r.tokens.append(tok)
        self.metrics.inc("tokens_generated")
        p = r.params
        if tok in self.eos_ids or tok in p.stop_token_ids:
            r.finish_reason = "stop"
            return True
        r.out.put(tok)
        if p.stop:
            r.text_so_far = self.tok.decode(r.tokens)
            if any(s in r.text_so_far for s in p.stop):
                r.finish_reason = "stop"
                return True
        if len(r.tokens) >= p.max_tokens:
            r.finish_reason = "length"
            return True
        return False

    def _finish(self, r: Request):
        r.t_done = time.perf_counter()
        r.out.put(None)
        self.metrics.inc("requests_finished")
        self._gens.pop(r.id, None)
        if r.slot >= 0:
            self.active.pop(r.slot, None)
            if self.paged:
                self.model.cache.release(r.slot)
            self.free_slots.append(r.slot)

    def _reserve_pages(self, r: Request, slot: int):
        """Paged cache: shares cached prefix pages and reserves the pages the
        whole request can reach. Returns the number of prompt tokens whose K/V
        are already cached, or None (request deferred) if the pool is full."""
        from .kv import NoPages

        c = self.model.cache
        try:
            n = c.match_prefix(slot, r.prompt_ids)
            c.ensure(slot, len(r.prompt_ids) + r.params.max_tokens)
        except NoPages:
            c.release(slot)
            return None
        if n:
            self.metrics.inc("prefix_cached_tokens", n)
        return n

    @torch.no_grad()
    def _admit(self):
        while self.free_slots and (self._deferred or not self.pending.empty()):
            r = self._deferred.popleft() if self._deferred else self.pending.get()
            slot = self.free_slots.pop(0)
            cached = 0
            if self.paged:
                cached = self._reserve_pages(r, slot)
                if cached is None:  # wait for running requests to release pages
                    self.free_slots.insert(0, slot)
                    self._deferred.appendleft(r)
                    return
            r.slot = slot
            self.active[slot] = r  # from here on an error path finishes it
            dev = self.model.device
            ids = torch.tensor([r.prompt_ids[cached:]], dtype=torch.long, device=dev)
            nxt, logits = self.model.prefill(ids, slots=torch.tensor([slot], dtype=torch.int32, device=dev),
                                             start_pos=cached, return_logits=True)
            if self.paged:
                self.model.cache.register_prompt(slot, r.prompt_ids)
            tok = int(sample_rows(logits, [r.params], [[]], [self._gen(r)])[0]) if not r.params.greedy else int(nxt[0])
            if self._emit(r, tok):
                self._finish(r)

    @torch.no_grad()
    def _tick(self):
        reqs = list(self.active.values())
        if not reqs:
            return
        dev = self.model.device
        toks = torch.tensor([r.tokens[-1] for r in reqs], dtype=torch.long, device=dev)
        pos = torch.tensor([len(r.prompt_ids) + len(r.tokens) - 1 for r in reqs], dtype=torch.int32, device=dev)
        slots = torch.tensor([r.slot for r in reqs], dtype=torch.int32, device=dev)
        want = any(not r.params.greedy for r in reqs)
        nxt = self.model.decode_step(toks, pos, slots, use_graph=self.use_graph, want_logits=want)
        if want:
            logits = self.model.buf["logits"][: len(reqs)]
            nxt = sample_rows(logits, [r.params for r in reqs], [r.tokens for r in reqs], [self._gen(r) for r in reqs])
        self.metrics.inc("decode_steps")
        out = nxt.tolist()
        for r, t in zip(reqs, out):
            if self._emit(r, int(t)):
                self._finish(r)

    def _loop(self):
        while not self._stop.is_set():
            try:
                self._admit()
                self.metrics.queue_depth = self.pending.qsize() + len(self._deferred)
                self.metrics.active = len(self.active)
                if self.active:
                    self._tick()
                else:
                    with self._wake:
                        if self.pending.empty() and not self._stop.is_set():
                            self._wake.wait(timeout=0.05)
            except Exception as e:  # noqa: BLE001 -- fail every request instead of dying silently
                import sys
                import traceback

                self.errors.append(traceback.format_exc())
                print(f"aether engine: {self.errors[-1]}", file=sys.stderr, flush=True)
                for r in list(self.active.values()):
                    r.finish_reason = f"error: {e}"
                    self._finish(r)
                while self._deferred or not self.pending.empty():
                    r = self._deferred.popleft() if self._deferred else self.pending.get()
                    r.finish_reason = f"error: {e}"
                    r.out.put(None)
