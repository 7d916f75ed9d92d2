"""Section timing without host syncs on the hot path.

``Tracer.section(name)`` brackets a region with CUDA events recorded on the
current stream (and an NVTX range, visible in Nsight Systems/Compute), or with
host timestamps for CPU work. Nothing waits while sections are recorded;
``Tracer.flush()`` synchronises once and turns the event pairs into
durations. ``summary()`` gives per-section count / total / mean milliseconds
and ``chrome_trace(path)`` writes a chrome://tracing / Perfetto JSON file.

Reference: the ``block_timing`` counters behind ``AETHER_DECODE_TIMING``
(runtime/src/serving.rs:410-450, 1352-1353), which synchronise the device
around every section, and the ``aether_prof_*``/``aether_timer_*`` stopwatches
(runtime/src/lib.rs:1377-1391). Enable with ``Tracer(enabled=True)`` or
``AETHER_TRACE=1``; disabled sections cost one attribute check.
"""
from __future__ import annotations

import contextlib
import json
import os
import time
from collections import defaultdict

import torch


class Tracer:
    def __init__(self, enabled: bool | None = None, nvtx: bool = True):
        self.enabled = os.environ.get("AETHER_TRACE", "0") == "1" if enabled is None else enabled
        self.nvtx = nvtx and torch.cuda.is_available()
        self._open: list = []  # (name, kind, start, end, host_t0)
        self._done: list = []  # (name, start_ms_host, dur_ms)
        self._t0 = time.perf_counter()

    @contextlib.contextmanager
    def section(self, name: str, device: bool | None = None):
        if not self.enabled:
            yield
            return
        use_cuda = torch.cuda.is_available() if device is None else device
        host0 = time.perf_counter()
        if self.nvtx:
            torch.cuda.nvtx.range_push(name)
        if use_cuda:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            try:
                yield
            finally:
                e1.record()
                if self.nvtx:
                    torch.cuda.nvtx.range_pop()
                self._open.append((name, e0, e1, host0))
        else:
            try:
                yield
            finally:
                if self.nvtx:
                    torch.cuda.nvtx.range_pop()
                self._done.append((name, (host0 - self._t0) * 1e3, (time.perf_counter() - host0) * 1e3))

    def flush(self) -> None:
        if self._open:
            torch.cuda.synchronize()
            for name, e0, e1, host0 in self._open:
                self._done.append((name, (host0 - self._t0) * 1e3, e0.elapsed_time(e1)))
            self._open.clear()

    def summary(self) -> dict:
        self.flush()
        agg = defaultdict(lambda: [0, 0.0])
        for name, _, dur in self._done:
            agg[name][0] += 1
            agg[name][1] += dur
        return {k: {"count": c, "total_ms": t, "mean_ms": t / c} for k, (c, t) in agg.items()}

    def chrome_trace(self, path: str) -> None:
        self.flush()
        ev = [{"name": n, "ph": "X", "ts": s * 1e3, "dur": d * 1e3, "pid": os.getpid(), "tid": 0}
              for n, s, d in self._done]
        with open(path, "w") as f:
            json.dump({"traceEvents": ev}, f)

    def reset(self) -> None:
        self.flush()
        self._done.clear()


_GLOBAL = None


def global_tracer() -> Tracer:
    global _GLOBAL
    if _GLOBAL is None:
        _GLOBAL = Tracer()
    return _GLOBAL
