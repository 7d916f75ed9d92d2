"""Crash breadcrumbs, the OOM flag and a device-memory leak check.

* ``crash_guard(step_fn, directory)`` -- a context manager for a training or
  serving loop: an exception escaping it writes ``crash_<pid>_<step>.dump``
  (JSON: step, time, exception, traceback, device memory statistics, caller
  extras) and re-raises. Reference: ``aether_crash_dump`` writing
  ``crash_<pid>_<step>.dump`` (runtime/src/lib.rs:2401,
  tests/runtime/crash_dump_v4.aether).
* ``oom_signal()`` / ``oom_check()`` -- a process-wide flag set when
  ``oom_guard()`` catches a device out-of-memory error, so a serving loop can
  shed load instead of dying (reference ``aether_oom_signal/check``,
  lib.rs:3676-3680).
* ``LeakCheck`` -- allocated device bytes before and after a region
  (reference GPU leak tracker, lib.rs:3660-3668).
"""
from __future__ import annotations

import contextlib
import json
import os
import time
import traceback

import torch

_OOM = False


def oom_signal() -> None:
    global _OOM
    _OOM = True


def oom_check(clear: bool = True) -> bool:
    global _OOM
    v = _OOM
    if clear:
        _OOM = False
    return v


@contextlib.contextmanager
def oom_guard():
    """Turns a device OOM into the OOM flag (the region's work is dropped)."""
    try:
        yield
    except torch.cuda.OutOfMemoryError:
        oom_signal()
        torch.cuda.empty_cache()


def _mem_stats() -> dict:
    if not torch.cuda.is_available():
        return {}
    return {"allocated": torch.cuda.memory_allocated(), "reserved": torch.cuda.memory_reserved(),
            "max_allocated": torch.cuda.max_memory_allocated()}


def write_crash_dump(step: int, exc: BaseException, directory: str = ".", extra: dict | None = None) -> str:
    os.makedirs(directory, exist_ok=True)
    path = os.path.join(directory, f"crash_{os.getpid()}_{step}.dump")
    rec = {"pid": os.getpid(), "step": step, "time": time.time(), "exception": repr(exc),
           "traceback": "".join(traceback.format_exception(type(exc), exc, exc.__traceback__)),
           "memory": _mem_stats(), "extra": extra or {}}
    with open(path + ".tmp", "w") as f:
        json.dump(rec, f, indent=1)
    os.replace(path + ".tmp", path)
    return path


@contextlib.contextmanager
def crash_guard(step_fn, directory: str = ".", extra_fn=None):
    """``step_fn()`` returns the current step when the crash happens."""
    try:
        yield
    except BaseException as e:
        if not isinstance(e, (KeyboardInterrupt, SystemExit, GeneratorExit)):
            write_crash_dump(int(step_fn()), e, directory, extra_fn() if extra_fn else None)
        raise


class LeakCheck:
    """with LeakCheck() as lc: ...; lc.leaked -> bytes still allocated."""

    def __enter__(self):
        self.before = torch.cuda.memory_allocated() if torch.cuda.is_available() else 0
        return self

    def __exit__(self, *a):
        self.after = torch.cuda.memory_allocated() if torch.cuda.is_available() else 0
        self.leaked = self.after - self.before
        return False
