"""Loader for the compiled sm_100a extension ``aether_b200._C``.

CUDA tensors always go through the native kernels; if the extension is missing
on a machine with a GPU every op raises instead of silently falling back.
"""
from __future__ import annotations

import os

import torch

_C = None
_ERR: Exception | None = None
try:  # pragma: no cover - depends on the build
    from . import _C as _C  # type: ignore[no-redef]
except Exception as e:  # noqa: BLE001
    _ERR = e


# Kernel launches issued per extension call (for the launch count a benchmark
# reports over its timed region).
_KERNELS_PER_CALL = {
    "rmsnorm_bwd": 2,
    "layernorm_bwd": 3,
    "attention_bwd": 3,
    "grad_norm": 2,
    "read_and_clear_status": 0,
}


class _CountingModule:
    """Proxy over ``_C`` that counts kernel launches while counting is on."""

    def __init__(self, mod):
        self._mod = mod
        self.enabled = False
        self.launches = 0
        self._cache = {}

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn
        if name not in self._cache:
            k = _KERNELS_PER_CALL.get(name, 1)

            def wrapped(*a, _fn=fn, _k=k, **kw):
                if self.enabled:
                    self.launches += _k
                return _fn(*a, **kw)

            self._cache[name] = wrapped
        return self._cache[name]


_PROXY = _CountingModule(_C) if _C is not None else None


def count_launches(enable: bool) -> int:
    """Turns launch counting on/off; returns the count so far (then resets on enable)."""
    if _PROXY is None:
        return 0
    n = _PROXY.launches
    if enable:
        _PROXY.launches = 0
    _PROXY.enabled = enable
    return n


def available() -> bool:
    return _C is not None


def C():
    """Returns the extension module or raises a clear error."""
    if _C is None:
        raise RuntimeError(
            "aether_b200 native extension is not built "
            f"({_ERR!r}); run `python -m aether_b200._build` (nvcc, sm_100a)"
        )
    return _PROXY


def so_path() -> str | None:
    return getattr(_C, "__file__", None) if _C is not None else None


def check_status() -> int:
    """Reads and clears the device status word that kernels with bounded waits
    set when a wait gives up (0 = ok)."""
    if _C is None or not torch.cuda.is_available():
        return 0
    return int(_C.read_and_clear_status())


def require_cuda_kernels() -> None:
    """Raise if a GPU is present but the native extension is not loaded."""
    if torch.cuda.is_available() and _C is None and not os.environ.get("AETHER_ALLOW_NO_EXT"):
        C()
