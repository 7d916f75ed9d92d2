"""In-tree build of the native code (no network, no pip install).

``build()`` compiles the torch extension ``aether_b200/_C`` for sm_100a with
``setup.py build_ext --inplace`` and the standalone C-ABI runtime
``aether_b200/libaether_rt.so`` with nvcc. Both land inside the package
directory so they travel with the source tree.
"""
from __future__ import annotations

import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def build_extension(verbose: bool = False) -> None:
    env = dict(os.environ)
    env.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 1)))
    cmd = [sys.executable, "setup.py", "build_ext", "--inplace"]
    out = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=not verbose, text=True)
    if out.returncode != 0:
        msg = (out.stdout or "")[-6000:] + (out.stderr or "")[-6000:]
        raise RuntimeError(f"extension build failed:\n{msg}")


def build_runtime(verbose: bool = False) -> None:
    rt = os.path.join(ROOT, "csrc", "rt")
    if not os.path.isdir(rt):
        return
    out = subprocess.run(["make", "-C", rt, f"-j{os.cpu_count() or 1}"], capture_output=not verbose, text=True)
    if out.returncode != 0:
        msg = (out.stdout or "")[-6000:] + (out.stderr or "")[-6000:]
        raise RuntimeError(f"runtime build failed:\n{msg}")


def build(verbose: bool = False) -> None:
    build_extension(verbose)
    build_runtime(verbose)


if __name__ == "__main__":
    build(verbose=True)
