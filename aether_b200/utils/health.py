"""Host-side failure detection for multi-rank jobs.

* ``Heartbeat`` -- every rank bumps a counter in a shared key-value store
  (torch.distributed's TCPStore) from a background thread; ``dead_ranks()``
  reports the ranks whose counter has not moved within ``timeout`` seconds
  (measured on the observer's own monotonic clock, so the ranks' clocks need
  not agree) and ranks that never joined. ``check()`` raises ``RankFailure``.
  A rank that leaves cleanly calls ``stop()``, which marks it done.
* ``abort_process_group()`` -- tears the communicator down so that ranks
  blocked in (or about to enter) a collective get an error instead of waiting
  for a peer that is gone; combined with a short process-group timeout this
  bounds every collective.
* ``Watchdog`` -- ``between_steps()`` runs the heartbeat check before the next
  launch of collectives and aborts the group on a failure.

The reference has no real failure detection: NCCL errors map to return codes
(runtime/src/nccl_real.rs:29-100), there is an OOM flag
(runtime/src/lib.rs:3676-3680) and a crash breadcrumb (lib.rs:2401). These
pieces are the detection layer a multi-GPU job needs; the device side of it
is the bounded waits in the in-kernel collectives, which record a status word
(``aether_b200._ext.check_status``) instead of hanging.
"""
from __future__ import annotations

import threading
import time

import torch.distributed as dist


class RankFailure(RuntimeError):
    def __init__(self, ranks, why="no heartbeat"):
        super().__init__(f"rank(s) {sorted(ranks)} failed: {why}")
        self.ranks = sorted(ranks)


class Heartbeat:
    def __init__(self, store, rank: int, world: int, period: float = 0.25, timeout: float = 3.0,
                 prefix: str = "aether/hb"):
        self.store, self.rank, self.world = store, rank, world
        self.period, self.timeout, self.prefix = period, timeout, prefix
        self._beat = 0
        self._stop = threading.Event()
        self._seen: dict = {}  # rank -> (last counter, monotonic time it changed)
        self._t_start = time.monotonic()
        self._thread = None

    def _key(self, r, what="n"):
        return f"{self.prefix}/{r}/{what}"

    def start(self) -> "Heartbeat":
        self.store.set(self._key(self.rank), "0")
        self._thread = threading.Thread(target=self._run, name="aether-heartbeat", daemon=True)
        self._thread.start()
        return self

    def _run(self):
        while not self._stop.wait(self.period):
            self._beat += 1
            try:
                self.store.set(self._key(self.rank), str(self._beat))
            except Exception:  # noqa: BLE001 -- the store itself is gone; observers will notice
                return

    def stop(self, clean: bool = True) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)
        if clean:
            try:
                self.store.set(self._key(self.rank, "done"), "1")
            except Exception:  # noqa: BLE001
                pass

    def dead_ranks(self) -> list:
        now = time.monotonic()
        dead = []
        for r in range(self.world):
            if r == self.rank:
                continue
            if self.store.check([self._key(r, "done")]):
                continue
            if not self.store.check([self._key(r)]):
                if now - self._t_start > self.timeout:
                    dead.append(r)  # never joined
                continue
            n = int(self.store.get(self._key(r)))
            last = self._seen.get(r)
            if last is None or last[0] != n:
                self._seen[r] = (n, now)
            elif now - last[1] > self.timeout:
                dead.append(r)
        return dead

    def check(self) -> None:
        dead = self.dead_ranks()
        if dead:
            raise RankFailure(dead)


def abort_process_group(group=None) -> None:
    """Best-effort teardown of a (possibly wedged) process group."""
    try:
        pg = group or dist.group.WORLD
        for dev in ("cuda", "cpu"):
            try:
                be = pg._get_backend(__import__("torch").device(dev))
            except Exception:  # noqa: BLE001
                continue
            if hasattr(be, "abort"):
                be.abort()
    except Exception:  # noqa: BLE001
        pass
    try:
        dist.destroy_process_group(group)
    except Exception:  # noqa: BLE001
        pass


class Watchdog:
    """Call ``between_steps()`` before each step's collectives; on a dead peer
    it aborts the process group and raises ``RankFailure``."""

    def __init__(self, heartbeat: Heartbeat, group=None):
        self.hb, self.group = heartbeat, group

    def between_steps(self) -> None:
        dead = self.hb.dead_ranks()
        if dead:
            self.hb.stop(clean=False)
            abort_process_group(self.group)
            raise RankFailure(dead)
