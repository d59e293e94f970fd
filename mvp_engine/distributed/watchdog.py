"""Host-side failure detection: a heartbeat watchdog over the rendezvous store.

The reference relies on torchrun alone: its process group has no timeout and
there is no heartbeat (mvp_engine/distributed/init.py:59-64).  Here every rank
runs a daemon thread that bumps a counter key ``<prefix>/<rank>`` in the
process group's store every ``interval_s`` and watches the other ranks'
counters.  A rank whose counter has not moved for ``timeout_s`` (measured on
this rank's own monotonic clock, so host clock skew does not matter) is
reported; the training loop calls :meth:`HeartbeatWatchdog.check` between
steps and gets a :class:`PeerFailureError` naming the silent ranks, before it
launches the next step's collectives.

Together with the explicit process-group timeout (``MVP_PG_TIMEOUT_S``) and the
bounded device-side waits of the peer-memory kernels (status word checked
after every step), no failure mode leaves a rank blocked forever.
"""

from __future__ import annotations

import os
import threading
import time
from typing import Optional

import torch.distributed as dist


class PeerFailureError(RuntimeError):
    def __init__(self, ranks: list[int], detail: str = "") -> None:
        self.ranks = sorted(ranks)
        super().__init__(f"peer rank(s) {self.ranks} stopped sending heartbeats{': ' + detail if detail else ''}")


class HeartbeatWatchdog:
    def __init__(self, store, rank: int, world: int, *, interval_s: float = 5.0, timeout_s: float = 300.0,
                 prefix: str = "mvp/heartbeat") -> None:
        if interval_s <= 0 or timeout_s <= interval_s:
            raise ValueError("heartbeat needs 0 < interval_s < timeout_s")
        self.store, self.rank, self.world = store, int(rank), int(world)
        self.interval_s, self.timeout_s, self.prefix = float(interval_s), float(timeout_s), prefix
        self._beat = 0
        self._seen: dict[int, tuple[str, float]] = {}
        self._failed: set[int] = set()
        self._last_store_ok = time.monotonic()
        self._store_error = ""
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self._lock = threading.Lock()

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def _tick(self) -> None:
        self._beat += 1
        self.store.set(self._key(self.rank), str(self._beat))
        now = time.monotonic()
        for r in range(self.world):
            if r == self.rank:
                continue
            key = self._key(r)
            val = self.store.get(key).decode() if self.store.check([key]) else ""
            last = self._seen.get(r)
            if last is None or last[0] != val:
                self._seen[r] = (val, now)
            elif now - last[1] > self.timeout_s:
                with self._lock:
                    self._failed.add(r)

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                self._tick()
                self._last_store_ok = time.monotonic()
            except Exception as exc:  # noqa: BLE001
                # One failed store round trip is treated like a missed heartbeat: only a store that
                # stays unreachable for timeout_s marks the peers as failed.
                self._store_error = repr(exc)
                if time.monotonic() - self._last_store_ok > self.timeout_s:
                    with self._lock:
                        self._failed.update(r for r in range(self.world) if r != self.rank)
            self._stop.wait(self.interval_s)

    def start(self) -> "HeartbeatWatchdog":
        if self._thread is None:
            self._tick()
            self._thread = threading.Thread(target=self._run, name="mvp-heartbeat", daemon=True)
            self._thread.start()
        return self

    def failed_ranks(self) -> list[int]:
        with self._lock:
            return sorted(self._failed)

    def check(self) -> None:
        failed = self.failed_ranks()
        if failed:
            raise PeerFailureError(failed, f"last store error {self._store_error}" if self._store_error else "")

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=self.interval_s * 2 + 1)
            self._thread = None


def start_default_watchdog() -> Optional[HeartbeatWatchdog]:
    """Watchdog on the default process group's store when running with 2+ ranks.

    ``MVP_HEARTBEAT_TIMEOUT_S`` (default 600; 0 disables) and ``MVP_HEARTBEAT_INTERVAL_S``
    (default 5) configure it.
    """
    timeout = float(os.environ.get("MVP_HEARTBEAT_TIMEOUT_S", "600"))
    if timeout <= 0 or not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() < 2:
        return None
    from torch.distributed.distributed_c10d import _get_default_store

    interval = float(os.environ.get("MVP_HEARTBEAT_INTERVAL_S", "5"))
    return HeartbeatWatchdog(_get_default_store(), dist.get_rank(), dist.get_world_size(), interval_s=interval,
                             timeout_s=timeout).start()
