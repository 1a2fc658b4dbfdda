"""Per-rank liveness watchdog over a key-value store (e.g. ``torch.distributed.TCPStore``).

Every rank runs two host threads: a beat thread that increments the rank's counter in the
store every ``interval_s``, and a monitor that reads every peer's counter and records, on its
own monotonic clock, when each one last changed.  A peer whose counter has not moved for
``timeout_s`` is declared failed (no clock agreement between hosts is needed); a peer that
has never beaten is only declared failed after ``startup_timeout_s`` (ranks start at different
times); a store that stops answering (its host rank died) counts as a failure too.
``on_failure`` is called once, from the monitor thread, with the set of failed ranks;
:func:`attach` connects it to an :class:`~lightbulb_b200.engine.async_engine.AsyncEngine`,
which then stops stepping, fails its in-flight requests and makes the server answer 503.

The reference has no multi-GPU failure handling.  This works entirely on the host: the
device side of failure handling is the bounded waits of the collective kernels, which report
an error code instead of spinning forever.
"""
from __future__ import annotations

import threading
import time
from typing import Callable, Dict, Iterable, Optional, Set

STORE_FAILURE = -1       # pseudo-rank reported when the store itself is unreachable


class Watchdog:
    def __init__(self, store, rank: int, world: int, interval_s: float = 0.5,
                 timeout_s: float = 5.0, on_failure: Optional[Callable[[Set[int]], None]] = None,
                 prefix: str = "lb_hb", startup_timeout_s: float = 120.0):
        if timeout_s <= 2 * interval_s:
            raise ValueError("timeout_s must exceed two heartbeat intervals")
        self.store, self.rank, self.world = store, rank, world
        self.interval, self.timeout = interval_s, timeout_s
        self.startup_timeout = max(startup_timeout_s, timeout_s)
        self.on_failure = on_failure
        self.prefix = prefix
        self.failed: Set[int] = set()
        self._seen: Dict[int, tuple] = {}          # peer -> (counter, local time of change)
        self._stop = threading.Event()
        self._paused = threading.Event()
        self._reported = False
        self._threads = []

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    # -- threads ------------------------------------------------------------------------
    def _beat(self) -> None:
        while not self._stop.is_set():
            if not self._paused.is_set():
                try:
                    self.store.add(self._key(self.rank), 1)
                except Exception:
                    self._declare({STORE_FAILURE})
                    return
            self._stop.wait(self.interval)

    def _monitor(self) -> None:
        start = time.monotonic()
        while not self._stop.is_set():
            now = time.monotonic()
            dead = set()
            for r in range(self.world):
                if r == self.rank:
                    continue
                try:
                    c = int(self.store.add(self._key(r), 0))      # read without changing
                except Exception:
                    dead.add(STORE_FAILURE)
                    break
                if c == 0:
                    # never beaten yet: ranks start at different times, so a peer is timed
                    # only after its first beat, and otherwise gets the (longer) startup limit
                    if now - start > self.startup_timeout:
                        dead.add(r)
                    continue
                prev = self._seen.get(r)
                if prev is None or prev[0] != c:
                    self._seen[r] = (c, now)
                elif now - prev[1] > self.timeout:
                    dead.add(r)
            if dead:
                self._declare(dead)
            self._stop.wait(self.interval)

    def _declare(self, dead: Iterable[int]) -> None:
        new = set(dead) - self.failed
        if not new:
            return
        self.failed |= new
        if not self._reported and self.on_failure is not None:
            self._reported = True
            try:
                self.on_failure(set(self.failed))
            except Exception:
                pass

    # -- control ------------------------------------------------------------------------
    def start(self) -> "Watchdog":
        for fn in (self._beat, self._monitor):
            t = threading.Thread(target=fn, name=f"lb-watchdog-{fn.__name__}", daemon=True)
            t.start()
            self._threads.append(t)
        return self

    def pause(self) -> None:
        """Stop beating (tests / planned maintenance); peers will declare this rank failed."""
        self._paused.set()

    def resume(self) -> None:
        self._paused.clear()

    def stop(self) -> None:
        self._stop.set()
        for t in self._threads:
            t.join(timeout=2 * self.interval + 1)

    @property
    def healthy(self) -> bool:
        return not self.failed


def attach(async_engine, watchdog: Watchdog) -> Watchdog:
    """Stop ``async_engine`` (and make the server report 503) when a peer rank fails."""
    def fail(dead: Set[int]) -> None:
        who = "the rendezvous store" if dead == {STORE_FAILURE} else \
            f"rank(s) {sorted(r for r in dead if r >= 0)}"
        async_engine.fail(f"{who} stopped heartbeating")
    watchdog.on_failure = fail
    return watchdog
