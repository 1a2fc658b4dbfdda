"""EOS-rate monitor (reference ``src/engine/eos_monitor.rs:36-176``).

Keeps the finish reasons of the last ``window`` completions and warns when the fraction that
stopped on EOS falls below ``threshold``: a sign that the chat template does not match the
model (it never emits its end-of-turn token).  Observation only.
"""
from __future__ import annotations

import collections
import logging
import threading

log = logging.getLogger("lightbulb_b200.eos_monitor")


class EosMonitor:
    def __init__(self, window: int = 20, threshold: float = 0.25):
        self.window = window
        self.threshold = threshold
        self._d = collections.deque(maxlen=window)
        self._lock = threading.Lock()
        self.warned = False
        self.resolved_by = None

    def record(self, finish_reason: str, resolved_by=None) -> None:
        with self._lock:
            self._d.append(finish_reason == "stop")
            self.resolved_by = resolved_by
            if len(self._d) == self.window and self.stop_rate() < self.threshold:
                if not self.warned:
                    log.warning("only %.0f%% of the last %d completions stopped on EOS "
                                "(template resolved by %s); check the chat template",
                                100 * self.stop_rate(), self.window, resolved_by)
                self.warned = True
            else:
                self.warned = False

    def stop_rate(self) -> float:
        return sum(self._d) / len(self._d) if self._d else 1.0

    def snapshot(self) -> dict:
        with self._lock:
            return {"window": self.window, "observed": len(self._d),
                    "eos_stop_rate": self.stop_rate(), "below_threshold": self.warned}
