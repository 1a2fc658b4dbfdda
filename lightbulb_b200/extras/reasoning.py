"""Reasoning controls behind ``/v1/lightbulb/reasoning/*`` (reference
``src/engine/reasoning_controls.rs``): a per-request budget (chains / steps / tokens) and a
convergence check over successive answers (stop when the last answers agree)."""
from __future__ import annotations

import threading
from dataclasses import asdict, dataclass, field
from typing import Dict, List, Optional


@dataclass
class ReasoningBudget:
    max_chains: Optional[int] = None
    max_steps: Optional[int] = None
    max_tokens: Optional[int] = None


@dataclass
class ConvergenceTracker:
    answers: List[str] = field(default_factory=list)
    window: int = 3

    def add(self, answer: str) -> None:
        self.answers.append(answer.strip())

    def converged(self) -> bool:
        a = self.answers[-self.window:]
        return len(a) == self.window and len(set(a)) == 1


class ReasoningControls:
    def __init__(self):
        self.budget = ReasoningBudget()
        self.trackers: Dict[str, ConvergenceTracker] = {}
        self.lock = threading.Lock()
        self.requests_with_budget = 0

    def set_budget(self, **kw) -> dict:
        with self.lock:
            self.budget = ReasoningBudget(**{k: kw.get(k) for k in ("max_chains", "max_steps",
                                                                      "max_tokens")})
        return asdict(self.budget)

    def clamp_max_tokens(self, requested: int) -> int:
        b = self.budget.max_tokens
        if b:
            self.requests_with_budget += 1
            return min(requested, b)
        return requested

    def convergence(self, key: str) -> dict:
        t = self.trackers.get(key)
        return {"key": key, "answers": len(t.answers) if t else 0,
                "converged": bool(t and t.converged())}

    def stats(self) -> dict:
        return {"budget": asdict(self.budget), "tracked": len(self.trackers),
                "requests_with_budget": self.requests_with_budget}
