"""Reasoning controls behind ``/v1/lightbulb/reasoning/*`` (reference
``src/engine/reasoning_controls.rs``): a per-request budget (chains / steps / tokens), a
convergence check over successive answers, and the budget-aware decoding controls of the
reference's ``ReasoningController``: overthinking detection from the next-token distributions
(low average entropy and low variance of the top probability over a window,
``reasoning_controls.rs:117-247``), repetition detection, termination policies (fixed steps,
confidence threshold, convergence of step scores, special token, any-of,
``reasoning_controls.rs:249-307``) and per-chain bookkeeping with statistics
(``reasoning_controls.rs:309-520``).

Instead of keeping whole logit vectors per step on the host (the reference stores each step's
logits), :func:`logits_stats` reduces a batch of logit rows on whatever device they live on to
the two numbers the detector needs (entropy, top probability) per row, and the controller keeps
a window of those.
"""
from __future__ import annotations

import threading
from collections import deque
from dataclasses import asdict, dataclass, field
from typing import Deque, Dict, List, Optional, Sequence, Tuple

import torch


def logits_stats(logits: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per row of ``logits`` [B, V]: softmax entropy (nats) and top probability, in fp32 on the
    logits' device (one pass of log-softmax; probabilities below 1e-10 contribute nothing, as
    in the reference's entropy)."""
    lf = logits.float()
    logp = torch.log_softmax(lf, dim=-1)
    p = logp.exp()
    ent = -(torch.where(p > 1e-10, p * logp, torch.zeros_like(p))).sum(-1)
    return ent, p.max(-1).values


def _variance(vals: Sequence[float]) -> float:
    if not vals:
        return 0.0
    m = sum(vals) / len(vals)
    return sum((v - m) ** 2 for v in vals) / len(vals)


@dataclass
class DecodingBudget:
    """Budget of one reasoning request (reference ``ReasoningBudget``)."""

    max_chains: int = 3
    max_steps_per_chain: int = 10
    max_total_tokens: int = 500
    enabled: bool = True
    verifier_frequency: int = 5

    def can_start_chain(self, chains: int) -> bool:
        return not self.enabled or chains < self.max_chains

    def can_continue_chain(self, steps: int) -> bool:
        return not self.enabled or steps < self.max_steps_per_chain

    def can_generate_tokens(self, current: int, new: int) -> bool:
        return not self.enabled or current + new <= self.max_total_tokens

    def should_verify(self, step: int) -> bool:
        return self.verifier_frequency > 0 and step % self.verifier_frequency == 0


@dataclass
class OverthinkingDetector:
    """Overthinking = over the last ``window_size`` steps the average entropy is below
    ``entropy_threshold`` AND the variance of the top probability is below
    ``variance_threshold``; repetition = the last ``window_size`` tokens equal the
    ``window_size`` before them."""

    window_size: int = 5
    entropy_threshold: float = 0.5
    variance_threshold: float = 0.1
    enabled: bool = True

    def is_overthinking(self, stats: Sequence[Tuple[float, float]]) -> bool:
        """``stats``: (entropy, top probability) per step, oldest first."""
        if not self.enabled or len(stats) < self.window_size:
            return False
        recent = list(stats)[-self.window_size:]
        avg_ent = sum(e for e, _ in recent) / self.window_size
        return avg_ent < self.entropy_threshold and \
            _variance([p for _, p in recent]) < self.variance_threshold

    def is_overthinking_logits(self, logits_history: Sequence) -> bool:
        """Same test from raw logit rows (lists or tensors), as the reference takes them."""
        rows = [torch.as_tensor(r, dtype=torch.float32) for r in logits_history]
        if not rows:
            return False
        ent, top = logits_stats(torch.stack(rows))
        return self.is_overthinking(list(zip(ent.tolist(), top.tolist())))

    def is_repeating(self, tokens: Sequence[int]) -> bool:
        w = self.window_size
        if not self.enabled or len(tokens) < 2 * w:
            return False
        return list(tokens[-w:]) == list(tokens[-2 * w:-w])


@dataclass
class TerminationPolicy:
    """One of: ``fixed_steps(n)``, ``confidence(t)``, ``convergence(window, threshold)``
    (variance of the last ``window`` step scores below ``threshold``), ``special_token(id)``,
    ``combined([...])`` (any member triggers)."""

    kind: str
    value: float = 0.0
    window: int = 0
    members: List["TerminationPolicy"] = field(default_factory=list)

    @staticmethod
    def fixed_steps(n: int) -> "TerminationPolicy":
        return TerminationPolicy("fixed_steps", float(n))

    @staticmethod
    def confidence(threshold: float) -> "TerminationPolicy":
        return TerminationPolicy("confidence", threshold)

    @staticmethod
    def convergence(window: int, threshold: float) -> "TerminationPolicy":
        return TerminationPolicy("convergence", threshold, window)

    @staticmethod
    def special_token(token: int) -> "TerminationPolicy":
        return TerminationPolicy("special_token", float(token))

    @staticmethod
    def combined(policies: List["TerminationPolicy"]) -> "TerminationPolicy":
        return TerminationPolicy("combined", members=list(policies))

    def should_terminate(self, step: int, confidence: float, recent_scores: Sequence[float],
                         token: int) -> bool:
        k = self.kind
        if k == "fixed_steps":
            return step >= int(self.value)
        if k == "confidence":
            return confidence >= self.value
        if k == "convergence":
            if len(recent_scores) < self.window:
                return False
            return _variance(list(recent_scores)[-self.window:]) < self.value
        if k == "special_token":
            return token == int(self.value)
        if k == "combined":
            return any(p.should_terminate(step, confidence, recent_scores, token)
                       for p in self.members)
        raise ValueError(f"unknown termination policy {k!r}")


@dataclass
class ReasoningChain:
    id: int
    steps: int = 0
    tokens: List[int] = field(default_factory=list)
    confidences: List[float] = field(default_factory=list)
    completed: bool = False
    termination_reason: Optional[str] = None

    def add_step(self, token: int, confidence: float) -> None:
        self.steps += 1
        self.tokens.append(int(token))
        self.confidences.append(float(confidence))

    def complete(self, reason: str) -> None:
        self.completed = True
        self.termination_reason = reason

    def average_confidence(self) -> float:
        return sum(self.confidences) / len(self.confidences) if self.confidences else 0.0


@dataclass
class ReasoningStats:
    total_chains: int
    completed_chains: int
    total_tokens: int
    avg_steps_per_chain: float
    avg_confidence: float


class ReasoningController:
    """Budget + overthinking + repetition + termination policy over reasoning chains.
    :meth:`record_step` returns True when the chain should stop (the reason is kept on the
    chain); checks run in the reference's order: step budget, token budget, overthinking,
    repetition, policy."""

    def __init__(self, budget: Optional[DecodingBudget] = None,
                 detector: Optional[OverthinkingDetector] = None,
                 policy: Optional[TerminationPolicy] = None, max_history: int = 20):
        self.budget = budget or DecodingBudget()
        self.detector = detector or OverthinkingDetector()
        self.policy = policy or TerminationPolicy.fixed_steps(self.budget.max_steps_per_chain)
        self.chains: List[ReasoningChain] = []
        self.total_tokens = 0
        self.history: Deque[Tuple[float, float]] = deque(maxlen=max_history)

    def start_chain(self) -> int:
        if not self.budget.can_start_chain(len(self.chains)):
            raise RuntimeError(f"Budget exceeded: max chains {self.budget.max_chains} reached")
        self.chains.append(ReasoningChain(len(self.chains)))
        return len(self.chains) - 1

    def record_step(self, chain_id: int, token: int, confidence: float,
                    stats: Optional[Tuple[float, float]] = None,
                    logits: Optional[torch.Tensor] = None) -> bool:
        """One decoding step of chain ``chain_id``: the chosen token, its confidence, and the
        step's (entropy, top probability) -- given directly or computed from ``logits``."""
        if not 0 <= chain_id < len(self.chains):
            raise KeyError(f"Invalid chain ID: {chain_id}")
        ch = self.chains[chain_id]
        if not self.budget.can_continue_chain(ch.steps):
            ch.complete("Budget: max steps reached")
            return True
        if not self.budget.can_generate_tokens(self.total_tokens, 1):
            ch.complete("Budget: max tokens reached")
            return True
        if stats is None and logits is not None:
            e, p = logits_stats(torch.as_tensor(logits).reshape(1, -1))
            stats = (float(e[0]), float(p[0]))
        if stats is not None:
            self.history.append((float(stats[0]), float(stats[1])))
        ch.add_step(token, confidence)
        self.total_tokens += 1
        if self.detector.is_overthinking(self.history):
            ch.complete("Overthinking detected")
            return True
        if self.detector.is_repeating(ch.tokens):
            ch.complete("Repetition detected")
            return True
        if self.policy.should_terminate(ch.steps, confidence, ch.confidences, token):
            ch.complete("Termination policy triggered")
            return True
        return False

    def get_chain(self, chain_id: int) -> Optional[ReasoningChain]:
        return self.chains[chain_id] if 0 <= chain_id < len(self.chains) else None

    def stats(self) -> ReasoningStats:
        n = len(self.chains)
        return ReasoningStats(
            total_chains=n, completed_chains=sum(c.completed for c in self.chains),
            total_tokens=self.total_tokens,
            avg_steps_per_chain=(sum(c.steps for c in self.chains) / n) if n else 0.0,
            avg_confidence=(sum(c.average_confidence() for c in self.chains) / n) if n else 0.0)

    def reset(self) -> None:
        self.chains.clear()
        self.total_tokens = 0
        self.history.clear()


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
