"""Eviction policies over cached token slots and their weighted voting.

Reference: ``src/cache/eviction_policy.rs:11-216`` -- an ``EvictionPolicy`` returns
(slot, score) pairs where a higher score means "evict sooner" and -inf means "never evict";
``VotingAggregator`` normalises each policy's finite scores to [0, 1], weights them and sums;
``RecencyPolicy`` protects the most recent tokens.  The reference's aggregator skips +inf scores
(a known defect: a slot that one policy marks as the *first* to go is dropped from that policy's
vote, ``policies.rs:31-43``).  Here +inf keeps its meaning: such a slot ranks above every finite
aggregate unless another policy vetoes it with -inf (a veto always wins).

Scores come from this engine's state: positions of a sequence's KV (``slot -> position``) and,
for :class:`H2OScorePolicy`, the device score pool that :class:`~.compression.H2OPolicy`
accumulates (cumulative decayed attention mass; score = 1 / mass, +inf when never attended).
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

Scores = List[Tuple[int, float]]


class EvictionPolicy:
    name = "base"

    def compute_eviction_scores(self, positions: Dict[int, int]) -> Scores:
        raise NotImplementedError

    def select_eviction_candidate(self, positions: Dict[int, int]) -> Optional[int]:
        s = [x for x in self.compute_eviction_scores(positions) if x[1] != -math.inf]
        return s[0][0] if s else None


def _sorted(scores: Scores) -> Scores:
    return sorted(scores, key=lambda x: (-x[1] if x[1] == x[1] else math.inf, x[0]))


class RecencyPolicy(EvictionPolicy):
    """Older tokens first; the ``num_recent_to_keep`` newest positions are never evicted."""
    name = "recency"

    def __init__(self, num_recent_to_keep: int = 4):
        self.keep = num_recent_to_keep

    def compute_eviction_scores(self, positions: Dict[int, int]) -> Scores:
        if not positions:
            return []
        mx = max(positions.values())
        thr = mx - self.keep
        return _sorted([(s, -math.inf if p > thr else float(mx - p)) for s, p in positions.items()])


class SinkPolicy(EvictionPolicy):
    """The first ``sinks`` positions are never evicted (StreamingLLM attention sinks)."""
    name = "sinks"

    def __init__(self, sinks: int = 4):
        self.sinks = sinks

    def compute_eviction_scores(self, positions: Dict[int, int]) -> Scores:
        return _sorted([(s, -math.inf if p < self.sinks else 0.0) for s, p in positions.items()])


class H2OScorePolicy(EvictionPolicy):
    """Heavy hitters: score = 1 / cumulative attention mass of the slot (+inf if it never
    received attention); the ``num_recent_to_keep`` newest positions are protected."""
    name = "h2o"

    def __init__(self, mass, num_recent_to_keep: int = 4):
        self.mass = mass  # slot -> cumulative mass (tensor indexed by slot, or dict)
        self.keep = num_recent_to_keep

    def _m(self, slot: int) -> float:
        m = self.mass[slot]
        return float(m.item() if hasattr(m, "item") else m)

    def compute_eviction_scores(self, positions: Dict[int, int]) -> Scores:
        if not positions:
            return []
        thr = max(positions.values()) - self.keep
        out = []
        for s, p in positions.items():
            if p > thr:
                out.append((s, -math.inf))
                continue
            m = self._m(s)
            out.append((s, math.inf if m <= 0.0 else 1.0 / m))
        return _sorted(out)


class VotingAggregator:
    """Weighted vote of several policies (weights are normalised)."""

    def __init__(self):
        self.policies: List[Tuple[EvictionPolicy, float]] = []

    def add_policy(self, policy: EvictionPolicy, weight: float = 1.0) -> "VotingAggregator":
        self.policies.append((policy, float(weight)))
        return self

    def compute_aggregated_scores(self, positions: Dict[int, int]) -> Scores:
        if not self.policies:
            return []
        total_w = sum(w for _, w in self.policies) or 1.0
        agg: Dict[int, float] = {}
        veto, first = set(), set()
        for pol, w in self.policies:
            sc = pol.compute_eviction_scores(positions)
            fin = [v for _, v in sc if math.isfinite(v)]
            lo, hi = (min(fin), max(fin)) if fin else (0.0, 1.0)
            rng = max(hi - lo, 1e-6)
            for slot, v in sc:
                agg.setdefault(slot, 0.0)
                if v == -math.inf:
                    veto.add(slot)
                elif v == math.inf:
                    first.add(slot)
                    agg[slot] += w / total_w          # counts as this policy's maximum
                else:
                    agg[slot] += (v - lo) / rng * w / total_w
        out = []
        for slot, v in agg.items():
            if slot in veto:
                out.append((slot, -math.inf))
            elif slot in first:
                out.append((slot, math.inf))
            else:
                out.append((slot, v))
        return _sorted(out)

    def select_eviction_candidate(self, positions: Dict[int, int]) -> Optional[int]:
        s = self.compute_aggregated_scores(positions)
        return s[0][0] if s and s[0][1] != -math.inf else None

    def select_evictions(self, positions: Dict[int, int], n: int) -> List[int]:
        """Up to ``n`` slots in eviction order, never a vetoed one."""
        return [s for s, v in self.compute_aggregated_scores(positions) if v != -math.inf][:n]


def keep_list(positions: Sequence[int], evict: Sequence[int]) -> List[int]:
    """Positions to keep (in order) after evicting ``evict``."""
    e = set(evict)
    return [p for p in positions if p not in e]
