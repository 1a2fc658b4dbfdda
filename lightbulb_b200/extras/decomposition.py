"""Problem decomposition over a knowledge base (host-side planning, no tensors).

Reference: ``src/engine/decomposition.rs:87-900``.  A problem lists the facts it needs; facts
already in the knowledge base are filled in, and the share of known facts (coverage) picks the
strategy:

* atomic        nothing to find and the problem is at most Simple: no sub-problems;
* computational coverage >= 0.9: one "compute" step;
* hybrid        coverage >= 0.5: one "find" step per missing fact, then a compute step that
                depends on all of them;
* structural    otherwise: one "find" step per required fact.

Sub-problems form a DAG; the plan exposes a topological order and the parallel levels (every
step whose dependencies are done runs in the same level).  The engine keeps a history, can
re-plan a problem after the knowledge base grew, and scores alternative formulations of a
problem on copies of its state (the reference branches JSON checkpoints for this).
"""
from __future__ import annotations

import copy
import enum
import itertools
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

from .knowledge import KnowledgeBase

_ids = itertools.count(1)


class DecompositionError(Exception):
    pass


class Strategy(str, enum.Enum):
    STRUCTURAL = "structural"
    COMPUTATIONAL = "computational"
    ATOMIC = "atomic"
    HYBRID = "hybrid"


class Complexity(enum.IntEnum):
    TRIVIAL = 0
    SIMPLE = 1
    MODERATE = 2
    COMPLEX = 3
    VERY_COMPLEX = 4

    @property
    def weight(self) -> float:
        return float(2 ** int(self))        # 1, 2, 4, 8, 16


@dataclass
class Problem:
    description: str
    required_facts: List[str] = field(default_factory=list)
    known_facts: Dict[str, str] = field(default_factory=dict)
    complexity: Complexity = Complexity.MODERATE
    metadata: Dict[str, str] = field(default_factory=dict)
    id: str = field(default_factory=lambda: f"prob_{next(_ids)}")
    created_at: float = field(default_factory=time.time)

    # builder helpers
    def requires(self, fact: str) -> "Problem":
        self.required_facts.append(fact)
        return self

    def with_known_fact(self, key: str, value: str) -> "Problem":
        self.known_facts[key] = value
        return self

    def with_complexity(self, c: Complexity) -> "Problem":
        self.complexity = c
        return self

    def is_atomic(self) -> bool:
        return not self.required_facts and self.complexity <= Complexity.SIMPLE

    def knowledge_coverage(self) -> float:
        if not self.required_facts:
            return 1.0
        return sum(f in self.known_facts for f in self.required_facts) / len(self.required_facts)


@dataclass
class SubProblem:
    id: str
    description: str
    depends_on: List[str] = field(default_factory=list)
    produces: List[str] = field(default_factory=list)
    success_criteria: List[str] = field(default_factory=list)
    complexity: Complexity = Complexity.SIMPLE


@dataclass
class Decomposition:
    problem: Problem
    sub_problems: List[SubProblem]
    strategy: Strategy
    depth: int = 0
    parallel_groups: List[List[str]] = field(default_factory=list)
    created_at: float = field(default_factory=time.time)

    @property
    def dependencies(self) -> Dict[str, List[str]]:
        return {s.id: list(s.depends_on) for s in self.sub_problems}

    def is_atomic(self) -> bool:
        return not self.sub_problems

    def execution_order(self) -> List[str]:
        """Topological order (Kahn); ties are broken by declaration order so the plan is
        deterministic.  Raises on a cycle or an unknown dependency."""
        ids = [s.id for s in self.sub_problems]
        known = set(ids)
        indeg = {i: 0 for i in ids}
        children: Dict[str, List[str]] = {i: [] for i in ids}
        for s in self.sub_problems:
            for d in s.depends_on:
                if d not in known:
                    raise DecompositionError(f"{s.id} depends on unknown step {d}")
                children[d].append(s.id)
                indeg[s.id] += 1
        ready = [i for i in ids if indeg[i] == 0]
        order: List[str] = []
        while ready:
            n = ready.pop(0)
            order.append(n)
            for c in children[n]:
                indeg[c] -= 1
                if indeg[c] == 0:
                    ready.append(c)
        if len(order) != len(ids):
            raise DecompositionError("dependency cycle in decomposition")
        return order

    def compute_parallel_groups(self) -> List[List[str]]:
        self.execution_order()                      # validates the DAG
        done: set = set()
        groups: List[List[str]] = []
        while len(done) < len(self.sub_problems):
            level = [s.id for s in self.sub_problems
                     if s.id not in done and all(d in done for d in s.depends_on)]
            groups.append(level)
            done.update(level)
        self.parallel_groups = groups
        return groups

    def complexity_score(self) -> float:
        """Product of the problem's complexity weight and factors for the number of steps,
        the depth, the unknowns and the dependency edges (higher = harder)."""
        edges = sum(len(s.depends_on) for s in self.sub_problems)
        return (self.problem.complexity.weight * (1 + 0.5 * len(self.sub_problems)) *
                (1 + 0.3 * self.depth) * (1 + 0.4 * len(self.problem.required_facts)) *
                (1 + 0.2 * edges))


@dataclass
class DecompositionConfig:
    max_depth: int = 5
    max_sub_problems: int = 10
    min_coverage_for_redecomp: float = 0.7
    auto_redecompose: bool = True
    track_history: bool = True


@dataclass
class HistoryEntry:
    problem: str
    strategy: Strategy
    sub_problem_count: int
    depth: int
    coverage: float
    was_redecomposed: bool = False
    success: bool = False
    timestamp: float = field(default_factory=time.time)


class DecompositionEngine:
    def __init__(self, kb: Optional[KnowledgeBase] = None,
                 config: Optional[DecompositionConfig] = None):
        self.kb = kb if kb is not None else KnowledgeBase()
        self.config = config or DecompositionConfig()
        self.history: List[HistoryEntry] = []
        self.active: Dict[str, Decomposition] = {}

    # -------------------------------------------------------------------------------
    def decompose(self, problem: Problem, depth: int = 0) -> Decomposition:
        if depth > self.config.max_depth:
            raise DecompositionError(f"maximum decomposition depth {self.config.max_depth} "
                                     f"exceeded ({depth})")
        self._enrich(problem)
        strategy = self.strategy_for(problem)
        subs = self._plan(problem, strategy)
        if len(subs) > self.config.max_sub_problems:
            raise DecompositionError(f"{len(subs)} sub-problems exceed the limit "
                                     f"{self.config.max_sub_problems}")
        d = Decomposition(problem, subs, strategy, depth)
        d.compute_parallel_groups()
        if self.config.track_history:
            self.history.append(HistoryEntry(problem.description, strategy, len(subs), depth,
                                             problem.knowledge_coverage()))
        self.active[problem.id] = d
        return d

    def _enrich(self, problem: Problem) -> None:
        for fact in problem.required_facts:
            if fact not in problem.known_facts:
                f = self.kb.get(fact)
                if f is not None:
                    problem.known_facts[fact] = f.content

    @staticmethod
    def strategy_for(problem: Problem) -> Strategy:
        if problem.is_atomic():
            return Strategy.ATOMIC
        cov = problem.knowledge_coverage()
        if cov >= 0.9:
            return Strategy.COMPUTATIONAL
        if cov >= 0.5:
            return Strategy.HYBRID
        return Strategy.STRUCTURAL

    @staticmethod
    def _plan(p: Problem, strategy: Strategy) -> List[SubProblem]:
        if strategy == Strategy.ATOMIC:
            return []
        compute = SubProblem(f"{p.id}:compute", f"Compute: {p.description}",
                             success_criteria=["Calculation complete"])
        if strategy == Strategy.COMPUTATIONAL:
            return [compute]
        if strategy == Strategy.STRUCTURAL:
            return [SubProblem(f"{p.id}:sub{i}", f"Find {f}", produces=[f],
                               success_criteria=[f"{f} is known"])
                    for i, f in enumerate(p.required_facts)]
        finds = [SubProblem(f"{p.id}:find{i}", f"Find {f}", produces=[f])
                 for i, f in enumerate(p.required_facts) if f not in p.known_facts]
        compute.depends_on = [s.id for s in finds]
        compute.success_criteria = []
        return finds + [compute]

    # -------------------------------------------------------------------------------
    def should_redecompose(self, problem_id: str) -> bool:
        d = self.active.get(problem_id)
        if not self.config.auto_redecompose or d is None:
            return False
        self._enrich(d.problem)
        return (d.problem.knowledge_coverage() >= self.config.min_coverage_for_redecomp and
                d.strategy not in (Strategy.COMPUTATIONAL, Strategy.ATOMIC))

    def redecompose(self, problem_id: str) -> Decomposition:
        d = self.active.get(problem_id)
        if d is None:
            raise DecompositionError(f"problem {problem_id} not found")
        nd = self.decompose(copy.deepcopy(d.problem), d.depth)
        if self.history:
            self.history[-1].was_redecomposed = True
        return nd

    def mark_success(self, problem_id: str, success: bool = True) -> None:
        desc = self.active[problem_id].problem.description if problem_id in self.active else None
        for h in reversed(self.history):
            if h.problem == desc:
                h.success = success
                break

    def stats(self) -> dict:
        n = len(self.history)
        return {
            "total_decompositions": n,
            "structural_count": sum(h.strategy == Strategy.STRUCTURAL for h in self.history),
            "computational_count": sum(h.strategy == Strategy.COMPUTATIONAL
                                       for h in self.history),
            "redecomposition_count": sum(h.was_redecomposed for h in self.history),
            "average_coverage": sum(h.coverage for h in self.history) / n if n else 0.0,
            "active_decompositions": len(self.active),
        }

    @staticmethod
    def score(d: Decomposition) -> float:
        """Higher is better: coverage bonus (2 x), +5 for atomic plans, -0.1 per step and
        -0.05 per dependency edge."""
        edges = sum(len(v) for v in d.dependencies.values())
        return (2.0 * d.problem.knowledge_coverage() + (5.0 if d.is_atomic() else 0.0)
                - 0.1 * len(d.sub_problems) - 0.05 * edges)

    def explore_variants(self, variants: List[Problem]) -> List[Tuple[Problem, Decomposition, float]]:
        """Plan each formulation on an isolated copy of this engine's state (knowledge base,
        history, active plans) and return them best first; this engine is left unchanged."""
        out = []
        for p in variants:
            branch = DecompositionEngine(copy.deepcopy(self.kb), self.config)
            branch.history = copy.deepcopy(self.history)
            branch.active = copy.deepcopy(self.active)
            d = branch.decompose(copy.deepcopy(p))
            out.append((p, d, self.score(d)))
        out.sort(key=lambda x: -x[2])
        return out
