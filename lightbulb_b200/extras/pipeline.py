"""Multi-stage generation pipelines: a DAG of stages (decompose, identify, generate, verify,
synthesize, custom), each rendered from a prompt template over its dependencies' outputs and
run by a caller-supplied executor (e.g. ``lambda prompt, stage: engine.generate(...)``).

Reference: ``src/engine/pipeline.rs:65-672`` (stage types and states, dependency validation,
cycle detection, parallel execution of independent stages under a concurrency limit, KV-cache
sharing between a stage and its dependents, statistics).  Here independent stages of a level
run on a thread pool of ``max_concurrent_stages`` workers; "cache sharing" means a stage's
prompt starts with its first dependency's output, so the engine's prefix cache reuses that
dependency's KV blocks; a failed stage marks its dependents skipped rather than aborting the
whole run.
"""
from __future__ import annotations

import enum
import time
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional


class PipelineError(RuntimeError):
    pass


class StageType(str, enum.Enum):
    DECOMPOSE = "decompose"
    IDENTIFY = "identify"
    GENERATE = "generate"
    VERIFY = "verify"
    SYNTHESIZE = "synthesize"
    CUSTOM = "custom"


class StageState(str, enum.Enum):
    PENDING = "pending"
    RUNNING = "running"
    COMPLETED = "completed"
    FAILED = "failed"
    SKIPPED = "skipped"


@dataclass
class Stage:
    id: str
    type: StageType = StageType.GENERATE
    depends_on: List[str] = field(default_factory=list)
    prompt_template: str = "{input}"      # fields: {input}, {deps}, and {<dependency id>}
    max_tokens: int = 256
    temperature: float = 0.0
    share_cache: bool = True


@dataclass
class StageResult:
    stage_id: str
    output: str
    elapsed_ms: float
    cache_shared: bool = False
    error: Optional[str] = None


@dataclass
class PipelineConfig:
    max_concurrent_stages: int = 4
    enable_cache_sharing: bool = True
    timeout_s: Optional[float] = 300.0
    parallel: bool = True


@dataclass
class PipelineStats:
    total_ms: float = 0.0
    stages_executed: int = 0
    parallel_stages: int = 0        # stages that ran in a level with others
    cache_shared: int = 0
    failed: int = 0


class Pipeline:
    def __init__(self, id: str = "pipeline", config: Optional[PipelineConfig] = None):
        self.id = id
        self.config = config or PipelineConfig()
        self.stages: Dict[str, Stage] = {}
        self.state: Dict[str, StageState] = {}
        self.results: Dict[str, StageResult] = {}
        self.stats = PipelineStats()

    def add(self, stage: Stage) -> "Pipeline":
        if stage.id in self.stages:
            raise PipelineError(f"duplicate stage {stage.id}")
        self.stages[stage.id] = stage
        self.state[stage.id] = StageState.PENDING
        return self

    def levels(self) -> List[List[str]]:
        """Stages grouped by dependency depth (each level only needs earlier levels)."""
        if not self.stages:
            raise PipelineError("no stages defined")
        for s in self.stages.values():
            for d in s.depends_on:
                if d not in self.stages:
                    raise PipelineError(f"stage {s.id} depends on unknown stage {d}")
        done: set = set()
        out: List[List[str]] = []
        while len(done) < len(self.stages):
            lvl = [i for i, s in self.stages.items()
                   if i not in done and all(d in done for d in s.depends_on)]
            if not lvl:
                raise PipelineError("circular dependency in pipeline")
            out.append(lvl)
            done.update(lvl)
        return out

    def _prompt(self, s: Stage, user_input: str) -> str:
        deps = {d: self.results[d].output for d in s.depends_on}
        body = s.prompt_template.format(input=user_input, deps="\n\n".join(deps.values()),
                                        **deps)
        if self.config.enable_cache_sharing and s.share_cache and s.depends_on:
            first = deps[s.depends_on[0]]
            if not body.startswith(first):
                body = first + "\n\n" + body      # shared prefix: KV reused by the engine
        return body

    def run(self, user_input: str, execute: Callable[[str, Stage], str]) -> Dict[str, StageResult]:
        levels = self.levels()
        t0 = time.perf_counter()
        workers = max(1, self.config.max_concurrent_stages if self.config.parallel else 1)
        with ThreadPoolExecutor(max_workers=workers) as pool:
            for lvl in levels:
                runnable = []
                for sid in lvl:
                    s = self.stages[sid]
                    if any(self.state[d] != StageState.COMPLETED for d in s.depends_on):
                        self.state[sid] = StageState.SKIPPED
                    else:
                        runnable.append(s)
                futures = {}
                for s in runnable:
                    self.state[s.id] = StageState.RUNNING
                    futures[s.id] = (pool.submit(self._run_one, s, user_input, execute))
                for sid, f in futures.items():
                    left = None
                    if self.config.timeout_s is not None:
                        left = max(0.0, self.config.timeout_s - (time.perf_counter() - t0))
                    try:
                        r = f.result(timeout=left)
                    except Exception as e:          # timeout or executor failure
                        r = StageResult(sid, "", 0.0, error=f"{type(e).__name__}: {e}")
                    self.results[sid] = r
                    self.state[sid] = StageState.FAILED if r.error else StageState.COMPLETED
                    self.stats.stages_executed += 1
                    self.stats.failed += r.error is not None
                    self.stats.cache_shared += r.cache_shared
                if len(futures) > 1:
                    self.stats.parallel_stages += len(futures)
        self.stats.total_ms = (time.perf_counter() - t0) * 1e3
        return self.results

    def _run_one(self, s: Stage, user_input: str, execute) -> StageResult:
        t = time.perf_counter()
        try:
            prompt = self._prompt(s, user_input)
            out = execute(prompt, s)
            shared = bool(self.config.enable_cache_sharing and s.share_cache and s.depends_on)
            return StageResult(s.id, out, (time.perf_counter() - t) * 1e3, shared)
        except Exception as e:
            return StageResult(s.id, "", (time.perf_counter() - t) * 1e3,
                               error=f"{type(e).__name__}: {e}")


def engine_executor(engine, **sampling) -> Callable[[str, Stage], str]:
    """Executor running each stage through :class:`LLMEngine` (greedy unless overridden).
    ``LLMEngine.generate`` is not re-entrant, so parallel stages take turns on it; stages that
    should share batches go through the asynchronous engine instead."""
    import threading

    from ..engine.sampling import SamplingParams
    lock = threading.Lock()

    def run(prompt: str, stage: Stage) -> str:
        sp = SamplingParams(temperature=stage.temperature, max_tokens=stage.max_tokens,
                            **sampling)
        with lock:
            seq = engine.generate(prompt, sp)[0]
            return seq.output_text or engine.tokenizer.decode(seq.output_token_ids)
    return run
