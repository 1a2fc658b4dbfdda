"""Prometheus text exposition (``/metrics``) and the admin metrics snapshot.

The reference's admin metrics return zeros (``src/api/admin.rs:184-194``); these come from
the live engine: request/token counters, TTFT / ITL quantiles and histograms, KV block usage,
prefix-cache hit rate, speculative acceptance and step count.
"""
from __future__ import annotations

import statistics
import threading
from typing import Dict, List


def _q(vals, p: float) -> float:
    if hasattr(vals, "snapshot"):
        vals = vals.snapshot()            # a consistent copy taken under the writer's lock
    if not vals:
        return 0.0
    s = sorted(vals)
    return s[min(len(s) - 1, int(p * len(s)))]


from ..engine.llm_engine import ITL_BUCKETS, TTFT_BUCKETS  # noqa: F401  (re-exported)


def _histogram(name: str, vals: List[float], bounds) -> List[str]:
    """Prometheus histogram lines: cumulative bucket counts, sum and count."""
    s = sorted(vals)
    out = [f"# TYPE {name} histogram"]
    i = 0
    for b in bounds:
        while i < len(s) and s[i] <= b:
            i += 1
        out.append(f'{name}_bucket{{le="{b}"}} {i}')
    out.append(f'{name}_bucket{{le="+Inf"}} {len(s)}')
    out.append(f"{name}_sum {sum(s)}")
    out.append(f"{name}_count {len(s)}")
    return out


def _histogram_cumulative(name: str, st) -> List[str]:
    """Histogram lines from cumulative counts kept since start (:class:`LatencySamples`)."""
    out = [f"# TYPE {name} histogram"]
    c = 0
    for b, n in zip(st.bounds, st.bucket_counts):
        c += n
        out.append(f'{name}_bucket{{le="{b}"}} {c}')
    out.append(f'{name}_bucket{{le="+Inf"}} {st.total}')
    out.append(f"{name}_sum {st.sum}")
    out.append(f"{name}_count {st.total}")
    return out


class Metrics:
    def __init__(self):
        self.lock = threading.Lock()
        self.requests: Dict[str, int] = {}
        self.errors = 0

    def count(self, route: str):
        with self.lock:
            self.requests[route] = self.requests.get(route, 0) + 1

    def snapshot(self, engine=None) -> dict:
        d = {"requests": dict(self.requests), "errors": self.errors}
        if engine is not None:
            st = engine.stats
            d.update({
                "steps": st.steps, "prompt_tokens": st.prompt_tokens,
                "generated_tokens": st.generated_tokens, "finished": st.finished,
                "ttft_p50_s": _q(st.ttfts, 0.5), "ttft_p99_s": _q(st.ttfts, 0.99),
                "itl_p50_s": _q(st.itls, 0.5), "itl_p99_s": _q(st.itls, 0.99),
                "kv_blocks_total": engine.blocks.num_blocks,
                "kv_blocks_free": engine.blocks.num_free_blocks(),
                "kv_usage": engine.blocks.usage(),
                "prefix_hit_rate": engine.blocks.prefix_hit_rate(),
                "running": len(engine.scheduler.running),
                "waiting": len(engine.scheduler.waiting),
                "preemptions": engine.scheduler.num_preemptions,
            })
            if engine.spec is not None:
                d["spec_acceptance"] = engine.spec.stats.acceptance_rate()
        return d

    def prometheus(self, engine=None) -> str:
        s = self.snapshot(engine)
        lines = []
        for route, n in s["requests"].items():
            lines.append(f'lb_requests_total{{route="{route}"}} {n}')
        lines.append(f"lb_errors_total {s['errors']}")
        for k in ("steps", "prompt_tokens", "generated_tokens", "finished", "ttft_p50_s",
                  "ttft_p99_s", "itl_p50_s", "itl_p99_s", "kv_blocks_total", "kv_blocks_free",
                  "kv_usage", "prefix_hit_rate", "running", "waiting", "preemptions",
                  "spec_acceptance"):
            if k in s:
                lines.append(f"lb_{k} {s[k]}")
        if engine is not None:
            for name, st in (("lb_ttft_seconds", engine.stats.ttfts),
                             ("lb_itl_seconds", engine.stats.itls)):
                lines += _histogram_cumulative(name, st) if hasattr(st, "bucket_counts") \
                    else _histogram(name, list(st), TTFT_BUCKETS if "ttft" in name
                                    else ITL_BUCKETS)
        return "\n".join(lines) + "\n"
