"""Request / sequence state.

Mirrors the reference's ``Request``/``RequestState``/``RequestContext``
(``src/engine/mod.rs:111-265``) and finish semantics (``src/engine/model_runner.rs:21-83``:
``"stop"`` on EOS or a stop string, otherwise ``"length"``), with the timing fields needed
for TTFT / ITL.
"""
from __future__ import annotations

import enum
import itertools
import time
from dataclasses import dataclass, field
from typing import List, Optional

from .sampling import SamplingParams

_seq_ids = itertools.count()
PENDING_TOKEN = -1   # output slot whose id is still on the device (overlapped decode)


class SeqStatus(enum.Enum):
    WAITING = "waiting"
    RUNNING = "running"
    AWAITING_TOOL = "awaiting_tool_result"
    FINISHED = "finished"


@dataclass(eq=False)
class Sequence:
    request_id: str
    prompt_token_ids: List[int]
    params: SamplingParams
    seq_id: int = field(default_factory=lambda: next(_seq_ids))
    output_token_ids: List[int] = field(default_factory=list)
    status: SeqStatus = SeqStatus.WAITING
    num_computed_tokens: int = 0     # tokens whose KV is in the cache
    num_cached_prefix: int = 0       # tokens reused from the prefix cache
    finish_reason: Optional[str] = None
    arrival_time: float = field(default_factory=time.perf_counter)
    first_token_time: Optional[float] = None
    token_times: List[float] = field(default_factory=list)
    priority: int = 1                # 0 low .. 3 critical (memory_aware_scheduler.rs:34-88)
    output_text: str = ""
    logprobs: List[float] = field(default_factory=list)
    max_new_tokens: int = 0          # budget after context truncation
    truncated: bool = False
    preemptions: int = 0
    evicted: int = 0                 # tokens dropped from the KV cache (compression)
    # speculative decoding
    spec_draft_tokens: List[int] = field(default_factory=list)
    # tool calls: the pending call while AWAITING_TOOL, context tokens injected afterwards
    pending_tool_call: Optional[dict] = None
    injected_tokens: int = 0
    tool_scan_from: int = 0          # output_text offset already scanned for tool calls
    # overlapped decode: the newest output is a placeholder (PENDING_TOKEN) until its step's
    # ids are read back; `hold` keeps a sequence that is about to finish out of the next step
    hold: bool = False

    def __post_init__(self) -> None:
        # prompt + generated ids in one list, appended in place (never rebuilt per step)
        self._tokens: List[int] = list(self.prompt_token_ids) + list(self.output_token_ids)

    def append_output(self, tok: int) -> None:
        self.output_token_ids.append(tok)
        self._tokens.append(tok)

    def append_placeholder(self):
        """Append a PENDING_TOKEN output; returns its (output index, token-list index)."""
        self.append_output(PENDING_TOKEN)
        return len(self.output_token_ids) - 1, len(self._tokens) - 1

    def set_output(self, out_idx: int, tok_idx: int, tok: int) -> None:
        """Fill a placeholder appended by :meth:`append_placeholder`."""
        self.output_token_ids[out_idx] = tok
        self._tokens[tok_idx] = tok

    def truncate_output(self, n: int) -> None:
        """Keep the first ``n`` generated tokens (speculative rollback of the newest outputs,
        which are always at the end of the token list)."""
        k = len(self.output_token_ids) - n
        if k > 0:
            del self.output_token_ids[n:]
            del self._tokens[len(self._tokens) - k:]

    def append_context(self, ids: List[int]) -> None:
        """Context tokens that are not model outputs (a tool's result): fed through the model
        as a mini-prefill into the preserved KV, never counted as generated tokens."""
        self._tokens.extend(ids)
        self.injected_tokens += len(ids)

    @property
    def all_token_ids(self) -> List[int]:
        return self._tokens

    @property
    def last_token(self) -> int:
        return self._tokens[-1]

    @property
    def num_tokens(self) -> int:
        return len(self._tokens)

    @property
    def prompt_len(self) -> int:
        return len(self.prompt_token_ids)

    @property
    def num_uncomputed(self) -> int:
        """Tokens still to feed through the model (1 in steady decode, more in prefill)."""
        return self.num_tokens - self.evicted - self.num_computed_tokens

    @property
    def is_prefilling(self) -> bool:
        return self.num_uncomputed > 1

    @property
    def finished(self) -> bool:
        return self.status == SeqStatus.FINISHED

    def ttft(self) -> Optional[float]:
        return None if self.first_token_time is None else self.first_token_time - self.arrival_time

    def itls(self) -> List[float]:
        t = self.token_times
        return [t[i] - t[i - 1] for i in range(1, len(t))]


def finish_reason_for(stopped_on_eos: bool) -> str:
    """``src/engine/model_runner.rs:77``: EOS/stop -> "stop", budget exhausted -> "length"."""
    return "stop" if stopped_on_eos else "length"


def effective_generation_budget(prompt_len: int, max_new: int, context_length: int):
    """Cap generation to what fits in the context (``src/model_fuel/engine_model.rs:56-104``).
    Returns (budget, truncated)."""
    room = max(0, context_length - prompt_len)
    if max_new > room:
        return room, True
    return max_new, False
