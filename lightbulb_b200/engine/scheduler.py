"""Continuous-batching scheduler.

Replaces the reference's one-request-at-a-time runner loop (``src/engine/model_runner.rs:383-398``),
its fixed ``SlotPool`` (``src/engine/slot_pool.rs``), the byte-estimate
``MemoryAwareScheduler`` (``src/engine/memory_aware_scheduler.rs:142-337``) and the chunked
prefill scheduler (``src/model/chunked_prefill.rs:60-330``, chunk 512) with one step planner:

1. every running sequence in decode gets one token (decode first keeps ITL low); if the
   block pool is exhausted the most recently admitted sequence is preempted (its blocks are
   freed and it is recomputed later, prefix cache permitting);
2. partially prefilled sequences continue with chunks of at most ``chunk_size`` tokens;
3. waiting requests are admitted by priority then arrival while the token budget and the
   sequence limit allow; admission checks block availability for the chunk it schedules
   (all-or-nothing per sequence, ``src/model_fuel/batched.rs:617-664``) and first reuses
   the longest cached prefix (``src/model_fuel/policies.rs:442-600``).

Memory admission is by KV blocks, not byte estimates; priorities (Low..Critical) order the
waiting queue as in the reference.
"""
from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass, field
from typing import Deque, List, Optional, Tuple

from ..config import SchedulerConfig
from ..kv.block_manager import BlockManager
from .sequence import Sequence, SeqStatus


@dataclass
class ScheduledChunk:
    seq: Sequence
    start: int          # first token index fed this step
    num_tokens: int     # tokens fed this step
    slots: List[int]
    needs_logits: bool  # chunk reaches the end of the known tokens -> sample
    logits_all: bool = False  # sample every row of the chunk (speculative verify)


@dataclass
class SchedulerOutput:
    decode: List[ScheduledChunk] = field(default_factory=list)
    prefill: List[ScheduledChunk] = field(default_factory=list)
    cow_pairs: List[int] = field(default_factory=list)
    preempted: List[Sequence] = field(default_factory=list)

    @property
    def chunks(self) -> List[ScheduledChunk]:
        return self.decode + self.prefill

    @property
    def num_tokens(self) -> int:
        return sum(c.num_tokens for c in self.decode) + sum(c.num_tokens for c in self.prefill)

    @property
    def empty(self) -> bool:
        return not self.decode and not self.prefill


class Scheduler:
    def __init__(self, cfg: SchedulerConfig, blocks: BlockManager, watermark_blocks: int = 0):
        self.cfg = cfg
        self.blocks = blocks
        self.waiting: Deque[Sequence] = deque()
        self.running: List[Sequence] = []
        self.watermark = watermark_blocks
        self.num_preemptions = 0

    # ---------------------------------------------------------------------------------
    def add(self, seq: Sequence) -> None:
        seq.status = SeqStatus.WAITING
        # priority order: higher priority first, FIFO within a priority
        if seq.priority > 1:
            idx = 0
            for i, s in enumerate(self.waiting):
                if s.priority < seq.priority:
                    idx = i
                    break
                idx = i + 1
            self.waiting.insert(idx, seq)
        else:
            self.waiting.append(seq)

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    def abort(self, request_id: str) -> Optional[Sequence]:
        for s in list(self.waiting):
            if s.request_id == request_id:
                self.waiting.remove(s)
                s.status = SeqStatus.FINISHED
                s.finish_reason = s.finish_reason or "abort"
                return s
        for s in list(self.running):
            if s.request_id == request_id:
                self.finish(s, "abort")
                return s
        return None

    def finish(self, seq: Sequence, reason: str) -> None:
        seq.status = SeqStatus.FINISHED
        seq.finish_reason = reason
        if seq in self.running:
            self.running.remove(seq)
        if self.blocks.has_seq(seq.seq_id):
            self.blocks.free_sequence(seq.seq_id)

    def _preempt(self, out: SchedulerOutput) -> bool:
        """Free the most recently admitted running sequence (recompute later)."""
        if not self.running:
            return False
        victim = self.running.pop()
        self.blocks.free_sequence(victim.seq_id)
        victim.num_computed_tokens = 0
        victim.evicted = 0  # compressed KV is rebuilt from the full token list
        victim.status = SeqStatus.WAITING
        victim.preemptions += 1
        self.waiting.appendleft(victim)
        out.preempted.append(victim)
        self.num_preemptions += 1
        for lst in (out.decode, out.prefill):
            for c in list(lst):
                if c.seq is victim:
                    lst.remove(c)
        return True

    # ---------------------------------------------------------------------------------
    def schedule(self) -> SchedulerOutput:
        out = SchedulerOutput()
        budget = self.cfg.max_num_batched_tokens
        bm = self.blocks

        # 1) decode tokens for running sequences
        i = 0
        while i < len(self.running):
            seq = self.running[i]
            if seq.status == SeqStatus.AWAITING_TOOL or seq.num_uncomputed != 1 or seq.hold:
                i += 1
                continue
            if budget <= 0:
                break
            while bm.blocks_needed(seq.seq_id, 1) > bm.num_free_blocks():
                if not self._preempt(out) or seq not in self.running:
                    break
            if seq not in self.running:
                continue
            # a pending id (overlapped decode, < 0) is recorded once it is known (set_tokens)
            last = seq.last_token
            slots, cow = bm.append_slots(seq.seq_id, 1, [last] if last >= 0 else [])
            out.cow_pairs += cow
            out.decode.append(ScheduledChunk(seq, seq.num_computed_tokens, 1, slots, True))
            budget -= 1
            i += 1

        # 2) continue partial prefills
        for seq in list(self.running):
            if budget <= 0:
                break
            if seq.num_uncomputed <= 1 or seq.status == SeqStatus.AWAITING_TOOL:
                continue
            n = min(seq.num_uncomputed, budget)
            if self.cfg.enable_chunked_prefill:
                n = min(n, self.cfg.chunk_size)
            elif n < seq.num_uncomputed:
                continue
            if bm.blocks_needed(seq.seq_id, n) > bm.num_free_blocks():
                continue
            out.prefill.append(self._prefill_chunk(seq, n, out))
            budget -= n

        # 3) admit waiting sequences
        while self.waiting and budget > 0 and len(self.running) < self.cfg.max_num_seqs:
            seq = self.waiting[0]
            new = not bm.has_seq(seq.seq_id)
            if new:
                bm.add_sequence(seq.seq_id)
                if seq.num_computed_tokens == 0:
                    cached = bm.match_prefix(seq.seq_id, seq.all_token_ids)
                    seq.num_computed_tokens = cached
                    seq.num_cached_prefix = max(seq.num_cached_prefix, cached)
            n = min(seq.num_uncomputed, budget)
            if self.cfg.enable_chunked_prefill:
                n = min(n, self.cfg.chunk_size)
            elif n < seq.num_uncomputed:
                if new:
                    bm.free_sequence(seq.seq_id)
                    seq.num_computed_tokens = 0
                break
            need = bm.blocks_needed(seq.seq_id, n)
            if need + (self.watermark if self.running else 0) > bm.num_free_blocks():
                if new:
                    bm.free_sequence(seq.seq_id)
                    seq.num_computed_tokens = 0
                break
            self.waiting.popleft()
            seq.status = SeqStatus.RUNNING
            self.running.append(seq)
            if n == 1 and seq.num_uncomputed == 1:
                slots, cow = bm.append_slots(seq.seq_id, 1, [seq.last_token])
                out.cow_pairs += cow
                out.prefill.append(ScheduledChunk(seq, seq.num_computed_tokens, 1, slots, True))
            else:
                out.prefill.append(self._prefill_chunk(seq, n, out))
            budget -= n
        return out

    def _prefill_chunk(self, seq: Sequence, n: int, out: SchedulerOutput) -> ScheduledChunk:
        start = seq.num_computed_tokens          # KV index
        t0 = start + seq.evicted                 # token index
        toks = seq.all_token_ids[t0:t0 + n]
        slots, cow = self.blocks.append_slots(seq.seq_id, n, toks)
        out.cow_pairs += cow
        return ScheduledChunk(seq, start, n, slots, t0 + n == seq.num_tokens)
