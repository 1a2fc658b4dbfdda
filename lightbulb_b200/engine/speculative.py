"""Speculative decoding: a small draft model proposes k tokens, the target verifies them in
ONE batched forward.

Reference: ``src/engine/speculative.rs:30-320`` drafts k tokens sequentially and verifies with
k separate target forwards (``:241-259``), accepts the longest prefix on which draft and
target agree plus the target's correction, and falls back to plain decoding when acceptance
stays below 0.3 after 10 rounds.  Here:

* the draft has its own paged KV pool, block manager and model runner (CUDA graphs for its
  one-token steps); it catches up on tokens it has not seen (prompt, corrections) first;
* the target runs ONE forward over k+1 tokens per sequence through the paged prefill
  kernel (causal within the chunk) and samples every row;
* acceptance: every row r is sampled with the seed of output index ``len(outputs) + r``
  (the seed the non-speculative path would use); tokens are taken from the target's samples up
  to and including the first row whose sample differs from the draft's proposal.  Greedy
  requests get exactly greedy-equality acceptance; sampled requests get exactly the tokens
  plain decoding would emit for the same seeds.  The draft samples with the same seeds
  (coupled draws), so similar distributions agree often;
* rejected KV is rolled back with block-manager truncation (target and draft);
* statistics and the reference's auto-fallback (acceptance < ``min_acceptance`` after
  ``fallback_after_rounds`` rounds -> plain decoding).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional

from .scheduler import ScheduledChunk, SchedulerOutput


@dataclass
class SpecStats:
    rounds: int = 0
    proposed: int = 0
    accepted: int = 0
    emitted: int = 0
    draft_s: float = 0.0
    verify_s: float = 0.0

    def acceptance_rate(self) -> float:
        return self.accepted / self.proposed if self.proposed else 0.0


class _SeqView:
    """A runner's view of a target sequence with extra (proposed) tokens appended.

    ``outputs_len`` is the output index of the first row the runner samples (it selects
    that row's seed): for the draft it counts the proposals so far, for the target verify
    only the real outputs."""

    def __init__(self, seq, tokens: List[int], outputs_len: int):
        self.seq_id = seq.seq_id
        self.request_id = seq.request_id
        self.params = seq.params
        self._tokens = tokens
        self._n_out = outputs_len

    @property
    def all_token_ids(self):
        return self._tokens

    @property
    def last_token(self):
        return self._tokens[-1]

    @property
    def output_token_ids(self):
        return range(self._n_out)


class SpeculativeDecoder:
    def __init__(self, engine, draft_runner, draft_blocks, k: int = 4,
                 min_acceptance: float = 0.3, fallback_after: int = 10):
        self.engine = engine
        self.draft = draft_runner
        self.dbm = draft_blocks
        self.k = k
        self.min_acc = min_acceptance
        self.fallback_after = fallback_after
        self.active = True
        self.stats = SpecStats()
        self.draft_len: Dict[int, int] = {}  # seq_id -> tokens with draft KV

    # ------------------------------------------------------------------------------
    def _draft_register(self, seq):
        if not self.dbm.has_seq(seq.seq_id):
            self.dbm.add_sequence(seq.seq_id)
            self.draft_len[seq.seq_id] = 0

    def _draft_release(self, seq):
        if self.dbm.has_seq(seq.seq_id):
            self.dbm.free_sequence(seq.seq_id)
        self.draft_len.pop(seq.seq_id, None)

    def step(self, eng):
        so = eng.scheduler.schedule()
        if so.empty:
            return []
        if so.prefill or not self.active:
            res = eng.runner.execute(so)
            if self.active:
                self._mirror(so)
            outs = eng._process(res.chunks, res.tokens)
            self._sweep(eng)
            return outs
        return self._spec_round(eng, so)

    def _mirror(self, so: SchedulerOutput):
        """Feed the tokens the target just consumed to the draft (keeps its KV in step with
        the prompt, bounded by the scheduler's token budget)."""
        chunks = []
        for c in so.decode + so.prefill:
            s = c.seq
            self._draft_register(s)
            start = self.draft_len[s.seq_id]
            end = c.start + c.num_tokens
            if end <= start:
                continue
            toks = s.all_token_ids
            slots, cow = self.dbm.append_slots(s.seq_id, end - start, toks[start:end])
            if cow:
                self.draft.kv.copy_blocks(cow)
            chunks.append(ScheduledChunk(_SeqView(s, toks, len(s.output_token_ids)), start,
                                         end - start, slots, False))
            self.draft_len[s.seq_id] = end
        if chunks:
            dec = [c for c in chunks if c.num_tokens == 1]
            pre = [c for c in chunks if c.num_tokens > 1]
            # logits are not needed: mark the last chunk so the runner samples one row
            tgt = (pre or dec)[-1]
            tgt.needs_logits = True
            self.draft.execute(SchedulerOutput(decode=dec, prefill=pre))

    def _sweep(self, eng):
        live = {s.seq_id for s in eng.scheduler.running}
        for sid in list(self.draft_len):
            if sid not in live:
                if self.dbm.has_seq(sid):
                    self.dbm.free_sequence(sid)
                self.draft_len.pop(sid, None)

    # ------------------------------------------------------------------------------
    def _spec_round(self, eng, so: SchedulerOutput):
        k = self.k
        seqs = [c.seq for c in so.decode]
        bm = eng.blocks
        # The scheduler reserved one slot per sequence; verify needs k more.
        for c in so.decode:
            if bm.blocks_needed(c.seq.seq_id, k) > bm.num_free_blocks():
                # not enough KV for speculation this step: plain decode
                res = eng.runner.execute(so)
                return eng._process(res.chunks, res.tokens)
        if so.cow_pairs:
            eng.kv.copy_blocks(so.cow_pairs)
            so.cow_pairs = []
        t0 = time.perf_counter()
        # ---- draft: catch up, then k proposals ------------------------------------
        # Proposal j + 1 takes proposal j as its input token straight from the device (the
        # runner's token forwarding), so the k draft steps launch back to back; each step's ids
        # are read on the host one step later, while the next step runs.  The draft block
        # manager keeps no prefix index, so placeholder ids stand in for tokens not yet read.
        props: Dict[int, List[int]] = {s.seq_id: [] for s in seqs}
        for s in seqs:
            self._draft_register(s)
        row_of: Dict[int, int] = {}            # seq_id -> row of the previous step's samples
        pending = None                         # (PendingTokens, seq_ids in row order)

        def collect(p):
            if p is not None:
                for sid, t in zip(p[1], p[0].tokens()):
                    props[sid].append(t)

        for step in range(k):
            chunks, src = [], []
            for s in seqs:
                sid = s.seq_id
                toks = s.all_token_ids + [0] * step
                dv = _SeqView(s, toks, len(toks) - s.prompt_len)
                start = self.draft_len[sid]
                n = len(toks) - start
                slots, cow = self.dbm.append_slots(sid, n, toks[start:])
                if cow:
                    self.draft.kv.copy_blocks(cow)
                chunks.append(ScheduledChunk(dv, start, n, slots, True))
                src.append(row_of[sid] if step > 0 else -1)
                self.draft_len[sid] = len(toks)
            if step == 0:
                dec = [c for c in chunks if c.num_tokens == 1]
                pre = [c for c in chunks if c.num_tokens > 1]
                res = self.draft.execute(SchedulerOutput(decode=dec, prefill=pre), defer=True)
            else:
                res = self.draft.execute(SchedulerOutput(decode=chunks, prefill=[]),
                                         src_rows=src, defer=True)
            collect(pending)
            order = [c.seq.seq_id for c in res.chunks]
            row_of = {sid: i for i, sid in enumerate(order)}
            pending = (res.pending, order)
        collect(pending)
        t1 = time.perf_counter()
        # ---- target verify: k+1 tokens per sequence, every row sampled -------------
        vchunks = []
        for c in so.decode:
            s = c.seq
            toks = props[s.seq_id]
            more, cow = bm.append_slots(s.seq_id, k, toks)
            if cow:
                eng.kv.copy_blocks(cow)
            view = _SeqView(s, s.all_token_ids + toks, len(s.output_token_ids))
            vchunks.append(ScheduledChunk(view, c.start, k + 1, c.slots + more, True,
                                          logits_all=True))
        # mark as prefill-shaped chunks (several query tokens) for the runner
        res = eng.runner.execute(SchedulerOutput(decode=[], prefill=vchunks))
        t2 = time.perf_counter()
        # ---- accept -----------------------------------------------------------------
        outs = []
        now = time.perf_counter()
        ti = 0
        eng.stats.steps += 1
        for c, dc in zip(vchunks, so.decode):
            s = dc.seq
            target = res.tokens[ti:ti + k + 1]
            ti += k + 1
            prop = props[s.seq_id]
            n = 0
            while n < k and prop[n] == target[n]:
                n += 1
            emit = target[:n + 1]
            self.stats.proposed += k
            self.stats.accepted += n
            # KV: x0 and the n accepted proposals are valid
            L0 = c.start
            keep = L0 + 1 + n
            bm.truncate(s.seq_id, keep)
            s.num_computed_tokens = keep
            dl = min(self.draft_len[s.seq_id], keep)
            self.dbm.truncate(s.seq_id, dl)
            self.draft_len[s.seq_id] = dl
            for tok in emit:
                if s.finished:
                    break
                outs.append(eng._append_token(s, tok, now))
                self.stats.emitted += 1
            # computed tokens exclude the newest sampled token
            if not s.finished:
                s.num_computed_tokens = min(s.num_computed_tokens, s.num_tokens - 1)
                bm.truncate(s.seq_id, s.num_computed_tokens)
        self.stats.rounds += 1
        self.stats.draft_s += t1 - t0
        self.stats.verify_s += t2 - t1
        if (self.stats.rounds >= self.fallback_after and
                self.stats.acceptance_rate() < self.min_acc):
            self.active = False  # reference auto-fallback
        self._sweep(eng)
        return outs


def attach_speculative(engine, draft_model, draft_cfg, k: int = 4, num_blocks: int = 0,
                       use_cuda_graphs: bool = True, min_acceptance: float = 0.3,
                       fallback_after: int = 10) -> SpeculativeDecoder:
    """Give ``engine`` a draft model (a ``LlamaModel`` with the same tokenizer)."""
    from ..kv.block_manager import BlockManager
    from ..models.llama import KVCache
    from .model_runner import ModelRunner
    c = engine.cfg
    nb = num_blocks or max(64, engine.blocks.num_blocks // 2)
    kv = KVCache(draft_cfg.num_layers, nb, draft_model.hkv, c.cache.block_size,
                 draft_cfg.head_dim_padded, device=draft_model.device)
    dbm = BlockManager(nb, c.cache.block_size, enable_prefix=False)
    runner = ModelRunner(draft_model, kv, dbm, c.scheduler.max_num_seqs,
                         c.scheduler.max_num_batched_tokens + c.scheduler.max_num_seqs * (k + 1),
                         c.scheduler.max_model_len + k + 1, use_cuda_graphs=use_cuda_graphs,
                         comm=draft_model.comm)
    spec = SpeculativeDecoder(engine, runner, dbm, k, min_acceptance, fallback_after)
    engine.spec = spec
    return spec
