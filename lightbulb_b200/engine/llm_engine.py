"""LLMEngine: the public offline/serving API.

Replaces the reference's ``ModelRunner`` thread + ``EngineModel`` trait
(``src/engine/model_runner.rs:129-528``) and the model managers
(``src/model/parallel_model_manager.rs``, ``src/model_fuel/engine_model.rs``) with a
continuous-batching engine:

    eng = LLMEngine.from_pretrained(path)            # safetensors dir / .gguf / AWQ dir
    eng.add_request("r1", prompt="...", params=SamplingParams(max_tokens=64))
    while eng.has_unfinished(): outs = eng.step()    # one scheduler iteration
    eng.generate(["a", "b"], params)                 # convenience

Every ``step()`` copies that step's inputs host->device from pinned memory and reads the
sampled ids back device->host (``last_step_io``).
"""
from __future__ import annotations

import bisect
import collections
import threading
import logging
import os
import time
import uuid
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence as Seq, Union

import torch

from ..config import CacheConfig, EngineConfig, ModelConfig, SchedulerConfig
from ..kv.block_manager import BlockManager
from ..models.llama import KVCache, LlamaModel
from .model_runner import ModelRunner
from .sampling import SamplingParams
from .scheduler import Scheduler
from ..utils import trace
from .sequence import Sequence, SeqStatus, effective_generation_budget
from .tokenizer import BaseTokenizer, ByteTokenizer, IncrementalDetokenizer

log = logging.getLogger("lightbulb_b200.engine")


@dataclass
class RequestOutput:
    request_id: str
    new_token_ids: List[int]
    new_text: str
    finished: bool
    finish_reason: Optional[str] = None
    prompt_tokens: int = 0
    completion_tokens: int = 0
    cached_tokens: int = 0
    tool_call: Optional[dict] = None   # set when the request paused on a tool call


TTFT_BUCKETS = (0.01, 0.025, 0.05, 0.1, 0.25, 0.5, 1.0, 2.5, 5.0, 10.0)     # seconds
ITL_BUCKETS = (0.001, 0.0025, 0.005, 0.01, 0.02, 0.05, 0.1, 0.25, 0.5)


class LatencySamples(collections.deque):
    """Latency samples of a long-running engine: the newest ``window`` values (quantiles) plus
    cumulative histogram counts, sum and count since start (monotone, as Prometheus expects),
    so memory stays bounded however many tokens are served.  The engine thread appends while
    server handlers read: :meth:`snapshot` copies under the same lock as :meth:`append`, and
    the window is small enough (8192) that sorting a copy costs well under a millisecond."""

    def __init__(self, bounds, window: int = 8192):
        super().__init__(maxlen=window)
        self.bounds = tuple(bounds)
        self.bucket_counts = [0] * (len(self.bounds) + 1)     # last: above every bound
        self.total = 0
        self.sum = 0.0
        self._lock = threading.Lock()

    def append(self, v: float) -> None:
        with self._lock:
            super().append(v)
            self.bucket_counts[bisect.bisect_left(self.bounds, v)] += 1
            self.total += 1
            self.sum += v

    def snapshot(self) -> list:
        with self._lock:
            return list(self)


@dataclass
class EngineStats:
    steps: int = 0
    prompt_tokens: int = 0
    generated_tokens: int = 0
    preemptions: int = 0
    ttfts: "LatencySamples" = field(default_factory=lambda: LatencySamples(TTFT_BUCKETS))
    itls: "LatencySamples" = field(default_factory=lambda: LatencySamples(ITL_BUCKETS))
    finished: int = 0


def derive_num_blocks(cfg: ModelConfig, cache: CacheConfig, tp_size: int, device,
                      reserve_bytes: int = 6 << 30) -> int:
    if cache.num_blocks > 0:
        return cache.num_blocks
    hkv = max(1, cfg.num_kv_heads // tp_size)
    per_block = KVCache.bytes_per_block(cfg.num_layers, hkv, cache.block_size,
                                         cfg.head_dim_padded)
    if torch.device(device).type != "cuda":
        return max(64, (512 << 20) // per_block)
    free, _total = torch.cuda.mem_get_info(torch.device(device))
    avail = int(free * cache.gpu_memory_utilization) - reserve_bytes
    return max(16, avail // per_block)


@dataclass
class _PendingStep:
    chunks: list                 # decode chunks of the launched step, in row order
    handle: object               # PendingTokens of the runner
    marks: list                  # per chunk: (output index, token-list index) of its placeholder
    rows: Dict[int, int]         # seq_id -> row (the forwarding source for the next step)


class LLMEngine:
    def __init__(self, cfg: EngineConfig, packed_weights: dict,
                 tokenizer: Optional[BaseTokenizer] = None, comm=None, tp_rank: int = 0,
                 tp_size: int = 1, model: Optional[LlamaModel] = None):
        self.cfg = cfg
        mcfg = cfg.model
        dev = packed_weights["embed"].device
        self.device = dev
        self.tokenizer = tokenizer or ByteTokenizer(mcfg.vocab_size)
        self.eos_ids = set(mcfg.eos_ids())
        if self.tokenizer.eos_token_ids:
            self.eos_ids |= set(self.tokenizer.eos_token_ids)
        max_len = cfg.scheduler.max_model_len
        if comm is not None and comm.world > 1 and dev.type == "cuda":
            self._setup_comm(comm, cfg, dev)
        self.model = model or LlamaModel(mcfg, packed_weights, tp_rank, tp_size,
                                         max_positions=max_len + 64, comm=comm)
        nb = derive_num_blocks(mcfg, cfg.cache, tp_size, dev)
        if comm is not None and comm.world > 1:
            nb = comm.min_int(nb)  # every rank must admit identically
        self.kv = KVCache(mcfg.num_layers, nb, self.model.hkv, cfg.cache.block_size,
                          mcfg.head_dim_padded, device=dev)
        self.blocks = BlockManager(nb, cfg.cache.block_size, cfg.cache.enable_prefix_caching)
        self.scheduler = Scheduler(cfg.scheduler, self.blocks)
        self.runner = ModelRunner(self.model, self.kv, self.blocks, cfg.scheduler.max_num_seqs,
                                  cfg.scheduler.max_num_batched_tokens, max_len,
                                  use_cuda_graphs=cfg.use_cuda_graphs, comm=comm)
        self.seqs: Dict[str, Sequence] = {}
        self.detok: Dict[str, IncrementalDetokenizer] = {}
        self.stats = EngineStats()
        self.detokenize = True  # incremental text per token (off for token-id-only clients)
        self.spec = None  # speculative decoder (engine/speculative.py) when configured
        self.kv_policy = None  # KV compression policy (kv/compression.py) when configured
        self.tool_detector = None  # tool-call detection (extras/tools.py) when enabled
        # overlapped decode: step N+1 is launched before step N's ids are read back
        self.overlap = bool(getattr(cfg, "overlap_decode", True))
        self._pending: Optional[_PendingStep] = None
        log.info("engine ready: %d KV blocks of %d tokens (%.1f GiB)", nb, cfg.cache.block_size,
                 self.kv.storage.numel() * 2 / 2**30)
        if cfg.cache.h2o_budget > 0:
            self.enable_kv_compression("h2o", cfg.cache.h2o_budget, cfg.cache.sink_tokens,
                                       decay=cfg.cache.h2o_decay)
        elif cfg.cache.streaming_window > 0:
            self.enable_kv_compression("streaming", cfg.cache.streaming_window,
                                       cfg.cache.sink_tokens)

    # ---------------------------------------------------------------------------------
    @classmethod
    def from_pretrained(cls, path: str, engine_cfg: Optional[EngineConfig] = None,
                        device: str = "cuda", **kw) -> "LLMEngine":
        from ..models.loader import load_model_dir
        mcfg, packed, tok = load_model_dir(path, device=device, tp_rank=kw.get("tp_rank", 0),
                                           tp_size=kw.get("tp_size", 1))
        cfg = engine_cfg or EngineConfig()
        cfg.model = mcfg
        return cls(cfg, packed, tok, **kw)

    @classmethod
    def random_init(cls, mcfg: ModelConfig, engine_cfg: Optional[EngineConfig] = None,
                    device: str = "cuda", seed: int = 0, **kw) -> "LLMEngine":
        from ..models.weights import random_packed_model
        cfg = engine_cfg or EngineConfig()
        cfg.model = mcfg
        packed = random_packed_model(mcfg, seed=seed, rank=kw.get("tp_rank", 0),
                                     world=kw.get("tp_size", 1), device=device)
        return cls(cfg, packed, None, **kw)

    # ---------------------------------------------------------------------------------
    def add_request(self, request_id: Optional[str] = None, prompt: Optional[str] = None,
                    params: Optional[SamplingParams] = None,
                    prompt_token_ids: Optional[List[int]] = None, priority: int = 1,
                    add_special_tokens: bool = True) -> Sequence:
        rid = request_id or uuid.uuid4().hex
        params = params or SamplingParams()
        if prompt_token_ids is None:
            prompt_token_ids = self.tokenizer.encode(prompt or "", add_special_tokens)
        if not prompt_token_ids:
            prompt_token_ids = [self.tokenizer.bos_token_id or 0]
        max_len = self.cfg.scheduler.max_model_len
        if len(prompt_token_ids) >= max_len:
            prompt_token_ids = prompt_token_ids[-(max_len - 1):]
        budget, trunc = effective_generation_budget(len(prompt_token_ids), params.max_tokens,
                                                    max_len)
        seq = Sequence(rid, list(prompt_token_ids), params, priority=priority)
        seq.max_new_tokens = budget
        seq.truncated = trunc
        if rid in self.seqs and not self.seqs[rid].finished:
            raise ValueError(f"duplicate request id {rid}")
        self.seqs[rid] = seq
        self.detok[rid] = IncrementalDetokenizer(self.tokenizer)
        self.scheduler.add(seq)
        self.stats.prompt_tokens += len(prompt_token_ids)
        return seq

    def attach_draft(self, draft_packed: dict, draft_cfg, k: int = 4, **kw):
        """Enable speculative decoding with a draft model (same tokenizer / vocabulary)."""
        from ..models.llama import LlamaModel
        from .speculative import attach_speculative
        dm = LlamaModel(draft_cfg, draft_packed, self.model.tp_rank, self.model.tp_size,
                        max_positions=self.cfg.scheduler.max_model_len + k + 64,
                        comm=self.model.comm)
        return attach_speculative(self, dm, draft_cfg, k=k,
                                  use_cuda_graphs=self.cfg.use_cuda_graphs, **kw)

    def abort(self, request_id: str) -> None:
        self.scheduler.abort(request_id)

    def release(self, request_id: str) -> bool:
        """Forget a finished request (its sequence and detokenizer state).  Long-running
        front ends call this once a request's last output is delivered, so the request table
        does not grow with every request served; returns False if it is unknown or still
        running."""
        s = self.seqs.get(request_id)
        if s is None or not s.finished:
            return False
        del self.seqs[request_id]
        self.detok.pop(request_id, None)
        return True

    def has_unfinished(self) -> bool:
        return self._pending is not None or self.scheduler.has_work()

    @staticmethod
    def _setup_comm(comm, cfg: EngineConfig, dev) -> None:
        """Enable the configured peer-memory collective before any CUDA graph is captured
        (every rank takes the same steps: the setup exchanges IPC handles)."""
        mode = cfg.parallel.comm
        busy = getattr(comm, "fused_requested", False) or comm.p2p_ar is not None or \
            getattr(comm, "rowpar", None) is not None
        rows = max(cfg.scheduler.max_num_seqs, cfg.scheduler.max_num_batched_tokens)
        if mode == "p2p" and not busy:
            comm.enable_rowpar(min(16384, rows), cfg.model.hidden_size, dev)
        elif mode == "allreduce" and not busy:
            comm.enable_p2p_allreduce(min(4096, rows) * cfg.model.hidden_size, dev)
        elif mode == "fused" and not busy:
            from ..parallel.fused import enable_fused
            enable_fused(comm)
        elif mode not in ("p2p", "allreduce", "fused", "nccl"):
            raise ValueError(f"parallel.comm must be p2p, allreduce, fused or nccl, not {mode!r}")

    def has_runnable(self) -> bool:
        """Work that can make progress (requests paused on a tool call wait for a result)."""
        return self._pending is not None or bool(self.scheduler.waiting) or any(
            s.status != SeqStatus.AWAITING_TOOL for s in self.scheduler.running)

    # ---- tool calls (reference src/engine/tool_call.rs, parallel_model_manager.rs) ----------
    def enable_tool_calls(self, detector=None):
        """Pause a request in AWAITING_TOOL (its KV kept) when its generated text contains a
        complete tool call; :meth:`inject_tool_result` resumes it."""
        from ..extras.tools import ToolCallDetector
        self.tool_detector = detector or ToolCallDetector()
        return self.tool_detector

    def awaiting_tool(self) -> List[Sequence]:
        return [s for s in self.scheduler.running if s.status == SeqStatus.AWAITING_TOOL]

    def inject_tool_result(self, request_id: str, text: Optional[str] = None,
                           token_ids: Optional[List[int]] = None) -> Sequence:
        """Append a tool's result as context after the paused request's output (a mini-prefill
        into the preserved KV on the next step) and resume generation."""
        for seq in self.scheduler.running:
            if seq.request_id == request_id and seq.status == SeqStatus.AWAITING_TOOL:
                break
        else:
            raise KeyError(f"{request_id}: no request awaiting a tool result")
        ids = list(token_ids) if token_ids is not None else self.tokenizer.encode(
            text or "", False)
        if seq.num_tokens + len(ids) >= self.cfg.scheduler.max_model_len:
            raise ValueError("tool result does not fit in the context")
        seq.append_context(ids)
        seq.pending_tool_call = None
        seq.status = SeqStatus.RUNNING
        return seq

    # ---------------------------------------------------------------------------------
    def step(self) -> List[RequestOutput]:
        """One scheduler iteration.  In steady decode (every running sequence decoding, nothing
        waiting, no speculative / KV-compression / tool-call hooks) the step is overlapped: the
        next decode step is launched first, with the input ids that are still on the device
        forwarded there, and the previous step's ids are read back and processed while it runs.
        The outputs returned are then those of the previous step."""
        with trace.nvtx_range("engine.step"):
            ok = self._overlap_ok()
            if self._pending is not None and not ok:
                return self._collect_pending()          # drain; the next call schedules
            if ok:
                return self._step_overlapped()
            if self.spec is not None and self.spec.active:
                return self.spec.step(self)
            with trace.nvtx_range("schedule"):
                so = self.scheduler.schedule()
            if so.empty:
                return []
            if trace.enabled("scheduler"):
                trace.debug("scheduler", "step: %d decode, %d prefill chunks, %d tokens",
                            len(so.decode), len(so.prefill), so.num_tokens)
            if self.kv_policy is not None and hasattr(self.kv_policy, "before_step"):
                self.kv_policy.before_step(so)
            with trace.nvtx_range("execute"):
                res = self.runner.execute(so)
            return self._process(res.chunks, res.tokens)

    # ---- overlapped decode ------------------------------------------------------------
    def _overlap_ok(self) -> bool:
        if not self.overlap or self.spec is not None or self.kv_policy is not None or \
                self.tool_detector is not None:
            return False
        sch = self.scheduler
        if sch.waiting or not sch.running:
            return False
        bm = self.blocks
        need = 0
        running = SeqStatus.RUNNING
        for s in sch.running:
            if s.status is not running or s.num_uncomputed != 1:
                return False
            need += bm.blocks_needed(s.seq_id, 1)
        # enough blocks for every sequence: the schedule cannot preempt
        return need <= bm.num_free_blocks()

    def _step_overlapped(self) -> List[RequestOutput]:
        prev = self._pending
        if prev is not None:
            # a sequence whose pending id is its last (length limit) sits the next step out
            max_len = self.cfg.scheduler.max_model_len
            for s in self.scheduler.running:
                if s.seq_id in prev.rows and (len(s.output_token_ids) >= s.max_new_tokens or
                                              s.num_tokens >= max_len):
                    s.hold = True
        with trace.nvtx_range("schedule"):
            so = self.scheduler.schedule()
        if so.prefill or so.preempted:
            raise RuntimeError("overlapped decode scheduled a prefill or a preemption")
        if so.empty:
            return self._collect_pending() if prev is not None else []
        rows = prev.rows if prev is not None else {}
        src = [rows.get(c.seq.seq_id, -1) for c in so.decode]
        with trace.nvtx_range("execute"):
            res = self.runner.execute(so, src_rows=src, defer=True)
        marks = []
        for c in so.decode:
            c.seq.num_computed_tokens += 1
            marks.append(c.seq.append_placeholder())
        self._pending = _PendingStep(so.decode, res.pending, marks,
                                     {c.seq.seq_id: i for i, c in enumerate(so.decode)})
        if prev is None:
            return []
        return self._collect(prev)

    def drain(self) -> List[RequestOutput]:
        """Finish an overlapped decode step still in flight and return its outputs (the engine
        is then quiescent: every sequence's tokens are on the host)."""
        return self._collect_pending()

    def _collect_pending(self) -> List[RequestOutput]:
        p, self._pending = self._pending, None
        return self._collect(p) if p is not None else []

    def _collect(self, p: "_PendingStep") -> List[RequestOutput]:
        with trace.nvtx_range("collect"):
            toks = p.handle.tokens()
        now = time.perf_counter()
        self.stats.steps += 1
        bm = self.blocks
        outs: List[RequestOutput] = []
        for c, (oi, ti), tok in zip(p.chunks, p.marks, toks):
            seq = c.seq
            seq.hold = False
            if seq.finished:
                if len(seq.output_token_ids) > oi:
                    seq.truncate_output(oi)
                continue
            seq.set_output(oi, ti, tok)
            if bm.has_seq(seq.seq_id):
                bm.set_tokens(seq.seq_id, [tok])
            outs.append(self._append_token(seq, tok, now, n_out=oi + 1, n_tok=ti + 1))
        return outs

    def enable_kv_compression(self, kind: str = "h2o", budget: int = 2048, sinks: int = 4,
                              **kw):
        """H2O heavy hitters (budget + sinks tokens kept) or StreamingLLM (sinks + window)."""
        from ..kv.compression import H2OPolicy, StreamingPolicy
        if kind == "h2o":
            self.kv_policy = H2OPolicy(self, budget=budget, sinks=sinks, **kw)
        elif kind == "streaming":
            self.kv_policy = StreamingPolicy(self, sinks=sinks, window=budget)
        else:
            raise ValueError(kind)
        return self.kv_policy

    def enable_segmented_cache(self, config=None, context_limit: Optional[int] = None,
                               segment_tokens: int = 64, knowledge_base=None):
        """Drive segmented spans and tiered storage from the step loop (see
        :class:`lightbulb_b200.kv.spans.SegmentedPolicy`): automatic spans, attention-scored
        eviction under context pressure with demotion to RAM / disk and a knowledge-base fact
        per demoted span, and ``<RETRIEVE:key>`` promotion.  Replaces any other KV policy."""
        from ..kv.spans import SegmentedPolicy
        self.kv_policy = SegmentedPolicy(self, config, context_limit, segment_tokens,
                                         knowledge_base)
        return self.kv_policy

    def inject_context(self, request_id: str, text: Optional[str] = None,
                       token_ids: Optional[List[int]] = None) -> Sequence:
        """Append context (a system note, a retrieved document, a tool's output) to a running
        request: the tokens are prefilled into its KV on the next step, then decoding resumes."""
        if self._pending is not None:
            raise RuntimeError("an overlapped decode step is in flight: inject after the "
                               "engine drained (with a KV policy set, steps are synchronous)")
        for seq in self.scheduler.running:
            if seq.request_id == request_id and not seq.finished:
                break
        else:
            raise KeyError(f"{request_id}: no running request")
        ids = list(token_ids) if token_ids is not None else self.tokenizer.encode(
            text or "", False)
        if seq.num_tokens + len(ids) >= self.cfg.scheduler.max_model_len:
            raise ValueError("context does not fit")
        seq.append_context(ids)
        return seq

    def _process(self, chunks, tokens) -> List[RequestOutput]:
        now = time.perf_counter()
        outs: List[RequestOutput] = []
        ti = 0
        self.stats.steps += 1
        for c in chunks:
            seq = c.seq
            seq.num_computed_tokens += c.num_tokens
            if not c.needs_logits:
                continue
            tok = tokens[ti]
            ti += 1
            if seq.finished:
                continue
            outs.append(self._append_token(seq, tok, now))
        if self.kv_policy is not None:
            self.kv_policy.after_step(self)
        return outs

    def _append_token(self, seq: Sequence, tok: int, now: float, n_out: Optional[int] = None,
                      n_tok: Optional[int] = None) -> RequestOutput:
        """Record sampled id ``tok``.  ``n_out`` / ``n_tok``: the output and token counts up to
        and including it, when it fills a placeholder (later placeholders may follow)."""
        if n_out is None:
            seq.append_output(tok)
            n_out, n_tok = len(seq.output_token_ids), seq.num_tokens
        if seq.first_token_time is None:
            seq.first_token_time = now
            self.stats.ttfts.append(now - seq.arrival_time)
        elif seq.token_times:
            self.stats.itls.append(now - seq.token_times[-1])
        seq.token_times.append(now)
        self.stats.generated_tokens += 1
        delta = ""
        p = seq.params
        if self.detokenize and (p.detokenize or p.stop):
            delta = self.detok[seq.request_id].push(tok)
            seq.output_text += delta
        reason = None
        p = seq.params
        if not p.ignore_eos and (tok in self.eos_ids or tok in p.stop_token_ids):
            reason = "stop"
        elif p.stop and any(s in seq.output_text for s in p.stop):
            reason = "stop"
            for s in p.stop:
                k = seq.output_text.find(s)
                if k >= 0:
                    seq.output_text = seq.output_text[:k]
        elif n_out >= seq.max_new_tokens:
            reason = "length"
        elif n_tok >= self.cfg.scheduler.max_model_len:
            reason = "length"
        call = None
        if reason is None and self.tool_detector is not None and seq.output_text:
            call = self.tool_detector.find(seq.output_text[seq.tool_scan_from:])
            if call is not None:
                seq.tool_scan_from = len(seq.output_text)
                seq.pending_tool_call = call
                seq.status = SeqStatus.AWAITING_TOOL
        if reason is not None:
            seq.truncate_output(n_out)     # drop a placeholder launched after this token
            self.scheduler.finish(seq, reason)
            self.stats.finished += 1
        return RequestOutput(seq.request_id, [tok], delta, reason is not None, reason,
                             seq.prompt_len, n_out, seq.num_cached_prefix, call)

    # ---------------------------------------------------------------------------------
    def generate(self, prompts: Union[str, List[str], None] = None,
                 params: Optional[SamplingParams] = None,
                 prompt_token_ids: Optional[List[List[int]]] = None) -> List[Sequence]:
        if isinstance(prompts, str):
            prompts = [prompts]
        seqs = []
        if prompt_token_ids is not None:
            for ids in prompt_token_ids:
                seqs.append(self.add_request(params=params, prompt_token_ids=ids))
        else:
            for p in prompts or []:
                seqs.append(self.add_request(prompt=p, params=params))
        while any(not s.finished for s in seqs) and self.has_runnable():
            self.step()
        return seqs

    def last_step_io(self):
        return self.runner.h2d_bytes, self.runner.d2h_bytes
