"""Model runner: turns a scheduler step into device inputs, runs the model, samples.

Replaces the reference's per-request ``ParallelModelManager::forward_batch``
(``src/model/parallel_model_manager.rs:1201-1936``: per-slot tensors, full-pool padding, a
D2H ``argmax().to_scalar()`` per request per step) and the Fuel plan-once / CUDA-graph
decode (``src/model_fuel/mod.rs:39-63``):

* every integer input of a step (ids, positions, KV slots, sequence lengths, query offsets,
  block tables, top-k) is packed into ONE pinned int32 buffer and copied with one H2D
  transfer; floats and seeds take one more each; the sampled ids come back in one D2H copy;
* decode-only steps replay a CUDA graph captured per batch-size bucket (static input
  buffers, fixed GEMM tile plans and split-KV factor); mixed prefill/decode steps run eager;
* sampling runs on the device for all rows of the step.
"""
from __future__ import annotations

import bisect
import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence as Seq

import numpy as np
import torch

from .. import ops
from ..models.llama import ForwardBatch, KVCache, LlamaModel, prefill_tiles
from .sampling import token_seed
from .scheduler import ScheduledChunk, SchedulerOutput

DEFAULT_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 224, 256, 320, 384, 512)


@dataclass
class StepResult:
    chunks: List[ScheduledChunk]
    tokens: Optional[List[int]]  # one per chunk with needs_logits, in chunk order
    logprobs: Optional[List[float]] = None
    pending: Optional["PendingTokens"] = None   # deferred launch: tokens arrive later


class PendingTokens:
    """Sampled ids of a launched step, copied to pinned host memory behind a CUDA event."""

    def __init__(self, host: torch.Tensor, n: int, event=None):
        self.host, self.n, self.event = host, n, event

    def tokens(self) -> List[int]:
        if self.event is not None:
            self.event.synchronize()
        return self.host[:self.n].tolist()


class _GraphBucket:
    def __init__(self, runner: "ModelRunner", bsz: int, greedy: bool = False):
        r = runner
        self.bsz = bsz
        self.greedy = greedy   # tensor parallel: every row greedy -> argmax without full logits
        dev = r.device
        W = r.max_blocks_per_seq
        self.W = W
        # int32 layout: ids | pos | slots | seq_lens | cu_q(B+1) | top_k | src | block_tables(B*W)
        self.n_int = 7 * bsz + 1 + bsz * W
        self.ints = torch.zeros(self.n_int, dtype=torch.int32, device=dev)
        self.floats = torch.zeros(2 * bsz, dtype=torch.float32, device=dev)
        self.seeds = torch.zeros(bsz, dtype=torch.int64, device=dev)
        o = 0

        def take(n):
            nonlocal o
            t = self.ints[o:o + n]
            o += n
            return t

        self.ids, self.pos, self.slots, self.seq_lens = take(bsz), take(bsz), take(bsz), take(bsz)
        self.cu_q = take(bsz + 1)
        self.top_k = take(bsz)
        self.src = take(bsz)           # row of the previous step whose sample feeds this row
        self.block_tables = take(bsz * W).view(bsz, W)
        self.temp, self.top_p = self.floats[:bsz], self.floats[bsz:]
        self.out_tokens = r.d_last_out[:bsz]   # shared by every bucket: read by the next step
        self.logits_idx = torch.arange(bsz, dtype=torch.int64, device=dev)
        self.splits = ops.decode_splits(bsz, r.model.hkv, r.max_model_len) if r.is_cuda else 1
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.launches = 0

    def batch(self) -> ForwardBatch:
        return ForwardBatch(self.ids, self.pos, self.slots, self.block_tables, self.seq_lens,
                            self.cu_q, self.logits_idx, num_decode=self.bsz,
                            decode_splits=self.splits)

    def run(self, runner: "ModelRunner"):
        ops.forward_tokens(self.ids, self.src, runner.d_last_out)
        logits = runner.model.forward(self.batch(), runner.kv)
        if self.greedy:
            runner.comm.argmax_vocab_parallel(logits, self.out_tokens)
        else:
            runner.postprocess_logits(logits, self.temp, self.top_k, self.top_p, self.seeds,
                                      self.out_tokens)


class ModelRunner:
    def __init__(self, model: LlamaModel, kv: KVCache, block_manager, max_num_seqs: int,
                 max_num_batched_tokens: int, max_model_len: int, use_cuda_graphs: bool = True,
                 graph_buckets: Seq[int] = DEFAULT_BUCKETS, comm=None):
        self.model = model
        self.kv = kv
        self.bm = block_manager
        self.device = model.device
        self.is_cuda = self.device.type == "cuda"
        self.max_num_seqs = max_num_seqs
        self.max_tokens = max_num_batched_tokens + max_num_seqs
        self.max_model_len = max_model_len
        self.block_size = kv.block_size
        self.max_blocks_per_seq = (max_model_len + self.block_size - 1) // self.block_size + 1
        self.use_graphs = use_cuda_graphs and self.is_cuda
        step = comm.world if (comm is not None and getattr(comm, "fused_requested", False)) else 1
        # fused tensor-parallel decode needs T % world == 0: round buckets up to multiples
        bk = sorted({((b + step - 1) // step) * step for b in graph_buckets if b <= max_num_seqs})
        top = ((max_num_seqs + step - 1) // step) * step
        self.buckets = bk or [top]
        if self.buckets[-1] < max_num_seqs:
            self.buckets.append(top)
        self.graphs: Dict[int, _GraphBucket] = {}
        self.graph_pool = None
        self.comm = comm
        pin = self.is_cuda
        n_int = 6 * self.max_tokens + 3 * (max_num_seqs + 1) + max_num_seqs * self.max_blocks_per_seq
        # sampled rows per step: one per sequence, or every row of a verify chunk
        ns = self.max_tokens + 1
        # Two sets of pinned input buffers, alternated per launch: with overlapped decode the
        # host fills step N+1's inputs while step N's H2D copy may still be queued behind
        # step N-1, so a step's buffer is rewritten only two launches later (after its ids
        # were read back, which orders its copies before).
        self._h_in = [(torch.zeros(n_int, dtype=torch.int32, pin_memory=pin),
                       torch.zeros(2 * ns, dtype=torch.float32, pin_memory=pin),
                       torch.zeros(ns, dtype=torch.int64, pin_memory=pin)) for _ in range(2)]
        self._h_in_k = 0
        self.h_ints, self.h_floats, self.h_seeds = self._h_in[0]
        # two pinned result buffers: a deferred step's ids stay readable while the next
        # step's copy lands in the other one
        self.h_outs = [torch.zeros(ns, dtype=torch.int32, pin_memory=pin) for _ in range(2)]
        self._hout_k = 0
        # the last step's sampled ids on the device (overlapped decode forwards them)
        self.d_last_out = torch.zeros(ns, dtype=torch.int32, device=self.device)
        self.d_ints = torch.zeros(n_int, dtype=torch.int32, device=self.device)
        self.d_floats = torch.zeros(2 * ns, dtype=torch.float32, device=self.device)
        self.d_seeds = torch.zeros(ns, dtype=torch.int64, device=self.device)
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self._events = None  # list of (start, end) CUDA events per step when enabled

    # ---- device step timing (CUDA events around each step's device work) -------------
    def enable_step_events(self):
        self._events = []
        return self._events

    def disable_step_events(self):
        self._events = None

    def step_events_total_ms(self) -> float:
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in (self._events or []))

    def _ev_start(self):
        if self._events is None:
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def _ev_end(self, start):
        if start is None:
            return
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self._events.append((start, e))

    def release_graphs(self):
        """Drop captured graphs (required before destroying an NCCL process group)."""
        for g in self.graphs.values():
            g.graph = None
        self.graphs.clear()
        torch.cuda.synchronize() if self.is_cuda else None

    # -------------------------------------------------------------------------------
    def postprocess_logits(self, logits, temp, top_k, top_p, seeds, out_tokens,
                           greedy: bool = False):
        if self.comm is not None and self.comm.world > 1:
            if greedy:
                self.comm.argmax_vocab_parallel(logits, out_tokens)
            else:
                self.comm.sample_vocab_parallel(logits, temp, top_k, top_p, seeds, out_tokens)
        else:
            ops.sample(logits, temp, top_k, top_p, seeds, out_tokens)

    def _sampling_rows(self, chunks: List[ScheduledChunk]):
        temps, topk, topp, seeds = [], [], [], []
        for c in chunks:
            if not c.needs_logits:
                continue
            p = c.seq.params
            rows = c.num_tokens if c.logits_all else 1
            # row i samples output token number len(outputs) + i (a verify chunk's rows are
            # the positions after each of its input tokens)
            base = len(c.seq.output_token_ids)
            for i in range(rows):
                temps.append(p.temperature)
                topk.append(p.top_k)
                topp.append(p.top_p)
                # greedy rows never read their seed: skip the hash
                seeds.append(token_seed(c.seq.request_id, base + i, p.seed)
                             if p.temperature > 0 else 0)
        return temps, topk, topp, seeds

    # -------------------------------------------------------------------------------
    def _next_host_inputs(self) -> None:
        self._h_in_k ^= 1
        self.h_ints, self.h_floats, self.h_seeds = self._h_in[self._h_in_k]

    def _next_hout(self) -> torch.Tensor:
        self._hout_k ^= 1
        return self.h_outs[self._hout_k]

    def _finish_out(self, dev_out: torch.Tensor, n: int, defer: bool):
        """Copy ``n`` sampled ids to pinned memory; return them, or a pending handle."""
        if not self.is_cuda:
            host = dev_out[:n].clone()
            return PendingTokens(host, n) if defer else host.tolist()
        h = self._next_hout()
        h[:n].copy_(dev_out[:n], non_blocking=True)
        self.d2h_bytes = n * 4
        if defer:
            ev = torch.cuda.Event()
            ev.record()
            return PendingTokens(h, n, ev)
        torch.cuda.current_stream().synchronize()
        return h[:n].tolist()

    def execute(self, so: SchedulerOutput, src_rows: Optional[List[int]] = None,
                defer: bool = False) -> StepResult:
        """Run one scheduled step.  ``src_rows[i] >= 0``: decode chunk i's input token is row
        ``src_rows[i]`` of the previous step's samples (still on the device).  ``defer``:
        return right after the launch, with the ids behind :class:`PendingTokens`."""
        if so.cow_pairs:
            self.kv.copy_blocks(so.cow_pairs)
        chunks = so.decode + so.prefill
        if not chunks:
            return StepResult([], [])
        if not so.prefill and self.use_graphs and len(chunks) <= self.buckets[-1]:
            toks = self._run_graph(chunks, src_rows, defer)
        else:
            toks = self._run_eager(chunks, len(so.decode), src_rows, defer)
        if defer:
            return StepResult(chunks, None, pending=toks)
        return StepResult(chunks, toks)

    # -------------------------------------------------------------------------------
    def _fill_block_tables(self, seqs, out_np: np.ndarray, width: int):
        self.bm.fill_block_tables([s.seq_id for s in seqs], out_np, width)

    def _greedy_variant(self, chunks) -> bool:
        """Tensor parallel only: a batch of greedy rows replays the graph whose sampling tail
        all-gathers (max, index) pairs instead of the full vocab-parallel logits."""
        return (self.comm is not None and self.comm.world > 1 and
                all(c.seq.params.temperature <= 0 for c in chunks))

    def _run_graph(self, chunks: List[ScheduledChunk], src_rows=None, defer: bool = False):
        B = len(chunks)
        bsz = self.buckets[bisect.bisect_left(self.buckets, B)]
        greedy = self._greedy_variant(chunks)
        g = self.graphs.get((bsz, greedy))
        if g is None:
            g = self._capture(bsz, greedy)
        W = g.W
        self._next_host_inputs()
        hi = self.h_ints[:g.n_int].numpy()
        hi[:] = 0
        ids, pos, slots = hi[:bsz], hi[bsz:2 * bsz], hi[2 * bsz:3 * bsz]
        seq_lens, cu_q = hi[3 * bsz:4 * bsz], hi[4 * bsz:5 * bsz + 1]
        top_k = hi[5 * bsz + 1:6 * bsz + 1]
        src = hi[6 * bsz + 1:7 * bsz + 1]
        bt = hi[7 * bsz + 1:].reshape(bsz, W)
        slots[:] = -1
        src[:] = -1
        for i, c in enumerate(chunks):
            s = c.seq
            ids[i] = s.last_token
            pos[i] = c.start + getattr(s, "evicted", 0)
            slots[i] = c.slots[0]
            seq_lens[i] = c.start + 1
        if src_rows is not None:
            sr = np.asarray(src_rows, dtype=np.int32)
            src[:B] = sr
            ids[:B][sr >= 0] = 0
        cu_q[:B + 1] = np.arange(B + 1, dtype=np.int32)
        cu_q[B + 1:] = B
        self._fill_block_tables([c.seq for c in chunks], bt[:B], W)
        temps, tk, tp, seeds = self._sampling_rows(chunks)
        top_k[:B] = tk
        hf = self.h_floats[:2 * bsz].numpy()
        hf[:] = 0
        hf[:B] = temps
        hf[bsz:bsz + B] = tp
        hs = self.h_seeds[:bsz].numpy()
        hs[:B] = seeds
        g.ints.copy_(self.h_ints[:g.n_int], non_blocking=True)
        g.floats.copy_(self.h_floats[:2 * bsz], non_blocking=True)
        g.seeds.copy_(self.h_seeds[:bsz], non_blocking=True)
        self.h2d_bytes = g.n_int * 4 + 2 * bsz * 4 + bsz * 8
        ev = self._ev_start()
        g.graph.replay()
        self._ev_end(ev)
        ops.launch_counter_add(g.launches)
        return self._finish_out(g.out_tokens, B, defer)

    def _capture(self, bsz: int, greedy: bool = False) -> _GraphBucket:
        # the warm-up runs write dummy samples into the shared last-ids buffer, which an
        # overlapped step launched next still has to read: keep its contents
        saved = self.d_last_out.clone()
        g = _GraphBucket(self, bsz, greedy)
        # valid dummy inputs: every row points at block 0 with one token, no KV write
        g.cu_q.copy_(torch.arange(bsz + 1, dtype=torch.int32))
        g.seq_lens.fill_(1)
        g.slots.fill_(-1)
        g.src.fill_(-1)
        g.temp.fill_(0.0)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                g.run(self)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        if self.graph_pool is None:
            self.graph_pool = torch.cuda.graph_pool_handle()
        graph = torch.cuda.CUDAGraph()
        n0 = ops.launch_counter_value()
        with torch.cuda.graph(graph, pool=self.graph_pool):
            g.run(self)
        g.launches = ops.launch_counter_value() - n0
        ops.launch_counter_add(-g.launches)  # capture launched nothing
        torch.cuda.synchronize()
        self.d_last_out.copy_(saved)
        g.graph = graph
        self.graphs[(bsz, greedy)] = g
        return g

    def capture_all(self, up_to: Optional[int] = None) -> None:
        tp = self.comm is not None and self.comm.world > 1
        for b in self.buckets:
            if up_to is None or b <= up_to:
                for greedy in ((False, True) if tp else (False,)):
                    if (b, greedy) not in self.graphs:
                        self._capture(b, greedy)

    def _run_eager(self, chunks: List[ScheduledChunk], num_decode: int, src_rows=None,
                   defer: bool = False):
        B = len(chunks)
        T = sum(c.num_tokens for c in chunks)
        width = max((len(self.bm.block_table(c.seq.seq_id)) for c in chunks), default=1)
        width = max(width, 1)
        self._next_host_inputs()
        hi = self.h_ints.numpy()
        o = 0

        def take(n):
            nonlocal o
            v = hi[o:o + n]
            o += n
            return v

        ids, pos, slots = take(T), take(T), take(T)
        seq_lens, cu_q = take(B), take(B + 1)
        nlog = sum((c.num_tokens if c.logits_all else 1) for c in chunks if c.needs_logits)
        logits_idx = take(nlog)
        top_k = take(nlog)
        src = take(num_decode)
        bt = take(B * width).reshape(B, width)
        n_int = o
        t = 0
        li = 0
        cu_q[0] = 0
        for i, c in enumerate(chunks):
            s = c.seq
            n = c.num_tokens
            t0 = c.start + getattr(s, "evicted", 0)   # token index (KV index + evicted)
            ids[t:t + n] = s.all_token_ids[t0:t0 + n]
            pos[t:t + n] = np.arange(t0, t0 + n, dtype=np.int32)
            slots[t:t + n] = c.slots
            t += n
            seq_lens[i] = c.start + n
            cu_q[i + 1] = t
            if c.needs_logits:
                if c.logits_all:
                    logits_idx[li:li + n] = np.arange(t - n, t, dtype=np.int32)
                    li += n
                else:
                    logits_idx[li] = t - 1
                    li += 1
        fwd = src_rows is not None and any(r >= 0 for r in src_rows)
        if fwd:
            # decode chunks come first, one token each: token row i is decode chunk i
            sr = np.asarray(src_rows, dtype=np.int32)
            src[:] = sr
            ids[:num_decode][sr >= 0] = 0
        self._fill_block_tables([c.seq for c in chunks], bt, width)
        temps, tk, tp, seeds = self._sampling_rows(chunks)
        top_k[:] = tk
        hf = self.h_floats[:2 * max(nlog, 1)].numpy()
        hf[:nlog] = temps
        hf[nlog:2 * nlog] = tp
        self.h_seeds[:nlog].numpy()[:] = seeds
        d = self.d_ints[:n_int]
        d.copy_(self.h_ints[:n_int], non_blocking=True)
        df = self.d_floats[:2 * nlog]
        df.copy_(self.h_floats[:2 * nlog], non_blocking=True)
        ds = self.d_seeds[:nlog]
        ds.copy_(self.h_seeds[:nlog], non_blocking=True)
        self.h2d_bytes = n_int * 4 + nlog * 16
        o = 0

        def dtake(n):
            nonlocal o
            v = d[o:o + n]
            o += n
            return v

        d_ids, d_pos, d_slots = dtake(T), dtake(T), dtake(T)
        d_seq_lens, d_cu_q = dtake(B), dtake(B + 1)
        d_logits_idx = dtake(nlog).long()
        d_top_k = dtake(nlog)
        d_src = dtake(num_decode)
        d_bt = dtake(B * width).view(B, width)
        if fwd:
            ops.forward_tokens(d_ids[:num_decode], d_src, self.d_last_out)
        cu_list = cu_q.tolist()
        ts, tr = prefill_tiles(cu_list, num_decode, self.model.group,
                               block_size=self.block_size, head_dim=self.model.d)
        tiles = torch.tensor([ts, tr], dtype=torch.int32).to(self.device, non_blocking=True) \
            if ts else None
        max_len = int(seq_lens.max()) if B else 1
        fb = ForwardBatch(d_ids, d_pos, d_slots, d_bt, d_seq_lens, d_cu_q, d_logits_idx,
                          num_decode=num_decode,
                          tile_seq=tiles[0] if tiles is not None else None,
                          tile_row0=tiles[1] if tiles is not None else None,
                          decode_splits=ops.decode_splits(num_decode, self.model.hkv, max_len)
                          if self.is_cuda else 1,
                          seq_lens_cpu=torch.from_numpy(seq_lens.copy()),
                          cu_q_cpu=torch.from_numpy(cu_q.copy()))
        ev = self._ev_start() if self.is_cuda else None
        logits = self.model.forward(fb, self.kv)
        out = torch.empty(nlog, dtype=torch.int32, device=self.device)
        self.postprocess_logits(logits, df[:nlog], d_top_k, df[nlog:2 * nlog], ds, out,
                                greedy=self._greedy_variant([c for c in chunks
                                                              if c.needs_logits]))
        if nlog <= self.d_last_out.shape[0]:
            self.d_last_out[:nlog].copy_(out)
        self._ev_end(ev)
        return self._finish_out(out, nlog, defer)
