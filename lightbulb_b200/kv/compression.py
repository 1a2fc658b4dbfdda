"""KV-cache compression policies: H2O heavy hitters and StreamingLLM sinks + window.

Reference: ``src/cache/h2o_policy.rs`` (cumulative decayed attention, decay 0.95, recent
tokens protected), ``src/cache/streaming_policy.rs:22-190`` (4 sink tokens + a window of
recent tokens, middle evicted) and the paged variants in ``src/model_fuel/policies.rs``
(``h2o_block_scores``, span-to-block maps).  H2O budget 2048 + 4 sinks.

* :class:`H2OPolicy`: the model accumulates, on the device, the last layer's attention mass
  of every decode query into a score pool parallel to the KV blocks (``h2o_accumulate``).
  When a sequence's KV exceeds ``budget + sinks + slack`` it keeps the sinks, the most recent
  ``recent`` tokens and the highest-scoring tokens in between (``budget`` in total beyond the
  sinks), copies them in order into fresh blocks (``kv_compact``, all layers at once) and
  swaps the block table.  Kept keys keep their rotary positions (keys are stored after RoPE);
  new tokens continue at their true positions (``Sequence.evicted``).
* :class:`StreamingPolicy`: block granularity, no copy: keeps the first block (sinks) and
  the last ``window`` tokens' blocks and drops whole blocks in between.
"""
from __future__ import annotations

from typing import List, Optional

import torch

from .. import ops


class H2OPolicy:
    def __init__(self, engine, budget: int = 2048, sinks: int = 4, recent: int = 64,
                 decay: float = 0.95, slack: int = 128):
        self.eng = engine
        self.budget, self.sinks, self.recent = budget, sinks, recent
        self.decay, self.slack = decay, slack
        kv = engine.kv
        self.score = torch.zeros(kv.num_blocks * kv.block_size, dtype=torch.float32,
                                 device=kv.storage.device)
        engine.model.h2o = self
        # softmax scale of the model's attention (1 / sqrt(true head_dim) for padded heads);
        # None -> 1 / sqrt(width of q)
        cfg = getattr(engine.model, "cfg", None)
        self.scale = 1.0 / (cfg.head_dim ** 0.5) if cfg is not None else None
        self._ws = None  # device workspaces of h2o_accumulate (logits, softmax partials)
        model = engine.model
        ecfg = getattr(engine, "cfg", None)
        if kv.storage.is_cuda and ecfg is not None and hasattr(model, "hq"):
            # allocated before any decode graph is captured
            bs = kv.block_size
            lmax = ((ecfg.scheduler.max_model_len + bs - 1) // bs + 1) * bs
            self._alloc(ecfg.scheduler.max_num_seqs, model.hq, lmax, kv.storage.device)
        self.compactions = 0

    def before_step(self, so) -> None:
        """Slots written this step start with a zero score (blocks are reused)."""
        slots = [x for c in so.decode + so.prefill for x in c.slots]
        if slots:
            idx = torch.tensor(slots, dtype=torch.int64).to(self.score.device, non_blocking=True)
            self.score.index_fill_(0, idx, 0.0)

    # called from the model on the last layer (inside the step, graph-capturable)
    def accumulate(self, q, k_cache, block_tables, seq_lens):
        scale = self.scale if self.scale is not None else 1.0 / (q.shape[-1] ** 0.5)
        if q.is_cuda:
            ws_l, ws_p = self._workspaces(q, block_tables, k_cache.shape[2])
            ops._need_c().h2o_accumulate(q, k_cache, block_tables, seq_lens, self.score,
                                         self.decay, scale, ws_l, ws_p)
            ops.launch_counter_add(2)
            return
        bs = k_cache.shape[2]
        for i in range(seq_lens.shape[0]):
            L = int(seq_lens[i])
            nb = (L + bs - 1) // bs
            blk = block_tables[i, :nb].long()
            slots = (blk[:, None] * bs + torch.arange(bs)[None]).flatten()[:L]
            k = k_cache[blk].permute(0, 2, 1, 3).reshape(nb * bs, k_cache.shape[1], -1)[:L]
            g = q.shape[1] // k.shape[1]
            kk = k.float().repeat_interleave(g, dim=1)
            s = torch.einsum("hd,khd->hk", q[i].float(), kk) * scale
            p = torch.softmax(s, dim=-1).sum(0)
            self.score[slots] = self.score[slots] * self.decay + p

    def _alloc(self, bmax, hq, lmax, device):
        tmax = (lmax + 255) // 256
        self._ws = (torch.empty(bmax, hq, lmax, dtype=torch.float32, device=device),
                    torch.empty(bmax, hq, tmax, 2, dtype=torch.float32, device=device))

    def _workspaces(self, q, block_tables, bs):
        """Logits [max seqs, Hq, max len] and softmax partials, sized from the engine limits at
        construction (the kernels read the live lengths on the device, so the decode CUDA
        graphs can capture them); grown here only for callers outside those limits."""
        lmax = block_tables.shape[1] * bs
        ws = self._ws
        if ws is None or ws[0].shape[0] < q.shape[0] or ws[0].shape[2] < lmax or \
                ws[0].shape[1] != q.shape[1]:
            self._alloc(q.shape[0], q.shape[1], lmax, q.device)
        return self._ws

    def after_step(self, engine) -> None:
        bs = engine.kv.block_size
        limit = self.budget + self.sinks + self.slack
        for seq in list(engine.scheduler.running):
            kvlen = seq.num_computed_tokens
            if kvlen <= limit or seq.num_uncomputed != 1 or not seq.output_token_ids:
                continue
            self.compact(engine, seq)

    def compact(self, engine, seq) -> None:
        bm = engine.blocks
        bs = engine.kv.block_size
        kvlen = seq.num_computed_tokens
        table = bm.block_table(seq.seq_id)
        slots = torch.tensor([table[p // bs] * bs + p % bs for p in range(kvlen)],
                             dtype=torch.int64)
        keep_n = self.sinks + self.budget
        mid_lo, mid_hi = self.sinks, kvlen - self.recent
        n_mid = keep_n - self.sinks - self.recent
        sc = self.score[slots[mid_lo:mid_hi].to(self.score.device)]
        top = torch.topk(sc, min(n_mid, sc.numel())).indices.cpu() + mid_lo
        keep = torch.cat([torch.arange(self.sinks), torch.sort(top).values,
                          torch.arange(mid_hi, kvlen)])
        new_len = keep.numel()
        nblk = (new_len + bs - 1) // bs
        fresh = bm.alloc_blocks(nblk)
        dst = torch.tensor([fresh[i // bs] * bs + i % bs for i in range(new_len)],
                           dtype=torch.int32)
        src = slots[keep].to(torch.int32)
        dev = engine.kv.storage.device
        if dev.type == "cuda":
            ops._need_c().kv_compact(engine.kv.storage, src.to(dev), dst.to(dev), self.score)
            ops.launch_counter_add(1)
        else:
            st = engine.kv.storage
            sb, so = src.long() // bs, src.long() % bs
            db, do = dst.long() // bs, dst.long() % bs
            st[:, :, db, :, do] = st[:, :, sb, :, so]
            self.score[dst.long()] = self.score[src.long()]
        bm.set_blocks(seq.seq_id, fresh, new_len)
        seq.evicted += kvlen - new_len
        seq.num_computed_tokens = new_len
        self.compactions += 1


class StreamingPolicy:
    """Sinks + window at block granularity (no copy: the middle blocks are dropped)."""

    def __init__(self, engine, sinks: int = 4, window: int = 2048):
        self.sinks, self.window = sinks, window
        self.evictions = 0

    def after_step(self, engine) -> None:
        bm = engine.blocks
        bs = engine.kv.block_size
        sink_blocks = (self.sinks + bs - 1) // bs
        for seq in list(engine.scheduler.running):
            kvlen = seq.num_computed_tokens
            if seq.num_uncomputed != 1:
                continue
            win_blocks = (self.window + bs - 1) // bs + 1
            table = bm.block_table(seq.seq_id)
            full_blocks = kvlen // bs
            if full_blocks <= sink_blocks + win_blocks:
                continue
            # drop whole full blocks between the sinks and the window; the tail stays
            drop = full_blocks - sink_blocks - win_blocks
            new = table[:sink_blocks] + table[sink_blocks + drop:]
            bm.set_blocks(seq.seq_id, new, kvlen - drop * bs)
            seq.evicted += drop * bs
            seq.num_computed_tokens = kvlen - drop * bs
            self.evictions += 1
