"""Pipeline parallelism: consecutive layer ranges on consecutive ranks, activations passed
point to point, micro-batches in flight on different stages at once (GPipe forward schedule).

Reference: ``src/multi_gpu/pipeline_parallel.rs`` -- even layer split with the remainder on the
last stage (``:16-105``), GPipe over micro-batches that runs the stages *one after another* in
a single process (``:127-240``: ``to_device(stage)`` then ``forward_layers``; no overlap), and
``ParallelismMode::Hybrid{tensor_world_size, pipeline_stages, micro_batch_size}`` as config only
(``config.rs:25-51``).  Here every stage is its own process (one GPU per rank, NCCL, or gloo on
CPU): stage s receives the residual stream of micro-batch m from stage s-1, runs its layers (with
its own paged KV for those layers) and sends the result on while stage s-1 already works on
micro-batch m+1.  The last stage applies the final norm and LM head, picks the next tokens
(greedy, first maximum) and broadcasts them, so every stage builds the same next step locally.

:class:`PipelineEngine` serves a static batch (prefill, then decode steps) -- the reference's PP
is also a library path, not wired into its server; the continuous-batching server uses TP.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from .. import ops
from ..config import ModelConfig


def split_layers(num_layers: int, stages: int) -> List[Tuple[int, int]]:
    """Even split; the last stage takes the remainder."""
    per = num_layers // stages
    out = []
    for s in range(stages):
        l0 = s * per
        l1 = num_layers if s == stages - 1 else l0 + per
        out.append((l0, l1))
    return out


@dataclass
class HybridConfig:
    """TP x PP layout of ``world`` ranks: rank = stage * tp + tp_rank."""
    tensor_world_size: int = 1
    pipeline_stages: int = 1
    micro_batch_size: int = 0       # 0: one micro-batch per stage

    def world(self) -> int:
        return self.tensor_world_size * self.pipeline_stages

    def coords(self, rank: int) -> Tuple[int, int]:
        return rank // self.tensor_world_size, rank % self.tensor_world_size

    def stage_group_ranks(self, stage: int) -> List[int]:
        t = self.tensor_world_size
        return list(range(stage * t, (stage + 1) * t))


def pack_stage(cfg: ModelConfig, weights, stage: int, stages: int, dtype=torch.bfloat16,
               device="cpu") -> dict:
    """Device-layout weights of one stage: its layers, plus embeddings on the first stage and
    the final norm + LM head on the last."""
    from ..models.weights import pack_layer
    l0, l1 = split_layers(cfg.num_layers, stages)[stage]
    packed = {"layers": [pack_layer(cfg, weights, i, 0, 1, dtype, device) for i in range(l0, l1)]}
    if stage == 0:
        packed["embed"] = weights["model.embed_tokens.weight"].to(device, dtype).contiguous()
    if stage == stages - 1:
        packed["norm"] = weights["model.norm.weight"].to(device, dtype).contiguous()
        lm = weights.get("lm_head.weight", weights["model.embed_tokens.weight"])
        packed["lm_head"] = lm.to(device, dtype).contiguous()
    return packed


class PipelineEngine:
    """Static-batch greedy generation over ``world`` pipeline stages (this rank = one stage)."""

    def __init__(self, cfg: ModelConfig, packed_stage: dict, rank: int, world: int,
                 device, max_seqs: int, max_len: int, micro_batches: int = 0,
                 block_size: int = 16, group=None):
        from ..models.llama import KVCache, LlamaModel
        self.cfg, self.rank, self.world = cfg, rank, world
        self.first, self.last = rank == 0, rank == world - 1
        self.device = torch.device(device)
        self.model = LlamaModel(cfg, packed_stage, max_positions=max_len + 8)
        self.bs = block_size
        self.per_seq = (max_len + block_size - 1) // block_size
        self.kv = KVCache(len(packed_stage["layers"]), max_seqs * self.per_seq + 1,
                          self.model.hkv, block_size, cfg.head_dim_padded, device=self.device)
        self.max_seqs = max_seqs
        self.mb = micro_batches or world
        self.group = group
        self.hidden = cfg.hidden_size

    # ---- batches ---------------------------------------------------------------------
    def _batch(self, seqs: List[int], toks: List[List[int]], starts: List[int]):
        """ForwardBatch for sequences ``seqs`` (global indices, static blocks) whose new tokens
        ``toks[i]`` start at KV position ``starts[i]``."""
        from ..models.llama import ForwardBatch, prefill_tiles
        bs = self.bs
        ids, pos, slots, cu = [], [], [0], []
        slot_l = []
        for s, t, st in zip(seqs, toks, starts):
            for j, tok in enumerate(t):
                p = st + j
                ids.append(tok)
                pos.append(p)
                slot_l.append((s * self.per_seq + p // bs) * bs + p % bs)
            slots.append(slots[-1] + len(t))
        decode = all(len(t) == 1 for t in toks)
        nd = len(seqs) if decode else 0
        bt = torch.tensor([[s * self.per_seq + j for j in range(self.per_seq)] for s in seqs],
                          dtype=torch.int32)
        sl = torch.tensor([st + len(t) for t, st in zip(toks, starts)], dtype=torch.int32)
        cu_q = torch.tensor(slots, dtype=torch.int32)
        logits_idx = torch.tensor([c - 1 for c in slots[1:]], dtype=torch.int64)
        dev = self.device
        tiles = None
        if not decode:
            ts, tr = prefill_tiles(slots, 0, self.model.group, head_dim=self.model.d,
                                   block_size=self.bs)
            tiles = (torch.tensor(ts, dtype=torch.int32, device=dev),
                     torch.tensor(tr, dtype=torch.int32, device=dev))
        return ForwardBatch(
            input_ids=torch.tensor(ids, dtype=torch.int32, device=dev),
            positions=torch.tensor(pos, dtype=torch.int32, device=dev),
            slots=torch.tensor(slot_l, dtype=torch.int32, device=dev),
            block_tables=bt.to(dev), seq_lens=sl.to(dev), cu_q=cu_q.to(dev),
            logits_idx=logits_idx.to(dev), num_decode=nd,
            tile_seq=tiles[0] if tiles else None, tile_row0=tiles[1] if tiles else None,
            decode_splits=ops.decode_splits(nd, self.model.hkv, int(sl.max()))
            if (decode and dev.type == "cuda") else 1,
            seq_lens_cpu=sl, cu_q_cpu=cu_q)

    # ---- one pipelined step ------------------------------------------------------------
    def _step(self, seqs: List[int], toks: List[List[int]], starts: List[int]) -> List[int]:
        n = len(seqs)
        mbs = max(1, min(self.mb, n))
        bounds = [(n * i // mbs, n * (i + 1) // mbs) for i in range(mbs)]
        out: List[int] = []
        for a, b in bounds:
            if a == b:
                continue
            fb = self._batch(seqs[a:b], toks[a:b], starts[a:b])
            T = fb.num_tokens
            x_in = None
            if not self.first:
                x_in = torch.empty(T, self.hidden, dtype=torch.bfloat16, device=self.device)
                dist.recv(x_in, self.rank - 1, group=self.group)
            y = self.model.forward_stage(fb, self.kv, x_in, first=self.first, last=self.last)
            if not self.last:
                dist.send(y.contiguous(), self.rank + 1, group=self.group)
            else:
                # greedy, first maximum wins
                mx = y.max(dim=1, keepdim=True).values
                idx = torch.arange(y.shape[1], device=y.device).expand_as(y)
                first_max = torch.where(y == mx, idx, y.shape[1]).min(dim=1).values
                out.extend(first_max.tolist())
        # the last stage tells every stage the tokens of this step
        t = torch.tensor(out if self.last else [0] * n, dtype=torch.int64,
                         device=self.device if self.device.type == "cuda" else "cpu")
        dist.broadcast(t, self.world - 1, group=self.group)
        return t.tolist()

    def generate(self, prompts: List[List[int]], max_new_tokens: int) -> List[List[int]]:
        assert len(prompts) <= self.max_seqs
        seqs = list(range(len(prompts)))
        outs: List[List[int]] = [[] for _ in prompts]
        nxt = self._step(seqs, prompts, [0] * len(prompts))
        lens = [len(p) for p in prompts]
        for i, t in enumerate(nxt):
            outs[i].append(t)
        for _ in range(max_new_tokens - 1):
            nxt = self._step(seqs, [[o[-1]] for o in outs], lens)
            lens = [l + 1 for l in lens]
            for i, t in enumerate(nxt):
                outs[i].append(t)
        return outs


def main(argv=None) -> int:
    """Self-check under torchrun: the pipeline's greedy tokens vs the fp32 oracle.

        torchrun --nproc-per-node N -m lightbulb_b200.parallel.pp [--micro-batches M]
    """
    import argparse
    import os
    ap = argparse.ArgumentParser()
    ap.add_argument("--micro-batches", type=int, default=0)
    ap.add_argument("--tokens", type=int, default=6)
    a = ap.parse_args(argv)
    from ..config import get_preset
    from ..models.reference import ReferenceLlama, greedy_generate
    from ..models.weights import random_weights
    from .comm import init_distributed
    rank, world, local = init_distributed(timeout_s=60)
    cuda = torch.cuda.is_available()
    dev = torch.device("cuda", local) if cuda else torch.device("cpu")
    cfg = get_preset("tiny-test", num_layers=max(2, world * 2))
    w = random_weights(cfg, seed=11, std=0.05)
    w = {k: v.to(torch.bfloat16).float() for k, v in w.items()}
    eng = PipelineEngine(cfg, pack_stage(cfg, w, rank, world, device=dev), rank, world, dev,
                         max_seqs=4, max_len=128, micro_batches=a.micro_batches)
    prompts = [list(range(5, 30)), [9, 8, 7], [100] * 17]
    outs = eng.generate(prompts, a.tokens)
    ok = True
    if rank == 0:
        ref = ReferenceLlama(cfg, w)
        for p, o in zip(prompts, outs):
            r = greedy_generate(ref, p, a.tokens)
            print("pp", o, "oracle", r, flush=True)
            ok &= (r == o)
    flag = torch.tensor([1 if ok else 0], dtype=torch.int64,
                        device=dev if cuda else "cpu")
    dist.broadcast(flag, 0)
    dist.destroy_process_group()
    return 0 if int(flag) == 1 else 1


if __name__ == "__main__":
    import sys
    sys.exit(main())
