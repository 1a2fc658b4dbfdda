"""Llama-family decoder over the sm_100a op set, with a paged KV cache.

Covers the reference's model graph (``src/model/custom_transformer.rs:450-628``
BatchedTransformer, ``custom_transformer_block.rs:304-357`` pre-LN blocks,
``custom_attention.rs:250-674`` attention, ``mlp_wrapper.rs:154-199`` SwiGLU) and the Fuel
batched paged decoder (``src/model_fuel/batched.rs:570-826``) in one forward that mixes
decode rows and chunked-prefill rows in the same step:

* one fused QKV GEMM, RoPE + paged KV append in one kernel (per-row positions);
* paged attention: the decode kernel for single-token rows, the prefill kernel for the rest;
* o_proj -> fused residual add + RMSNorm -> gate_up GEMM with SwiGLU epilogue -> down_proj ->
  fused residual add + next layer's RMSNorm;
* logits (fp32) only for the rows that sample.

Tensor parallelism (``comm`` hooks) is injected by :mod:`lightbulb_b200.parallel.tp`.
"""
from __future__ import annotations

import math

from dataclasses import dataclass
from typing import Callable, List, Optional

import torch

from .. import ops
from ..config import ModelConfig


class KVCache:
    """Paged KV storage: per layer K and V tensors of shape [num_blocks, Hkv, BS, D]."""

    def __init__(self, num_layers: int, num_blocks: int, num_kv_heads: int, block_size: int,
                 head_dim: int, dtype=torch.bfloat16, device="cuda"):
        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.storage = torch.zeros(num_layers, 2, num_blocks, num_kv_heads, block_size, head_dim,
                                   dtype=dtype, device=device)
        self.k = [self.storage[i, 0] for i in range(num_layers)]
        self.v = [self.storage[i, 1] for i in range(num_layers)]

    @staticmethod
    def bytes_per_block(num_layers, num_kv_heads, block_size, head_dim, elt=2) -> int:
        return num_layers * 2 * num_kv_heads * block_size * head_dim * elt

    def copy_blocks(self, pairs: List[int]) -> None:
        """Copy-on-write: pairs = [src0, dst0, src1, dst1, ...]."""
        if not pairs:
            return
        src = torch.tensor(pairs[0::2], device=self.storage.device, dtype=torch.long)
        dst = torch.tensor(pairs[1::2], device=self.storage.device, dtype=torch.long)
        self.storage[:, :, dst] = self.storage[:, :, src]


@dataclass
class ForwardBatch:
    """Device-side inputs of one forward step (tokens ordered: decode seqs first)."""

    input_ids: torch.Tensor      # [T] int32
    positions: torch.Tensor      # [T] int32
    slots: torch.Tensor          # [T] int32 (block * BS + offset, -1 = no KV write)
    block_tables: torch.Tensor   # [B, W] int32
    seq_lens: torch.Tensor       # [B] int32: KV length after this step
    cu_q: torch.Tensor           # [B + 1] int32
    logits_idx: torch.Tensor     # [R] int64 rows that produce logits
    num_decode: int              # first num_decode sequences have exactly one query token
    tile_seq: Optional[torch.Tensor] = None    # prefill attention work list
    tile_row0: Optional[torch.Tensor] = None
    decode_splits: int = 1
    seq_lens_cpu: Optional[torch.Tensor] = None
    cu_q_cpu: Optional[torch.Tensor] = None

    @property
    def num_tokens(self) -> int:
        return self.input_ids.shape[0]


def prefill_tiles(cu_q: List[int], first_seq: int, group: int,
                  rows_per_tile: Optional[int] = None, block_size: int = 16,
                  head_dim: int = 128):
    """Work list for the prefill attention kernel: (seq, first packed row) per CTA, with the
    tile height of the kernel that ``ops.paged_attention`` selects for this geometry."""
    if rows_per_tile is None:
        rows_per_tile = ops.prefill_rows_per_tile(group, block_size, head_dim)
    seqs, rows = [], []
    for s in range(first_seq, len(cu_q) - 1):
        n = (cu_q[s + 1] - cu_q[s]) * group
        for r in range(0, n, rows_per_tile):
            seqs.append(s)
            rows.append(r)
    return seqs, rows


class LlamaModel:
    """Weights in device layout (see ``models/weights.py``) + forward."""

    def __init__(self, cfg: ModelConfig, packed: dict, tp_rank: int = 0, tp_size: int = 1,
                 max_positions: Optional[int] = None, comm=None):
        self.cfg = cfg
        self.w = packed
        self.layers = packed["layers"]
        self.tp_rank, self.tp_size = tp_rank, tp_size
        self.hq = cfg.num_heads // tp_size
        self.hkv = max(1, cfg.num_kv_heads // tp_size)
        self.d = cfg.head_dim_padded          # device head width (narrow heads zero-padded)
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        self.group = self.hq // self.hkv
        ref = packed.get("embed")
        self.device = (ref if ref is not None else packed["layers"][0]["qkv"]).device
        mp = max_positions or cfg.max_position_embeddings
        self.cos_sin = ops.rope_table(mp, cfg.head_dim, cfg.rope_theta, self.device)
        self.comm = comm  # tensor-parallel communicator (None = single GPU)
        self.h2o = None   # H2O policy: accumulates last-layer attention mass (kv/compression.py)
        self.vocab_local = packed["lm_head"].shape[0] if "lm_head" in packed else 0

    # ------------------------------------------------------------------------------
    def fused_ok(self, b: ForwardBatch) -> bool:
        c = self.comm
        if c is None or c.world <= 1 or not getattr(c, "fused_requested", False):
            return False
        if self.device.type != "cuda":
            return False
        T = b.num_tokens
        return (b.num_decode == len(b.cu_q) - 1 == T and T % c.world == 0 and
                T <= getattr(c, "fused_max_rows", 512) and b.logits_idx.numel() == T)

    def forward_fused(self, b: ForwardBatch, kv: KVCache) -> torch.Tensor:
        """Decode step with GEMM + reduce-scatter + residual + RMSNorm + all-gather fused over
        NVLink peer memory (see :mod:`lightbulb_b200.parallel.fused`)."""
        from ..parallel.fused import ensure_fused
        cfg = self.cfg
        F = ensure_fused(self.comm, cfg.hidden_size, self.device)
        T = b.num_tokens
        R = T // F.world
        r0 = F.rank * R
        hq, hkv, d = self.hq, self.hkv, self.d
        eps = cfg.rms_norm_eps
        x = F.residual[:R]
        ops.embedding(b.input_ids[r0:r0 + R], self.w["embed"], out=x)
        F.norm_gather(self.layers[0]["ln_in"], R, eps, x_in=x, add_residual=False)
        h = F.gather[:T]
        attn = torch.empty(T, hq * d, dtype=torch.bfloat16, device=self.device)
        for i, L in enumerate(self.layers):
            qkv = F.gemm_consume(h, L["qkv"])
            self._rope_kv(qkv, b, kv, i, L)
            q = qkv[:, :hq * d].view(T, hq, d)
            ops.paged_attention(q, kv.k[i], kv.v[i], b.block_tables, b.seq_lens, b.cu_q,
                                attn.view(T, hq, d), self.group, decode=True,
                                num_splits=b.decode_splits, scale=self.scale)
            F.gemm_scatter(attn, L["o"], R)
            F.norm_gather(L["ln_post"], R, eps)
            act = F.gemm_consume(h, L["gate_up"], mode=ops.EPI_SWIGLU)
            F.gemm_scatter(act, L["down"], R)
            nw = self.layers[i + 1]["ln_in"] if i + 1 < len(self.layers) else self.w["norm"]
            F.norm_gather(nw, R, eps)
        return F.gemm_consume(h, self.w["lm_head"], mode=ops.EPI_F32)

    def rowpar_ok(self, b: ForwardBatch) -> bool:
        c = self.comm
        X = getattr(c, "rowpar", None) if c is not None else None
        return X is not None and self.device.type == "cuda" and X.fits(b.num_tokens)

    def forward_rowpar(self, b: ForwardBatch, kv: KVCache) -> torch.Tensor:
        """Tensor-parallel forward over the row-parallel exchange
        (:mod:`lightbulb_b200.parallel.rowpar`): every row-parallel GEMM is followed by ONE
        kernel that reduces this rank's token rows, adds them to its shard of the residual
        stream, normalises them and all-gathers the normalised rows; decode-sized batches push
        the GEMM output straight from its epilogue into the owners' receive slots."""
        from ..parallel.rowpar import owned_rows
        cfg = self.cfg
        X = self.comm.rowpar
        T = b.num_tokens
        hq, hkv, d = self.hq, self.hkv, self.d
        eps = cfg.rms_norm_eps
        x = ops.embedding(b.input_ids, self.w["embed"])      # every row; only own rows kept
        h = ops.rmsnorm(x, self.layers[0]["ln_in"], eps)
        r0, n = owned_rows(T, X.world, X.rank)
        x_own = x[r0:r0 + n]                                  # this rank's residual rows
        attn = torch.empty(T, hq * d, dtype=torch.bfloat16, device=self.device)
        nd = b.num_decode
        nl = len(self.layers)
        for i, L in enumerate(self.layers):
            qkv = ops.gemm(h, L["qkv"])
            self._rope_kv(qkv, b, kv, i, L)
            q = qkv[:, :hq * d].view(T, hq, d)
            a3 = attn.view(T, hq, d)
            if nd > 0:
                ops.paged_attention(q, kv.k[i], kv.v[i], b.block_tables[:nd], b.seq_lens[:nd],
                                    b.cu_q[:nd + 1], a3, self.group, decode=True,
                                    num_splits=b.decode_splits, scale=self.scale,
                                    seq_lens_cpu=b.seq_lens_cpu, cu_q_cpu=b.cu_q_cpu)
            if b.tile_seq is not None and b.tile_seq.numel() > 0:
                ops.paged_attention(q, kv.k[i], kv.v[i], b.block_tables, b.seq_lens, b.cu_q,
                                    a3, self.group, decode=False, tile_seq=b.tile_seq,
                                    tile_row0=b.tile_row0, seq_lens_cpu=b.seq_lens_cpu,
                                    cu_q_cpu=b.cu_q_cpu, scale=self.scale)
            if self.h2o is not None and nd > 0 and i == nl - 1:
                self.h2o.accumulate(q[:nd], kv.k[i], b.block_tables[:nd], b.seq_lens[:nd])
            h = X.gemm_norm(attn, L["o"], x_own, L["ln_post"], eps)
            act = ops.gemm(h, L["gate_up"], mode=ops.EPI_SWIGLU)
            nw = self.layers[i + 1]["ln_in"] if i + 1 < nl else self.w["norm"]
            h = X.gemm_norm(act, L["down"], x_own, nw, eps)
        hl = h.index_select(0, b.logits_idx) if b.logits_idx.numel() != T else h
        return ops.gemm(hl, self.w["lm_head"], mode=ops.EPI_F32)

    def forward(self, b: ForwardBatch, kv: KVCache) -> torch.Tensor:
        """Returns fp32 logits [len(b.logits_idx), vocab_local]."""
        if self.fused_ok(b):
            return self.forward_fused(b, kv)
        if self.rowpar_ok(b):
            return self.forward_rowpar(b, kv)
        return self.forward_stage(b, kv)

    def forward_stage(self, b: ForwardBatch, kv: KVCache, x_in: Optional[torch.Tensor] = None,
                      first: bool = True, last: bool = True) -> torch.Tensor:
        """The layers this model holds, as one pipeline stage: ``first`` embeds ``b.input_ids``
        (else ``x_in`` is the residual stream [T, H] from the previous stage), ``last`` applies
        the final norm and the LM head (fp32 logits of ``b.logits_idx``); a middle or first
        stage returns the residual stream after its last layer."""
        cfg = self.cfg
        T = b.num_tokens
        hq, hkv, d = self.hq, self.hkv, self.d
        eps = cfg.rms_norm_eps
        dev = self.device
        comm = self.comm

        if first:
            x = ops.embedding(b.input_ids, self.w["embed"])      # residual stream [T, H]
        else:
            x = x_in
        h = ops.rmsnorm(x, self.layers[0]["ln_in"], eps)
        attn = torch.empty(T, hq * d, dtype=torch.bfloat16, device=dev)
        nd = b.num_decode
        for i, L in enumerate(self.layers):
            qkv = ops.gemm(h, L["qkv"])
            self._rope_kv(qkv, b, kv, i, L)
            q = qkv[:, :hq * d].view(T, hq, d)
            a3 = attn.view(T, hq, d)
            if nd > 0:
                ops.paged_attention(q, kv.k[i], kv.v[i], b.block_tables[:nd], b.seq_lens[:nd],
                                    b.cu_q[:nd + 1], a3, self.group, decode=True,
                                    num_splits=b.decode_splits, scale=self.scale,
                                    seq_lens_cpu=b.seq_lens_cpu, cu_q_cpu=b.cu_q_cpu)
            if b.tile_seq is not None and b.tile_seq.numel() > 0:
                ops.paged_attention(q, kv.k[i], kv.v[i], b.block_tables, b.seq_lens, b.cu_q,
                                    a3, self.group, decode=False, tile_seq=b.tile_seq,
                                    tile_row0=b.tile_row0, seq_lens_cpu=b.seq_lens_cpu,
                                    cu_q_cpu=b.cu_q_cpu, scale=self.scale)
            if self.h2o is not None and nd > 0 and i == len(self.layers) - 1 and last:
                self.h2o.accumulate(q[:nd], kv.k[i], b.block_tables[:nd], b.seq_lens[:nd])
            if comm is not None:
                h = comm.gemm_all_reduce_rmsnorm(attn, L["o"], x, L["ln_post"], eps)
            else:
                h = ops.rmsnorm(ops.gemm(attn, L["o"]), L["ln_post"], eps, residual=x)
            act = ops.gemm(h, L["gate_up"], mode=ops.EPI_SWIGLU)
            if i + 1 < len(self.layers):
                nw = self.layers[i + 1]["ln_in"]
            elif last:
                nw = self.w["norm"]
            else:
                nw = self._ones(x.shape[1])  # stage boundary: only the residual update matters
            if comm is not None:
                h = comm.gemm_all_reduce_rmsnorm(act, L["down"], x, nw, eps)
            else:
                h = ops.rmsnorm(ops.gemm(act, L["down"]), nw, eps, residual=x)
        if not last:
            return x
        hl = h.index_select(0, b.logits_idx) if b.logits_idx.numel() != T else h
        return ops.gemm(hl, self.w["lm_head"], mode=ops.EPI_F32)

    def _rope_kv(self, qkv: torch.Tensor, b: ForwardBatch, kv: KVCache, i: int, L) -> None:
        """RoPE + paged KV append of layer ``i`` (with Qwen3's per-head q/k RMSNorm when the
        layer carries ``q_norm`` / ``k_norm``)."""
        ops.rope_kv(qkv, b.positions, b.slots, self.cos_sin, kv.k[i], kv.v[i], self.hq,
                    self.hkv, q_norm=L.get("q_norm"), k_norm=L.get("k_norm"),
                    norm_dim=self.cfg.head_dim, eps=self.cfg.rms_norm_eps)

    def _ones(self, n: int) -> torch.Tensor:
        t = getattr(self, "_ones_cache", None)
        if t is None or t.numel() != n:
            t = torch.ones(n, dtype=torch.bfloat16, device=self.device)
            self._ones_cache = t
        return t
