"""Operator layer.

CUDA tensors are served by the hand-written sm_100a kernels in ``lightbulb_b200._C``; if
that extension is missing on a CUDA device every op raises (there is no silent eager
fallback on the GPU).  CPU tensors are served by plain-PyTorch restatements of the same
math so that the engine, scheduler and model plumbing run in CPU tests.
"""
from __future__ import annotations

import math
import threading
from typing import Optional

import torch

try:  # the extension is built in-tree by ``python setup.py build_ext --inplace``
    from .. import _C  # type: ignore
except Exception as _e:  # pragma: no cover - exercised on machines without the build
    _C = None
    _C_ERR = _e
else:
    _C_ERR = None

EPI_STORE, EPI_SWIGLU, EPI_F32 = 0, 1, 2
SPLITS_STREAMK = 1000   # gemm(splits=...): stream-K over (tile, k-block) in the persistent kernel
GEMV_MAX_ROWS = 4       # gemm() with at most this many rows (and an automatic plan) uses the GEMV

# Decode attention implementation: "tma" (warp-specialised TMA pipeline, default) or
# "cpasync" (the generic paged kernel, also used for non-16 block sizes).
import os as _os
_DECODE_IMPL = _os.environ.get("LB_DECODE_ATTN", "tma")

# Number of our own CUDA kernels launched (eager calls counted here; CUDA-graph replays add
# the count recorded when the graph was captured).
_launches = [0]


def launch_counter_reset() -> None:
    _launches[0] = 0


def launch_counter_value() -> int:
    return _launches[0]


def launch_counter_add(n: int) -> None:
    _launches[0] += n


def have_cuda_kernels() -> bool:
    return _C is not None


def _need_c():
    if _C is None:
        raise RuntimeError(
            "lightbulb_b200._C (sm_100a kernels) is not built; run `python setup.py build_ext "
            f"--inplace`: {_C_ERR}")
    return _C


class _DeviceScratch:
    """Per-device workspaces shared by kernels that run back to back on one stream:
    split-K partial tiles + tile counters for the GEMM, split-KV partials for attention,
    and the device error word every bounded wait reports into."""

    def __init__(self, device: torch.device, ws_floats: int = 24 << 20):
        self.device = device
        self.gemm_ws = torch.empty(ws_floats, dtype=torch.float32, device=device)
        self.gemm_counters = torch.zeros(1 << 16, dtype=torch.int32, device=device)
        self.err = torch.zeros(4, dtype=torch.int32, device=device)
        self.attn_o: Optional[torch.Tensor] = None
        self.attn_lse: Optional[torch.Tensor] = None
        self._retired: list = []

    def attn_buffers(self, splits: int, rows: int, d: int):
        need = splits * rows
        if self.attn_lse is None or self.attn_lse.numel() < need:
            # Never free a replaced buffer: captured CUDA graphs may still point at it.
            if self.attn_o is not None:
                self._retired.append((self.attn_o, self.attn_lse))
            need = max(need, 1 << 16)
            self.attn_o = torch.empty(need * d, dtype=torch.float32, device=self.device)
            self.attn_lse = torch.empty(need, dtype=torch.float32, device=self.device)
        return self.attn_o, self.attn_lse


_scratch: dict = {}
_lock = threading.Lock()


def scratch(device: torch.device) -> _DeviceScratch:
    key = (device.type, device.index if device.index is not None else torch.cuda.current_device())
    s = _scratch.get(key)
    if s is None:
        with _lock:
            s = _scratch.get(key)
            if s is None:
                s = _DeviceScratch(torch.device("cuda", key[1]))
                _scratch[key] = s
    return s


class KernelError(RuntimeError):
    pass


_ERR_NAMES = {1: "TMA load wait timed out", 2: "smem slot wait timed out",
              3: "TMEM accumulator wait timed out", 4: "TMEM release wait timed out",
              5: "peer flag wait timed out", 6: "index out of bounds", 7: "drain timed out"}


def check_errors(device: Optional[torch.device] = None, reset: bool = True) -> None:
    """Raise if any kernel on ``device`` recorded an error (bounded wait expired, OOB)."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    s = scratch(dev)
    code = int(s.err[0].item())
    if code:
        if reset:
            s.err.zero_()
        raise KernelError(f"device kernel error {code}: {_ERR_NAMES.get(code, '?')}")


# ------------------------------------------------------------------------------------
# GEMM
# ------------------------------------------------------------------------------------
def gemm(a: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
         residual: Optional[torch.Tensor] = None, mode: int = EPI_STORE, bt: int = 0,
         splits: int = 0) -> torch.Tensor:
    """``out = a @ w.T`` (+ residual) with epilogue ``mode``:
    EPI_STORE -> bf16 [M, N]; EPI_F32 -> fp32 [M, N]; EPI_SWIGLU -> bf16 [M, N/2] of
    ``silu(gate) * up`` for gate/up rows interleaved in 64-row groups."""
    from ..formats.quant import QuantWeight
    if isinstance(w, QuantWeight):
        return gemm_quant(a, w, out, mode, splits)
    m, n = a.shape[0], w.shape[0]
    if out is None:
        if mode == EPI_SWIGLU:
            out = torch.empty(m, n // 2, dtype=torch.bfloat16, device=a.device)
        elif mode == EPI_F32:
            out = torch.empty(m, n, dtype=torch.float32, device=a.device)
        else:
            out = torch.empty(m, n, dtype=torch.bfloat16, device=a.device)
    if a.is_cuda:
        C = _need_c()
        if 0 < m <= GEMV_MAX_ROWS and bt == 0 and splits == 0 and a.shape[1] % 8 == 0:
            # 1-4 tokens: a pure weight stream, served by the GEMV kernel
            C.gemv_bf16(a, w, out, residual, mode)
            _launches[0] += 1
            return out
        s = scratch(a.device)
        if splits < 0:
            # a forced cluster split-K plan must fit the shared workspace: refuse it here rather
            # than in the extension
            need = gemm_plan(m, n, a.shape[1], bt, splits)[3]
            if need > s.gemm_ws.numel():
                raise ValueError(f"gemm: cluster split-K plan (bt {bt}, splits {splits}) needs "
                                 f"{need} workspace floats > {s.gemm_ws.numel()}")
        C.gemm_bf16(a, w, out, residual, mode, s.gemm_ws, s.gemm_counters, s.err, bt, splits,
                    None)
        _launches[0] += 1
        return out
    # CPU restatement
    y = a.float() @ w.float().T
    if mode == EPI_SWIGLU:
        g = y.view(m, -1, 2, 64)
        y = (torch.nn.functional.silu(g[:, :, 0]) * g[:, :, 1]).reshape(m, -1)
        out.copy_(y.to(out.dtype))
    elif mode == EPI_F32:
        out.copy_(y)
    else:
        if residual is not None:
            y = y + residual.float()
        out.copy_(y.to(out.dtype))
    return out


def gemm_pair(a: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
              residual: Optional[torch.Tensor] = None, mode: int = EPI_STORE,
              bt: int = 0) -> torch.Tensor:
    """:func:`gemm` on SM pairs (tcgen05 ``cta_group::2``, 256-row weight tiles), bypassing the
    dispatch policy (tests and benchmarks)."""
    m, n = a.shape[0], w.shape[0]
    if out is None:
        cols = n // 2 if mode == EPI_SWIGLU else n
        dt = torch.float32 if mode == EPI_F32 else torch.bfloat16
        out = torch.empty(m, cols, dtype=dt, device=a.device)
    _need_c().gemm_bf16_pair(a, w, out, residual, mode, scratch(a.device).err, bt)
    _launches[0] += 1
    return out


def use_int_zero_kernel(w) -> bool:
    """Small batches of 4-bit weights with integer zero points (AWQ) run on the integer-weight
    kernel (``gemm_quant_iz``: weights exact in tensor memory, scale applied per group after
    the MMA); ``LB_QUANT_IZ=0`` keeps them on the full-dequant kernel."""
    return (getattr(w, "int_zero", False) and w.bits == 4 and w.group % 64 == 0
            and _os.environ.get("LB_QUANT_IZ", "1") != "0")


def gemm_quant(a: torch.Tensor, w, out: Optional[torch.Tensor] = None, mode: int = EPI_STORE,
               splits: int = 0) -> torch.Tensor:
    """``a @ dequant(w).T`` for a :class:`~lightbulb_b200.formats.quant.QuantWeight`."""
    m, n = a.shape[0], w.shape[0]
    if out is None:
        if mode == EPI_SWIGLU:
            out = torch.empty(m, n // 2, dtype=torch.bfloat16, device=a.device)
        elif mode == EPI_F32:
            out = torch.empty(m, n, dtype=torch.float32, device=a.device)
        else:
            out = torch.empty(m, n, dtype=torch.bfloat16, device=a.device)
    if a.is_cuda:
        sc = scratch(a.device)
        if m <= 32 and use_int_zero_kernel(w):
            _need_c().gemm_quant_iz(a, w.qw, w.scales, w.offsets, w.group, out, mode,
                                    max(0, splits), sc.err, sc.gemm_ws)
        else:
            _need_c().gemm_quant(a, w.qw, w.scales, w.offsets, w.bits, w.group, out, mode,
                                 max(0, splits), sc.err, sc.gemm_ws)
        _launches[0] += 1
        return out
    return gemm(a, w.dequantize(torch.bfloat16), out, None, mode)


def gemm_plan(m: int, n: int, k: int, bt: int = 0, splits: int = 0):
    return tuple(_need_c().gemm_plan(m, n, k, bt, splits))


# ------------------------------------------------------------------------------------
# Norm / embedding / rope
# ------------------------------------------------------------------------------------
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, residual: Optional[torch.Tensor] = None,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """If ``residual`` is given: ``residual += x`` then ``out = rmsnorm(residual)``."""
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    if x.is_cuda:
        _need_c().rmsnorm(x, residual, w, out, eps)
        _launches[0] += 1
        return out
    if residual is not None:
        residual.copy_((residual.float() + x.float()).to(residual.dtype))
        src = residual.float()
    else:
        src = x.float()
    y = src * torch.rsqrt(src.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    out.copy_(y.to(out.dtype))
    return out


def forward_tokens(ids: torch.Tensor, src: torch.Tensor, last: torch.Tensor) -> None:
    """In place: ``ids[i] = last[src[i]]`` where ``src[i] >= 0`` (overlapped decode feeds the
    previous step's sampled tokens without a host round trip)."""
    if ids.is_cuda:
        _need_c().forward_tokens(ids, src, last, scratch(ids.device).err)
        _launches[0] += 1
        return
    n = ids.shape[0]
    s = src[:n].long()
    m = s >= 0
    if bool(m.any()):
        ids[m] = last[s[m]].to(ids.dtype)


def embedding(ids: torch.Tensor, table: torch.Tensor, out: Optional[torch.Tensor] = None):
    if out is None:
        out = torch.empty(ids.shape[0], table.shape[1], dtype=table.dtype, device=table.device)
    if table.is_cuda:
        _need_c().embedding(ids, table, out, scratch(table.device).err)
        _launches[0] += 1
        return out
    out.copy_(table[ids.long()])
    return out


def rope_table(max_pos: int, head_dim: int, theta: float, device) -> torch.Tensor:
    """[max_pos, head_dim] fp32: cos(pos * inv_freq) | sin(pos * inv_freq), computed in fp64."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cat([torch.cos(ang), torch.sin(ang)], dim=1).float().to(device)


def rope_kv(qkv: torch.Tensor, positions: torch.Tensor, slots: Optional[torch.Tensor],
            cos_sin: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, hq: int,
            hkv: int, q_norm: Optional[torch.Tensor] = None,
            k_norm: Optional[torch.Tensor] = None, norm_dim: int = 0,
            eps: float = 1e-6) -> None:
    """Rotate q (in place) and k of ``qkv`` [T, (hq + 2 hkv) D] and write k, v to their slots.
    D = the cache's head width; the rotation covers the first ``cos_sin.shape[1]`` lanes of
    each head (the true head_dim when heads are zero-padded).  ``q_norm`` / ``k_norm`` [D]:
    per-head RMSNorm (over ``norm_dim`` lanes) of q / k before the rotation (Qwen3)."""
    if qkv.is_cuda:
        _need_c().rope_kv(qkv, positions, slots, cos_sin, k_cache, v_cache, hq, hkv,
                          scratch(qkv.device).err, q_norm, k_norm, norm_dim, eps)
        _launches[0] += 1
        return
    d = k_cache.shape[-1]           # head stride (padded width)
    r = cos_sin.shape[1]            # rotary width (true head_dim)
    t = qkv.shape[0]
    half = r // 2
    cs = cos_sin[positions.long()]
    c, s = cs[:, None, :half], cs[:, None, half:]
    x = qkv[:, :(hq + hkv) * d].view(t, hq + hkv, d).float()
    nd = norm_dim or r
    for lo, hi, nw in ((0, hq, q_norm), (hq, hq + hkv, k_norm)):
        if nw is not None:
            xs = x[:, lo:hi]
            inv = torch.rsqrt(xs.pow(2).sum(-1, keepdim=True) / nd + eps)
            x[:, lo:hi] = (xs * inv * nw.float()).to(qkv.dtype).float()
    x1, x2 = x[..., :half], x[..., half:r]
    rot = torch.cat([x1 * c - x2 * s, x1 * s + x2 * c, x[..., r:]], -1).to(qkv.dtype)
    qkv[:, :hq * d].copy_(rot[:, :hq].reshape(t, -1))
    if slots is not None:
        bs = k_cache.shape[2]
        sl = slots.long()
        ok = sl >= 0
        blk, off = sl[ok] // bs, sl[ok] % bs
        k = rot[:, hq:][ok]
        v = qkv[:, (hq + hkv) * d:(hq + 2 * hkv) * d].view(t, hkv, d)[ok]
        k_cache[blk, :, off] = k
        v_cache[blk, :, off] = v


# ------------------------------------------------------------------------------------
# Attention
# ------------------------------------------------------------------------------------
def decode_splits(num_seqs: int, num_kv_heads: int, max_kv_len: int, sms: int = 148,
                  ctas_per_sm: int = 2) -> int:
    """Split-KV factor for decode.  Splitting only pays when the (sequence, KV head) CTAs
    cannot fill one wave of ``sms * ctas_per_sm`` slots (measured: at 512 CTAs a 4-way split
    is 1.6x slower than none); then split so the CTAs cover the slots, each split keeping
    >= 512 keys."""
    ctas = num_seqs * num_kv_heads
    slots = sms * ctas_per_sm
    if ctas == 0 or ctas >= slots:
        return 1
    return max(1, min(32, (slots + ctas - 1) // ctas, max(1, max_kv_len // 512)))


_PREFILL_IMPL = _os.environ.get("LB_PREFILL_ATTN", "tc")


def prefill_rows_per_tile(group: int, block_size: int = 16, head_dim: int = 128) -> int:
    """Packed query rows per CTA of the prefill / verify attention kernel that will run for
    this geometry: 256 for the tcgen05 kernel (two 128-row query tiles; block size 16, head
    dim 128, power-of-two GQA group <= 16; ``LB_PREFILL_ATTN=fa2`` selects the mma.sync
    kernel), 64 otherwise.  The work list (``models.llama.prefill_tiles``) must be built with
    the same value."""
    if (_PREFILL_IMPL == "tc" and block_size == 16 and head_dim == 128 and 1 <= group <= 16
            and group & (group - 1) == 0):
        return 256
    return 64


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    block_tables: torch.Tensor, seq_lens: torch.Tensor, cu_q: torch.Tensor,
                    out: torch.Tensor, group: int, decode: bool,
                    tile_seq: Optional[torch.Tensor] = None,
                    tile_row0: Optional[torch.Tensor] = None, num_splits: int = 1,
                    causal: bool = True, seq_lens_cpu=None, cu_q_cpu=None,
                    scale: Optional[float] = None) -> torch.Tensor:
    """q: [T, Hq, D] (may be a strided view of the QKV buffer); out: [T, Hq, D].  ``scale``
    defaults to 1 / sqrt(D) (pass 1 / sqrt(true head_dim) for zero-padded heads)."""
    d = q.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    if q.is_cuda:
        C = _need_c()
        po = pl = None
        if decode and num_splits > 1:
            po, pl = scratch(q.device).attn_buffers(num_splits, q.shape[0] * q.shape[1], d)
        if decode and k_cache.shape[2] == 16 and group <= 16 and _DECODE_IMPL == "tma":
            # one query token per sequence, token i belongs to sequence i
            C.paged_decode_tma(q, k_cache, v_cache, out, block_tables, seq_lens, group, scale,
                               num_splits, po, pl, scratch(q.device).err)
            _launches[0] += 2 if num_splits > 1 else 1
            return out
        if not decode and prefill_rows_per_tile(group, k_cache.shape[2], d) == 256:
            C.paged_attention_tc(q, k_cache, v_cache, out, block_tables, seq_lens, cu_q,
                                 tile_seq, tile_row0, group, scale, causal,
                                 scratch(q.device).err)
            _launches[0] += 1
            return out
        C.paged_attention(q, k_cache, v_cache, out, block_tables, seq_lens, cu_q, tile_seq,
                          tile_row0, group, scale, decode, num_splits, po, pl, causal,
                          scratch(q.device).err)
        _launches[0] += 2 if (decode and num_splits > 1) else 1
        return out
    # CPU restatement
    bs = k_cache.shape[2]
    nseq = seq_lens.shape[0]
    sl = (seq_lens_cpu if seq_lens_cpu is not None else seq_lens).tolist()[:nseq]
    cq = (cu_q_cpu if cu_q_cpu is not None else cu_q).tolist()[:nseq + 1]
    from ..models.reference import attention_ref
    for i, L in enumerate(sl):
        q0, q1 = cq[i], cq[i + 1]
        if q1 == q0:
            continue
        nb = (L + bs - 1) // bs
        blocks = block_tables[i, :nb].long()
        k = k_cache[blocks].permute(0, 2, 1, 3).reshape(nb * bs, k_cache.shape[1], d)[:L]
        v = v_cache[blocks].permute(0, 2, 1, 3).reshape(nb * bs, v_cache.shape[1], d)[:L]
        qpos = torch.arange(L - (q1 - q0), L)
        o = attention_ref(q[q0:q1], k, v, qpos, torch.arange(L), causal=causal, scale=scale)
        out[q0:q1] = o.to(out.dtype)
    return out


# ------------------------------------------------------------------------------------
# Sampling
# ------------------------------------------------------------------------------------
def sample(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
           top_p: torch.Tensor, seeds: torch.Tensor, out: Optional[torch.Tensor] = None,
           logprobs: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    if logits.is_cuda:
        _need_c().sample_tokens(logits, temperature, top_k, top_p, seeds, out, logprobs)
        _launches[0] += 1
        return out
    from ..engine.sampling import sample_row_reference
    for r in range(logits.shape[0]):
        out[r] = sample_row_reference(logits[r], float(temperature[r]), int(top_k[r]),
                                      float(top_p[r]), int(seeds[r]))
    return out
