"""KV compression policies: KIVI quantisation, R-KV selection, low-rank projection.

Reference: ``src/cache/kv_compression.rs`` -- ``CompressionPolicy`` (``:89-160``), KIVI
(``:415-566``: asymmetric 2/4-bit quantisation, keys per channel, values per token; its grouped
mode is a ``todo!`` at ``:446``), R-KV (``:570-735``: keep tokens scoring high on importance and
low on redundancy with already kept tokens), LowRank (``:737-1045``; the reference's version
returns random data, ``policies.rs:24-30``) and RelationshipAware.

KIVI here is complete (grouped and ungrouped), works on any device, and keeps the most recent
``residual`` tokens in full precision as KIVI prescribes.  The tier store uses it to shrink
demoted KV; the functions are also usable directly on ``[tokens, heads, head_dim]`` tensors.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch


# ---------------------------------------------------------------------------------------
# bit packing
# ---------------------------------------------------------------------------------------
def _pack(q: torch.Tensor, bits: int) -> torch.Tensor:
    """uint8 values < 2**bits along the last dim -> packed bytes (little end first)."""
    per = 8 // bits
    n = q.shape[-1]
    pad = (-n) % per
    if pad:
        q = torch.nn.functional.pad(q, (0, pad))
    q = q.to(torch.uint8).reshape(*q.shape[:-1], -1, per)
    out = torch.zeros(q.shape[:-1], dtype=torch.uint8, device=q.device)
    for i in range(per):
        out |= q[..., i] << (bits * i)
    return out


def _unpack(p: torch.Tensor, bits: int, n: int) -> torch.Tensor:
    per = 8 // bits
    mask = (1 << bits) - 1
    parts = [(p >> (bits * i)) & mask for i in range(per)]
    return torch.stack(parts, -1).reshape(*p.shape[:-1], -1)[..., :n]


@dataclass
class QuantTensor:
    packed: torch.Tensor      # uint8
    scale: torch.Tensor       # fp16, one per group
    zero: torch.Tensor        # fp16 (minimum of the group)
    bits: int
    shape: tuple
    axis: int                 # 0: groups run along tokens (per-channel), 1: along channels
    group: int = 0            # elements per quantisation group

    def nbytes(self) -> int:
        return (self.packed.numel() + 2 * self.scale.numel() + 2 * self.zero.numel())


def quantize(x: torch.Tensor, bits: int, group: int, per_channel: bool) -> QuantTensor:
    """Asymmetric min/max quantisation of ``x`` [T, H, D].

    per_channel=True (keys): each channel (h, d) is quantised over groups of ``group`` tokens;
    per_channel=False (values): each token is quantised over groups of ``group`` channels."""
    T, H, D = x.shape
    xf = x.float()
    if per_channel:
        g = min(group, T) if group > 0 else T
        pad = (-T) % g
        xp = torch.nn.functional.pad(xf, (0, 0, 0, 0, 0, pad)) if pad else xf
        v = xp.reshape(-1, g, H, D).permute(0, 2, 3, 1)            # [G, H, D, g]
    else:
        g = min(group, H * D) if group > 0 else H * D
        flat = xf.reshape(T, H * D)
        pad = (-(H * D)) % g
        xp = torch.nn.functional.pad(flat, (0, pad)) if pad else flat
        v = xp.reshape(T, -1, g)                                    # [T, G, g]
    lo = v.amin(-1, keepdim=True)
    hi = v.amax(-1, keepdim=True)
    qmax = (1 << bits) - 1
    scale = (hi - lo).clamp_min(1e-8) / qmax
    q = torch.round((v - lo) / scale).clamp(0, qmax)
    return QuantTensor(_pack(q, bits), scale.half(), lo.half(), bits, (T, H, D),
                       0 if per_channel else 1, g)


def dequantize(qt: QuantTensor) -> torch.Tensor:
    T, H, D = qt.shape
    q = _unpack(qt.packed, qt.bits, qt.group).float()
    v = q * qt.scale.float() + qt.zero.float()
    if qt.axis == 0:                                                 # [G, H, D, g]
        return v.permute(0, 3, 1, 2).reshape(-1, H, D)[:T]
    return v.reshape(T, -1)[:, :H * D].reshape(T, H, D)              # [T, G, g]


@dataclass
class KiviBlock:
    k: Optional[QuantTensor]
    v: Optional[QuantTensor]
    k_tail: torch.Tensor        # most recent tokens in full precision
    v_tail: torch.Tensor
    n: int

    def nbytes(self) -> int:
        b = self.k_tail.numel() * self.k_tail.element_size() * 2
        if self.k is not None:
            b += self.k.nbytes() + self.v.nbytes()
        return b


class KiviCompressor:
    """KIVI: keys per channel, values per token, ``bits`` in {2, 4}, full-precision residual of
    the ``residual`` most recent tokens."""

    def __init__(self, bits: int = 4, group: int = 32, residual: int = 32):
        assert bits in (2, 4, 8)
        self.bits, self.group, self.residual = bits, group, residual

    def compress(self, k: torch.Tensor, v: torch.Tensor) -> KiviBlock:
        T = k.shape[0]
        r = min(self.residual, T)
        head = T - r
        if head > 0:
            qk = quantize(k[:head], self.bits, self.group, per_channel=True)
            qv = quantize(v[:head], self.bits, self.group, per_channel=False)
        else:
            qk = qv = None
        return KiviBlock(qk, qv, k[head:].clone(), v[head:].clone(), T)

    def decompress(self, b: KiviBlock, dtype=None):
        dtype = dtype or b.k_tail.dtype
        if b.k is None:
            return b.k_tail.to(dtype), b.v_tail.to(dtype)
        k = torch.cat([dequantize(b.k).to(dtype), b.k_tail.to(dtype)])
        v = torch.cat([dequantize(b.v).to(dtype), b.v_tail.to(dtype)])
        return k, v


# ---------------------------------------------------------------------------------------
# selection policies
# ---------------------------------------------------------------------------------------
def rkv_select(keys: torch.Tensor, importance: torch.Tensor, budget: int, lam: float = 0.5,
               protect_first: int = 0, protect_last: int = 0) -> List[int]:
    """R-KV: greedily keep tokens maximising ``importance - lam * redundancy`` where redundancy is
    the largest cosine similarity (over heads, averaged) of a token's keys with the kept set.
    ``keys`` [T, H, D], ``importance`` [T] (e.g. H2O attention mass).  Returns sorted indices."""
    T = keys.shape[0]
    if budget >= T:
        return list(range(T))
    kn = torch.nn.functional.normalize(keys.float(), dim=-1)            # [T, H, D]
    imp = importance.float().clone()
    if imp.max() > imp.min():
        imp = (imp - imp.min()) / (imp.max() - imp.min())
    kept = list(range(protect_first)) + list(range(max(protect_first, T - protect_last), T))
    kept = sorted(set(kept))
    red = torch.zeros(T)
    taken = torch.zeros(T, dtype=torch.bool)
    for i in kept:
        taken[i] = True
    if kept:
        sims = torch.einsum("thd,khd->tkh", kn, kn[kept]).mean(-1)       # [T, K]
        red = sims.max(1).values
    while len(kept) < budget:
        score = imp - lam * red
        score[taken] = -float("inf")
        j = int(torch.argmax(score))
        kept.append(j)
        taken[j] = True
        s = torch.einsum("thd,hd->th", kn, kn[j]).mean(-1)
        red = torch.maximum(red, s)
    return sorted(kept)


@dataclass
class LowRankBlock:
    u: torch.Tensor      # [H, T, r]
    vt: torch.Tensor     # [H, r, D]
    shape: tuple


def lowrank_compress(x: torch.Tensor, rank: int) -> LowRankBlock:
    """Per-head truncated SVD of ``x`` [T, H, D] (keeps the ``rank`` largest directions)."""
    T, H, D = x.shape
    m = x.float().permute(1, 0, 2)                                      # [H, T, D]
    U, S, Vh = torch.linalg.svd(m, full_matrices=False)
    r = min(rank, S.shape[-1])
    return LowRankBlock(U[..., :r] * S[:, None, :r], Vh[:, :r], (T, H, D))


def lowrank_decompress(b: LowRankBlock) -> torch.Tensor:
    return torch.bmm(b.u, b.vt).permute(1, 0, 2)


def relationship_select(keys: torch.Tensor, importance: torch.Tensor, budget: int,
                        window: int = 8) -> List[int]:
    """RelationshipAware: importance spread to neighbours (tokens next to heavy hitters keep
    their phrase context); top ``budget`` by the smoothed score."""
    T = keys.shape[0]
    if budget >= T:
        return list(range(T))
    imp = importance.float().view(1, 1, -1)
    k = torch.ones(1, 1, 2 * window + 1) / (2 * window + 1)
    sm = torch.nn.functional.conv1d(imp, k, padding=window).view(-1)[:T]
    score = 0.5 * importance.float() + 0.5 * sm
    return sorted(torch.topk(score, budget).indices.tolist())
