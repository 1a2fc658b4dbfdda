"""Quantized linear weights in the layout of the dequant-fused tcgen05 GEMM.

``QuantWeight`` holds packed integers ``qw`` [N, K*bits/8] and per-group fp16 ``scales`` /
``offsets`` [N, K/group], with ``w = q * scale - offset``.  Packing (chosen so the GPU kernel
converts without int->float instructions):

* 4-bit: each little-endian 32-bit word holds 8 K-consecutive values e0..e7 with
  e(2i) in bits [4i, 4i+4) and e(2i+1) in bits [16+4i, 20+4i);
* 8-bit: one byte per value, stored as q + 128 (q signed).

Converters:

* AWQ (q 0..15, zero z, scale s, group 128):     scale = s, offset = z * s
* GGUF Q8_0 (int8 q, fp16 d per 32):              scale = d, offset = 0
* GGUF Q4_K (super-block 256: d, dmin, 6-bit sc/m per 32, 4-bit q):
                                                  scale = d * sc, offset = dmin * m
Row slicing / concatenation (fused QKV, gate/up interleave, tensor-parallel shards) act on
whole rows, and column shards (row-parallel layers) on whole groups.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch


@dataclass
class QuantWeight:
    qw: torch.Tensor       # [N, K * bits / 8] uint8
    scales: torch.Tensor   # [N, K / group] fp16
    offsets: torch.Tensor  # [N, K / group] fp16
    bits: int
    group: int
    # offsets are integer multiples of the scales (offset = z * s, z in 0..15: AWQ zero points),
    # which lets small batches use the integer-weight kernel (per-group rescale after the MMA)
    int_zero: bool = False

    @property
    def shape(self):
        return (self.qw.shape[0], self.qw.shape[1] * 8 // self.bits)

    @property
    def device(self):
        return self.qw.device

    def to(self, device=None, dtype=None) -> "QuantWeight":
        return QuantWeight(self.qw.to(device), self.scales.to(device), self.offsets.to(device),
                           self.bits, self.group, self.int_zero)

    def contiguous(self) -> "QuantWeight":
        return QuantWeight(self.qw.contiguous(), self.scales.contiguous(),
                           self.offsets.contiguous(), self.bits, self.group, self.int_zero)

    def rows(self, idx) -> "QuantWeight":
        return QuantWeight(self.qw[idx], self.scales[idx], self.offsets[idx], self.bits,
                           self.group, self.int_zero)

    def cols(self, k0: int, k1: int) -> "QuantWeight":
        assert k0 % self.group == 0 and k1 % self.group == 0 and k0 % 64 == 0
        b = self.bits
        return QuantWeight(self.qw[:, k0 * b // 8:k1 * b // 8],
                           self.scales[:, k0 // self.group:k1 // self.group],
                           self.offsets[:, k0 // self.group:k1 // self.group], b, self.group,
                           self.int_zero)

    def pad_head_rows(self, n_heads: int, d: int, dp: int) -> "QuantWeight":
        """Insert all-zero rows (q = 0, scale = offset = 0 -> w = 0) after each head's d rows."""
        if d == dp:
            return self

        def pad(t):
            out = torch.zeros((n_heads, dp) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
            out[:, :d] = t.reshape((n_heads, d) + tuple(t.shape[1:]))
            return out.reshape((n_heads * dp,) + tuple(t.shape[1:]))
        return QuantWeight(pad(self.qw), pad(self.scales), pad(self.offsets), self.bits,
                           self.group, self.int_zero)

    def unpack(self) -> torch.Tensor:
        """Integer values [N, K] (int16)."""
        if self.bits == 4:
            return unpack4(self.qw)
        return self.qw.to(torch.int16) - 128

    def dequantize(self, dtype=torch.float32) -> torch.Tensor:
        q = self.unpack().float()
        n, k = q.shape
        s = self.scales.float().repeat_interleave(self.group, 1)
        o = self.offsets.float().repeat_interleave(self.group, 1)
        return (q * s - o).to(dtype)


def pack4(q: torch.Tensor) -> torch.Tensor:
    """[N, K] values 0..15 -> [N, K/2] uint8 in the kernel's word layout."""
    n, k = q.shape
    e = q.to(torch.int64).view(n, k // 8, 8)
    word = torch.zeros(n, k // 8, dtype=torch.int64)
    for i in range(4):
        word |= e[:, :, 2 * i] << (4 * i)
        word |= e[:, :, 2 * i + 1] << (16 + 4 * i)
    b = torch.stack([(word >> (8 * j)) & 0xFF for j in range(4)], -1)
    return b.to(torch.uint8).reshape(n, k // 2).contiguous()


def unpack4(qw: torch.Tensor) -> torch.Tensor:
    n, kb = qw.shape
    b = qw.to(torch.int64).view(n, kb // 4, 4)
    word = b[..., 0] | (b[..., 1] << 8) | (b[..., 2] << 16) | (b[..., 3] << 24)
    out = torch.empty(n, kb // 4, 8, dtype=torch.int16)
    for i in range(4):
        out[..., 2 * i] = ((word >> (4 * i)) & 0xF).to(torch.int16)
        out[..., 2 * i + 1] = ((word >> (16 + 4 * i)) & 0xF).to(torch.int16)
    return out.reshape(n, kb * 2)


def cat_rows(ws) -> QuantWeight:
    b, g = ws[0].bits, ws[0].group
    assert all(w.bits == b and w.group == g for w in ws)
    return QuantWeight(torch.cat([w.qw for w in ws]), torch.cat([w.scales for w in ws]),
                       torch.cat([w.offsets for w in ws]), b, g, all(w.int_zero for w in ws))


def interleave_rows(gate: QuantWeight, up: QuantWeight, group_rows: int = 64) -> QuantWeight:
    f = gate.qw.shape[0]
    idx = torch.arange(2 * f).view(-1, 2, group_rows)
    order = torch.empty(2 * f, dtype=torch.long)
    both = torch.cat([torch.arange(f), torch.arange(f) + f])
    gg = both[:f].view(-1, group_rows)
    uu = both[f:].view(-1, group_rows)
    order = torch.stack([gg, uu], 1).reshape(-1)
    cat = cat_rows([gate, up])
    return cat.rows(order)


def from_awq(q: torch.Tensor, z: torch.Tensor, s: torch.Tensor, group: int) -> QuantWeight:
    """q [N, K] 0..15, z [N, K/g] 0..15, s [N, K/g]."""
    qw = pack4(q)
    sf = s.float()
    return QuantWeight(qw, sf.to(torch.float16), (z.float() * sf).to(torch.float16), 4, group,
                       int_zero=True)


def from_q8_0(raw: np.ndarray, n: int, k: int) -> QuantWeight:
    blk = raw.reshape(n, k // 32, 34)
    d = blk[:, :, 0:2].copy().view(np.float16).reshape(n, k // 32)
    qs = (blk[:, :, 2:].reshape(n, k).view(np.int8).astype(np.int16) + 128).astype(np.uint8)
    return QuantWeight(torch.from_numpy(qs).contiguous(),
                       torch.from_numpy(d.astype(np.float16)),
                       torch.zeros(n, k // 32, dtype=torch.float16), 8, 32)


def _scale_min_k4(sc12: np.ndarray):
    """[..., 12] packed -> (sc [..., 8], m [..., 8]) 6-bit values (the Q4_K packing)."""
    q = sc12.astype(np.int32)
    sc = np.empty(q.shape[:-1] + (8,), np.int32)
    mn = np.empty_like(sc)
    for j in range(4):
        sc[..., j] = q[..., j] & 63
        mn[..., j] = q[..., j + 4] & 63
        sc[..., j + 4] = (q[..., j + 8] & 0xF) | ((q[..., j] >> 6) << 4)
        mn[..., j + 4] = (q[..., j + 8] >> 4) | ((q[..., j + 4] >> 6) << 4)
    return sc, mn


def from_q4_k(raw: np.ndarray, n: int, k: int) -> QuantWeight:
    nb = k // 256
    blk = raw.reshape(n, nb, 144)
    d = blk[:, :, 0:2].copy().view(np.float16).astype(np.float32).reshape(n, nb)
    dmin = blk[:, :, 2:4].copy().view(np.float16).astype(np.float32).reshape(n, nb)
    sc, mn = _scale_min_k4(blk[:, :, 4:16])                    # [n, nb, 8]
    qs = blk[:, :, 16:].reshape(n, nb, 4, 32)                  # pairs of sub-blocks
    lo = qs & 0xF
    hi = qs >> 4
    vals = np.stack([lo, hi], axis=3).reshape(n, nb, 8, 32)    # sub-block order
    vals = vals.reshape(n, k).astype(np.uint8)
    qw = pack4(torch.from_numpy(vals))
    scale = (d[:, :, None] * sc).reshape(n, nb * 8)
    off = (dmin[:, :, None] * mn).reshape(n, nb * 8)
    return QuantWeight(qw.contiguous(), torch.from_numpy(scale.astype(np.float16)),
                       torch.from_numpy(off.astype(np.float16)), 4, 32)
