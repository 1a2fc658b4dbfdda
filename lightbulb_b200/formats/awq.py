"""AWQ int4 checkpoints: config, unpacking, repacking, random-init creation.

Reference: ``src/loaders/awq.rs:19-250`` (``quantization_config``: bits, group_size,
version gemm/gemv, zero_point, modules_to_not_convert; ``AwqLinear`` = qweight / qzeros /
scales; w = (q - z) * s per group of ``group_size`` input features).

Two on-disk packings are accepted and recognised by shape:

* AutoAWQ "gemm": ``qweight [in, out/8]`` int32, 8 nibbles per int32 along the OUTPUT dim in
  the interleaved order (0, 2, 4, 6, 1, 3, 5, 7); ``qzeros [in/g, out/8]`` packed the same way;
* K-packed (the reference's ``AwqLinear`` shapes): ``qweight [in/8, out]`` int32 with 8
  consecutive input features per int32 (nibble i = feature 8r + i); ``qzeros [in/g, out/8]``.

``scales [in/g, out]`` fp16 in both.  Internally every linear becomes the device layout used
by the int4 GEMM kernel: ``q [out, in/2]`` uint8 (two K-consecutive nibbles per byte, low
nibble first), ``scales [out, in/g]`` and ``zeros [out, in/g]`` (fp16).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)        # nibble slot -> column offset within 8
AWQ_SLOT = [AWQ_ORDER.index(c) for c in range(8)]  # column offset -> nibble slot


@dataclass
class AwqConfig:
    bits: int = 4
    group_size: int = 128
    version: str = "gemm"
    zero_point: bool = True
    modules_to_not_convert: List[str] = field(default_factory=list)

    @classmethod
    def from_config(cls, cfg: dict) -> "AwqConfig":
        q = cfg.get("quantization_config")
        if not q:
            raise KeyError("no quantization_config in config.json")
        if "bits" not in q or "group_size" not in q:
            raise KeyError("quantization_config needs bits and group_size")
        return cls(int(q["bits"]), int(q["group_size"]), q.get("version", "gemm"),
                   bool(q.get("zero_point", True)), list(q.get("modules_to_not_convert") or []))


def unpack_int32_nibbles(x: torch.Tensor) -> torch.Tensor:
    """[..., n] int32 -> [..., n, 8] values 0..15 (slot order)."""
    x = x.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(0, 32, 4, device=x.device)
    return ((x.unsqueeze(-1) >> shifts) & 0xF).to(torch.uint8)


def pack_int32_nibbles(v: torch.Tensor) -> torch.Tensor:
    """[..., n, 8] 0..15 -> [..., n] int32."""
    shifts = torch.arange(0, 32, 4, device=v.device)
    s = (v.to(torch.int64) << shifts).sum(-1)
    s = torch.where(s >= 2**31, s - 2**32, s)
    return s.to(torch.int32)


def awq_unpack(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
               group: int):
    """Any accepted packing -> (q [out, in] uint8, zeros [out, in/g] uint8, scales [out, in/g])."""
    ng, out = scales.shape
    inf = ng * group
    if qweight.shape == (inf, out // 8):          # AutoAWQ gemm: packed along out
        v = unpack_int32_nibbles(qweight)            # [in, out/8, 8] slots
        v = v[..., AWQ_SLOT].reshape(inf, out)       # column order
        q = v.t().contiguous()
    elif qweight.shape == (inf // 8, out):         # packed along in
        v = unpack_int32_nibbles(qweight.t().contiguous())   # [out, in/8, 8]
        q = v.reshape(out, inf)
    else:
        raise ValueError(f"unrecognised AWQ qweight shape {tuple(qweight.shape)}")
    z = unpack_int32_nibbles(qzeros)[..., AWQ_SLOT].reshape(ng, out).t().contiguous()
    return q, z, scales.t().contiguous()


def awq_dequant(q: torch.Tensor, z: torch.Tensor, s: torch.Tensor, group: int) -> torch.Tensor:
    """(q [out, in], zeros [out, in/g], scales [out, in/g]) -> float32 [out, in]."""
    out, inf = q.shape
    qf = q.float().view(out, inf // group, group)
    return ((qf - z.float()[..., None]) * s.float()[..., None]).view(out, inf)


def awq_pack_gemm(q: torch.Tensor, z: torch.Tensor, s: torch.Tensor):
    """Inverse of awq_unpack for the AutoAWQ gemm packing."""
    out, inf = q.shape
    v = q.t().reshape(inf, out // 8, 8)[..., list(AWQ_ORDER)]
    qweight = pack_int32_nibbles(v)
    zz = z.t().reshape(z.shape[1], out // 8, 8)[..., list(AWQ_ORDER)]
    return qweight, pack_int32_nibbles(zz), s.t().contiguous().to(torch.float16)


def random_awq_linear(out_f: int, in_f: int, group: int, gen: torch.Generator,
                      scale_lo: float = 0.001, scale_hi: float = 0.02):
    """Random uint4 weights, fp16 scales ~U[lo, hi], zeros U{0..15}."""
    q = torch.randint(0, 16, (out_f, in_f), generator=gen, dtype=torch.uint8)
    z = torch.randint(0, 16, (out_f, in_f // group), generator=gen, dtype=torch.uint8)
    s = (torch.rand(out_f, in_f // group, generator=gen) * (scale_hi - scale_lo) + scale_lo)
    return q, z, s.to(torch.float16)


def save_awq_checkpoint(path: str, cfg, weights: Dict[str, torch.Tensor], group: int = 128,
                        seed: int = 0) -> None:
    """Write an AutoAWQ-gemm style checkpoint: every q/k/v/o/gate/up/down projection is
    random int4 (the float weights given for them are ignored), the rest as given."""
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    g = torch.Generator().manual_seed(seed)
    out = {}
    for name, t in weights.items():
        if name.endswith("_proj.weight"):
            base = name[:-len(".weight")]
            o, i = t.shape
            q, z, s = random_awq_linear(o, i, group, g)
            qw, qz, sc = awq_pack_gemm(q, z, s)
            out[base + ".qweight"], out[base + ".qzeros"], out[base + ".scales"] = qw, qz, sc
        else:
            out[name] = t.to(torch.float16).contiguous()
    save_file(out, os.path.join(path, "model.safetensors"))
    d = cfg.to_hf_dict()
    d["quantization_config"] = {"quant_method": "awq", "bits": 4, "group_size": group,
                                "version": "gemm", "zero_point": True}
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(d, f, indent=2)
