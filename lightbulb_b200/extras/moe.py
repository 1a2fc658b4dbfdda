"""Mixture-of-experts token routing (host / device tensor math).

Reference: ``src/engine/moe_router.rs:73-455`` -- softmax over expert logits, top-k experts per
token, per-expert capacity ``ceil(tokens * capacity_factor / experts)``; policies TokenDrop
(assignments beyond capacity are dropped, earlier tokens first), ExpandedDrop (capacity + m),
Reroute and Unlimited; per-expert token batches, drop counts, load imbalance statistics.

The assignment order is the reference's (token-major, then rank), but the capacity check is a
vectorised running count per expert, so routing a batch is a handful of tensor ops on whatever
device the logits live on.  Reroute sends a dropped assignment to the best-scoring expert that
still has room and is not already chosen by that token.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch


@dataclass
class RouterConfig:
    num_experts: int
    top_k: int = 2
    capacity_factor: float = 1.25
    policy: str = "token_drop"       # token_drop | expanded_drop | reroute | unlimited
    expansion_factor: int = 0        # expanded_drop: extra slots per expert
    renormalize: bool = True         # combine weights renormalised over the chosen experts


@dataclass
class RoutingResult:
    expert_ids: torch.Tensor         # [T, k] chosen experts (after reroute)
    weights: torch.Tensor            # [T, k] combine weights (0 for dropped)
    dropped: torch.Tensor            # [T, k] bool
    expert_loads: torch.Tensor       # [E] kept assignments per expert
    capacity: int
    aux_loss: float                  # load-balancing loss E * sum_e f_e * P_e

    @property
    def num_dropped(self) -> int:
        return int(self.dropped.sum())

    def expert_batches(self) -> Dict[int, List[int]]:
        out: Dict[int, List[int]] = {}
        t, k = self.expert_ids.shape
        ids = self.expert_ids.tolist()
        dr = self.dropped.tolist()
        for i in range(t):
            for j in range(k):
                if not dr[i][j]:
                    out.setdefault(ids[i][j], []).append(i)
        return out

    def load_imbalance(self) -> float:
        l = self.expert_loads.float()
        return float(l.max() / l.mean().clamp_min(1e-9)) if l.numel() else 0.0


@dataclass
class RouterStats:
    total_tokens: int = 0
    total_dropped: int = 0
    ops: int = 0
    max_imbalance: float = 0.0
    avg_imbalance: float = 0.0
    expert_counts: Optional[torch.Tensor] = None


class MoERouter:
    def __init__(self, cfg: RouterConfig):
        if cfg.capacity_factor <= 0:
            raise ValueError("capacity_factor must be > 0")
        if not 1 <= cfg.top_k <= cfg.num_experts:
            raise ValueError("top_k must be in [1, num_experts]")
        self.cfg = cfg
        self.stats = RouterStats(expert_counts=torch.zeros(cfg.num_experts, dtype=torch.long))

    def capacity(self, num_tokens: int) -> int:
        c = self.cfg
        base = math.ceil(num_tokens * c.capacity_factor / c.num_experts)
        if c.policy == "expanded_drop":
            return base + c.expansion_factor
        if c.policy == "unlimited":
            return num_tokens * c.top_k
        return base

    def route(self, logits: torch.Tensor) -> RoutingResult:
        c = self.cfg
        T, E = logits.shape
        if E != c.num_experts:
            raise ValueError(f"logits [{T}, {E}] for {c.num_experts} experts")
        probs = torch.softmax(logits.float(), dim=-1)
        top_p, top_i = torch.topk(probs, c.top_k, dim=-1)               # [T, k]
        cap = self.capacity(T)
        flat = top_i.reshape(-1)                                         # token-major order
        onehot = torch.nn.functional.one_hot(flat, E)
        pos = (onehot.cumsum(0) * onehot).sum(-1) - 1                    # running count
        dropped = (pos >= cap).reshape(T, c.top_k)
        if c.policy == "unlimited":
            dropped = torch.zeros_like(dropped)
        ids = top_i.clone()
        if c.policy == "reroute" and bool(dropped.any()):
            loads = torch.bincount(top_i[~dropped], minlength=E)
            order = torch.argsort(probs, dim=-1, descending=True)
            for t, j in dropped.nonzero().tolist():
                for e in order[t].tolist():
                    if loads[e] < cap and e not in ids[t].tolist():
                        ids[t, j] = e
                        top_p[t, j] = probs[t, e]
                        loads[e] += 1
                        dropped[t, j] = False
                        break
        w = torch.where(dropped, torch.zeros_like(top_p), top_p)
        if c.renormalize:
            w = w / w.sum(-1, keepdim=True).clamp_min(1e-9)
        loads = torch.bincount(ids[~dropped], minlength=E)
        # Switch-style balance loss on the first choice: fraction routed f_e, mean prob P_e
        f = torch.bincount(top_i[:, 0], minlength=E).float() / max(1, T)
        aux = float(E * (f * probs.mean(0)).sum())
        res = RoutingResult(ids, w, dropped, loads, cap, aux)
        s = self.stats
        s.total_tokens += T
        s.total_dropped += res.num_dropped
        s.ops += 1
        s.expert_counts += loads.cpu()
        imb = res.load_imbalance()
        s.max_imbalance = max(s.max_imbalance, imb)
        s.avg_imbalance += (imb - s.avg_imbalance) / s.ops
        return res


def combine(expert_outputs: Dict[int, torch.Tensor], result: RoutingResult, T: int,
            hidden: int) -> torch.Tensor:
    """Weighted sum of expert outputs back into token order.  ``expert_outputs[e]`` has one row
    per token of ``result.expert_batches()[e]`` (in that order)."""
    out = torch.zeros(T, hidden)
    batches = result.expert_batches()
    for e, toks in batches.items():
        y = expert_outputs[e]
        for row, t in enumerate(toks):
            j = (result.expert_ids[t] == e).nonzero()[0, 0]
            out[t] += result.weights[t, j] * y[row].float()
    return out
