"""Fused tensor-parallel decode path over NVLink peer memory.

One symmetric buffer per rank (dedicated cudaMalloc, CUDA IPC handle exchanged over the
process group, opened by every peer):

    [ flags (4 KiB) | reduce-scatter slots [world][R][H] bf16 | gather rows [world*R][H] bf16 ]

flags[0] = reduce-scatter arrivals, flags[1] = gather arrivals, flags[2] = local
grid-completion counter.  Per transformer layer (T tokens, R = T / world rows per rank):

  1. QKV GEMM reads the gathered normed rows (TMA, local memory) after a bounded wait on
     flags[1] >= world; last CTA resets it;
  2. attention (local heads);
  3. o_proj GEMM scatters each output row to its owner's slot for this rank (P2P stores in the
     epilogue) and raises flags[0] of every owner;
  4. rs_norm_ag: owner sums the world slots (+ residual), RMSNorm, stores the normed row into
     every rank's gather buffer, raises flags[1] everywhere;
  5. gate_up (SwiGLU epilogue) consumes the gather, down_proj scatters, rs_norm_ag again.

The residual stream is token-sharded (each rank keeps R rows).  Used for decode steps whose
token count is a multiple of world; other steps use the NCCL path.
"""
from __future__ import annotations

import math
from typing import List

import torch
import torch.distributed as dist

from .. import ops

FLAG_BYTES = 4096


class _DevView:
    """A raw device pointer as a torch tensor (``__cuda_array_interface__``)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape),
                                         "typestr": typestr, "version": 3}


def _view(ptr: int, shape, dtype: torch.dtype) -> torch.Tensor:
    ts = {torch.bfloat16: "<f2", torch.int32: "<i4"}[dtype]  # bf16 viewed through 2-byte type
    t = torch.as_tensor(_DevView(ptr, shape, ts), device="cuda")
    return t.view(dtype) if dtype == torch.bfloat16 else t


class FusedTP:
    def __init__(self, comm, hidden: int, max_rows: int, device: torch.device):
        C = ops._need_c()
        self.C = C
        self.comm = comm
        self.world, self.rank = comm.world, comm.rank
        self.H = hidden
        self.R_max = max(1, math.ceil(max_rows / self.world))
        self.rs_bytes = self.world * self.R_max * hidden * 2
        self.g_bytes = self.world * self.R_max * hidden * 2
        total = FLAG_BYTES + self.rs_bytes + self.g_bytes
        self.base = C.ipc_alloc(total)
        h = C.ipc_export(self.base).to(device)
        allh = torch.empty(self.world * h.numel(), dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(allh, h, group=comm.group)
        allh = allh.view(self.world, -1).cpu()
        self.peer_base: List[int] = []
        for r in range(self.world):
            self.peer_base.append(self.base if r == self.rank else C.ipc_open(allh[r].contiguous()))
        torch.cuda.synchronize()
        comm.barrier()
        self.rs_peers = [b + FLAG_BYTES for b in self.peer_base]
        self.g_peers = [b + FLAG_BYTES + self.rs_bytes for b in self.peer_base]
        self.rs_flag_peers = [b + 0 for b in self.peer_base]
        self.g_flag_peers = [b + 4 for b in self.peer_base]
        self.rs_flag = self.base
        self.g_flag = self.base + 4
        self.done = self.base + 8
        self.gather = _view(self.g_peers[self.rank], (self.world * self.R_max, hidden),
                            torch.bfloat16)
        self.residual = torch.empty(self.R_max, hidden, dtype=torch.bfloat16, device=device)
        # shape/stride carrier for scatter GEMMs (row stride H; the data goes to peers)
        self._row_shape = torch.empty(1, hidden, dtype=torch.bfloat16, device=device)
        self.err = ops.scratch(device).err
        self.ws = ops.scratch(device).gemm_ws  # cluster split-K exchange

    # ------------------------------------------------------------------------------
    def gemm_consume(self, a: torch.Tensor, w: torch.Tensor, mode: int = ops.EPI_STORE):
        """GEMM whose input rows arrive from every rank (waits on the gather flag)."""
        m, n = a.shape[0], w.shape[0]
        if mode == ops.EPI_SWIGLU:
            out = torch.empty(m, n // 2, dtype=torch.bfloat16, device=a.device)
        elif mode == ops.EPI_F32:
            out = torch.empty(m, n, dtype=torch.float32, device=a.device)
        else:
            out = torch.empty(m, n, dtype=torch.bfloat16, device=a.device)
        self.C.gemm_bf16_tp(a, w, out, mode, self.err, 0, [], [], 0, self.rank, 0,
                            self.g_flag, self.world, self.done, ws=self.ws)
        ops.launch_counter_add(1)
        return out

    def gemm_scatter(self, a: torch.Tensor, w: torch.Tensor, R: int):
        """Row-parallel GEMM whose output rows go straight to their owners (P2P)."""
        assert w.shape[0] == self.H
        self.C.gemm_bf16_tp(a, w, self._row_shape, ops.EPI_STORE, self.err, 0, self.rs_peers,
                            self.rs_flag_peers, R, self.rank, R * self.H, 0, 0, self.done,
                            ws=self.ws)
        ops.launch_counter_add(1)

    def norm_gather(self, w: torch.Tensor, R: int, eps: float, x_in=None,
                    add_residual: bool = True):
        res = self.residual[:R]
        self.C.rs_norm_ag(self.rs_peers[self.rank], x_in, res, w, self.g_peers,
                          self.g_flag_peers, self.rs_flag, self.done, self.rank, R, R, eps,
                          add_residual, self.err)
        ops.launch_counter_add(1)

    def close(self):
        for r, b in enumerate(self.peer_base):
            if r != self.rank:
                try:
                    self.C.ipc_close(b)
                except Exception:
                    pass
        try:
            self.C.ipc_free(self.base)
        except Exception:
            pass


def enable_fused(comm, hidden: int = 0, max_rows: int = 512):
    """Mark the communicator for the fused path; buffers are created by the model once the
    hidden size is known (``LlamaModel`` calls :func:`ensure_fused`)."""
    comm.fused_requested = True
    comm.fused_max_rows = max_rows
    return comm


def ensure_fused(comm, hidden: int, device) -> "FusedTP":
    if getattr(comm, "fused", None) is None:
        comm.fused = FusedTP(comm, hidden, getattr(comm, "fused_max_rows", 512), device)
    return comm.fused
