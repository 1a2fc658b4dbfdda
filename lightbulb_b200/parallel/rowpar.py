"""Row-parallel exchange for tensor parallelism (``csrc/kernels/tp_rowpar.cu``).

A tensor-parallel transformer layer ends each sub-layer with a row-parallel GEMM (o_proj,
down_proj) whose per-rank partial sums must be added, added to the residual stream and
RMS-normalised before the next column-parallel GEMM.  The reference does this as an all-reduce
through device 0 plus separate add and norm ops (``src/multi_gpu/tensor_parallel.rs:119-133``,
``src/model/custom_transformer_block.rs:304-357``).  Here it is one kernel per sub-layer:

* token rows are owned in contiguous ranges (``ceil(T / world)`` per rank); the residual stream
  is sharded the same way, so each rank keeps only its own rows current;
* the GEMM either pushes its output rows straight into their owners' receive slots
  (:meth:`RowParallelExchange.gemm`, decode-sized batches: the cluster split-K GEMM's epilogue
  does the peer stores) or writes a local partial that the exchange kernel pushes itself
  (:meth:`RowParallelExchange.norm` with ``partial``; any GEMM);
* the owner sums every rank's rows in rank order, adds its residual rows, normalises them and
  pushes the normalised rows to every peer, which copy them into the full ``[T, H]`` input of
  the next GEMM.

Receive slots hold a sentinel until written (the data is its own flag), so no flags or
barriers are exchanged; an epoch word in the buffer header selects one of two slot parities.
"""
from __future__ import annotations

import os
from typing import List, Optional

import torch
import torch.distributed as dist

from .. import ops


def owned_rows(T: int, world: int, rank: int):
    """(first row, row count) of ``rank``'s share of ``T`` token rows."""
    rp = (T + world - 1) // world
    r0 = rank * rp
    return r0, max(0, min(rp, T - r0))


class RowParallelExchange:
    def __init__(self, comm, max_tokens: int, hidden: int, device: torch.device,
                 ctas: int = 0):
        C = ops._need_c()
        self.C, self.comm = C, comm
        self.world, self.rank = comm.world, comm.rank
        self.max_tokens, self.hidden = int(max_tokens), int(hidden)
        self.device = device
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        self.ctas = ctas or sms
        nbytes = C.rowpar_buffer_bytes(self.max_tokens, self.hidden, self.world)
        self.base = C.ipc_alloc(nbytes)
        C.rowpar_prepare(self.base, self.max_tokens, self.hidden, self.world)
        h = C.ipc_export(self.base).to(device)
        allh = torch.empty(self.world * h.numel(), dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(allh, h, group=comm.group)
        allh = allh.view(self.world, -1).cpu()
        self.bases: List[int] = [self.base if r == self.rank else
                                 C.ipc_open(allh[r].contiguous()) for r in range(self.world)]
        torch.cuda.synchronize()
        comm.barrier()
        recv1_off, self.rp_max, _recv2_off, _t_max = C.rowpar_geometry(
            self.max_tokens, self.hidden, self.world)
        self.recv1 = [b + recv1_off for b in self.bases]
        self.epoch_ptr = self.base
        # GEMM-epilogue push for decode-sized batches: off unless LB_ROWPAR_PUSH=1 (measured
        # slower at TP2: the split-K epilogue's per-thread stores cost more than the
        # exchange kernel's own push phase)
        self.push = os.environ.get("LB_ROWPAR_PUSH", "0") == "1"
        self.err = ops.scratch(device).err
        self.ws = ops.scratch(device).gemm_ws
        self.calls = 0

    def fits(self, T: int) -> bool:
        return 1 <= T <= self.max_tokens

    def push_ok(self, T: int, n: int) -> bool:
        """Whether the GEMM epilogue should push (decode-sized batches, where the cluster
        split-K GEMM is the kernel of choice anyway)."""
        return self.push and T <= 512 and n == self.hidden

    def gemm(self, a: torch.Tensor, w: torch.Tensor) -> None:
        """Row-parallel GEMM ``a @ w.T`` whose output rows go straight to their owners."""
        self.C.gemm_bf16_rowpar(a, w, self.err, self.recv1, self.rank, self.rp_max,
                                self.epoch_ptr, self.ws)
        ops.launch_counter_add(1)

    def norm(self, partial: Optional[torch.Tensor], x_own: torch.Tensor, w: torch.Tensor,
             T: int, eps: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``x_own += sum_ranks(partial)[own rows]``; returns ``rmsnorm(x) * w`` for all ``T``
        rows.  ``partial=None``: the rows were pushed by :meth:`gemm`."""
        h = out if out is not None else torch.empty(T, self.hidden, dtype=torch.bfloat16,
                                                    device=x_own.device)
        self.C.rowpar_norm(h, partial, x_own, w, self.bases, self.rank, T, self.max_tokens,
                           float(eps), self.ctas, self.err)
        ops.launch_counter_add(1)
        self.calls += 1
        return h

    def gemm_norm(self, a: torch.Tensor, w: torch.Tensor, x_own: torch.Tensor,
                  norm_w: torch.Tensor, eps: float) -> torch.Tensor:
        """Row-parallel layer + residual + RMSNorm: pushing GEMM when the batch is decode-sized,
        else a local GEMM whose partial the exchange kernel pushes."""
        T = a.shape[0]
        if self.push_ok(T, w.shape[0]):
            self.gemm(a, w)
            return self.norm(None, x_own, norm_w, T, eps)
        return self.norm(ops.gemm(a, w), x_own, norm_w, T, eps)

    def close(self):
        for r, b in enumerate(self.bases):
            if r != self.rank:
                self.C.ipc_close(b)
        self.C.ipc_free(self.base)
        self.bases = []


def selfcheck(argv=None) -> int:
    """``torchrun --nproc-per-node N -m lightbulb_b200.parallel.rowpar``: the exchange against
    an fp32 reference built from NCCL all-gathers, for token counts that do not divide by the
    world size (and fewer tokens than ranks), both GEMM modes (pushing epilogue and local
    partial), calls interleaved so both slot parities are used, a partial lane holding the
    sentinel bit pattern, and a CUDA-graph replay.  Every rank's normalised rows must be
    bitwise identical.  Exit code 0 = pass."""
    from .comm import TPComm, init_distributed
    rank, world, local = init_distributed(timeout_s=60)
    dev = torch.device("cuda", local)
    comm = TPComm()
    H, K = 4096, 512
    X = RowParallelExchange(comm, 640, H, dev)
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    g0 = torch.Generator(device=dev).manual_seed(7)
    bad = []

    def reference(parts, x0, wn, eps):
        y = torch.stack([p.float() for p in parts]).sum(0).to(torch.bfloat16).float()
        xr = (x0.float() + y).to(torch.bfloat16).float()
        return xr, xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + eps) * wn.float()

    cases = [(256, True), (256, False), (1, True), (3, False), (255, True), (640, False),
             (37, True), (512, True), (129, False)]
    for it, (T, push) in enumerate(cases):
        a = (torch.randn(T, K, device=dev, generator=g) * 0.5).to(torch.bfloat16)
        w = (torch.randn(H, K, device=dev, generator=g) * 0.05).to(torch.bfloat16)
        x0 = torch.randn(T, H, device=dev, generator=g0).to(torch.bfloat16)
        wn = (1 + 0.1 * torch.randn(H, device=dev, generator=g0)).to(torch.bfloat16)
        partial = ops.gemm(a, w)
        if it == 3 and rank == 0:
            partial.view(torch.int16)[0, 5] = -1      # 0xFFFF: a NaN with the sentinel's bits
        r0, n = owned_rows(T, world, rank)
        x = x0.clone()
        x_own = x[r0:r0 + n]
        if push and T <= 512:
            X.gemm(a, w)
            h = X.norm(None, x_own, wn, T, 1e-5)
        else:
            h = X.norm(partial, x_own, wn, T, 1e-5)
        parts = [torch.empty_like(partial) for _ in range(world)]
        dist.all_gather(parts, partial)
        xr, hr = reference(parts, x0, wn, 1e-5)
        fin = torch.isfinite(hr).all(-1)
        own = slice(r0, r0 + n)
        if n and (x[own].float() - xr[own]).abs().max().item() > 0.02 * xr.abs().max().item() + 1e-2:
            bad.append((T, push, "residual"))
        if fin.any() and ((h.float()[fin] - hr[fin]).norm() / hr[fin].norm()).item() > 1e-2:
            bad.append((T, push, "norm"))
        if (~fin).any() and not torch.isnan(h.float()[~fin]).any(-1).all():
            bad.append((T, push, "nan row lost"))
        hs = [torch.empty_like(h) for _ in range(world)]
        dist.all_gather(hs, h)
        if not all(torch.equal(hs[0].view(torch.int16), t.view(torch.int16)) for t in hs):
            bad.append((T, push, "ranks differ"))
    # CUDA graph: three exchanges per replay (odd: the parity carried by the epoch word must
    # alternate across replays too), replayed twice
    T = 256
    a = (torch.randn(T, K, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    w = (torch.randn(H, K, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    wn = torch.ones(H, device=dev, dtype=torch.bfloat16)
    r0, n = owned_rows(T, world, rank)
    xg = torch.zeros(T, H, device=dev, dtype=torch.bfloat16)
    hout = torch.empty(T, H, device=dev, dtype=torch.bfloat16)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    torch.cuda.synchronize()
    comm.barrier()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        for _ in range(3):
            X.gemm(a, w)
            X.norm(None, xg[r0:r0 + n], wn, T, 1e-5, out=hout)
    torch.cuda.synchronize()
    comm.barrier()
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    part = ops.gemm(a, w)
    parts = [torch.empty_like(part) for _ in range(world)]
    dist.all_gather(parts, part)
    y = torch.stack([p.float() for p in parts]).sum(0).to(torch.bfloat16).float()
    xr = torch.zeros(T, H, device=dev)
    for _ in range(6):
        xr = (xr + y).to(torch.bfloat16).float()
    if n and (xg[r0:r0 + n].float() - xr[r0:r0 + n]).abs().max().item() > 0.05 * xr.abs().max().item():
        bad.append(("graph", "residual"))
    hr = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-5)
    if ((hout.float() - hr).norm() / hr.norm()).item() > 1e-2:
        bad.append(("graph", "norm"))
    del graph
    ops.check_errors(dev)
    torch.cuda.synchronize()
    if rank == 0:
        print(f"row-parallel exchange world={world}: {'ok' if not bad else bad}", flush=True)
    ok = torch.tensor([int(not bad)], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    torch.cuda.synchronize()
    X.close()
    comm.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0 if int(ok.item()) == 1 else 1


if __name__ == "__main__":
    import sys
    sys.exit(selfcheck())
