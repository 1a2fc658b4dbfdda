"""Two-shot all-reduce over NVLink peer memory (``csrc/kernels/allreduce.cu``).

For the decode step's partial sums (o_proj and down_proj outputs under tensor parallelism,
[tokens, hidden] bf16, ~2 MB) NCCL's ring all-reduce is latency-bound (~24-36 us on 2-8 B200s).
This kernel pushes each slice of the partial into its owner's receive buffer with peer stores,
the owner reduces it and pushes the result to every peer, all in one launch and with no flags or
fences: receive slots hold a sentinel NaN until written, readers poll the data itself and write
the sentinel back.

The receive buffer is one dedicated ``cudaMalloc`` per rank whose CUDA-IPC handle every peer
opens (the same plumbing as :mod:`.fused`).  Results are identical on every rank (each element is
summed by its owner in rank order, then copied).
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist

from .. import ops


class P2PAllReduce:
    def __init__(self, comm, max_elems: int, device: torch.device, ctas: int = 0):
        C = ops._need_c()
        self.C, self.comm = C, comm
        self.world, self.rank = comm.world, comm.rank
        self.max_elems = int(max_elems)
        # one CTA per SM: enough peer loads in flight to cover NVLink latency
        self.ctas = ctas or min(256, torch.cuda.get_device_properties(device).multi_processor_count)
        nbytes = C.allreduce_buffer_bytes(self.max_elems, self.world)
        self.base = C.ipc_alloc(nbytes)
        C.allreduce_prepare(self.base, self.max_elems, self.world)   # sentinel-filled slots
        h = C.ipc_export(self.base).to(device)
        allh = torch.empty(self.world * h.numel(), dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(allh, h, group=comm.group)
        allh = allh.view(self.world, -1).cpu()
        self.bases: List[int] = [self.base if r == self.rank else
                                 C.ipc_open(allh[r].contiguous()) for r in range(self.world)]
        torch.cuda.synchronize()
        comm.barrier()
        # local staging buffer for the partial (peers never read it: the kernel pushes)
        self._input = torch.empty(self.max_elems, dtype=torch.bfloat16, device=device)
        self.err = ops.scratch(device).err
        self.calls = 0

    def fits(self, n: int) -> bool:
        return n % 8 == 0 and n <= self.max_elems

    def input(self, m: int, n: int) -> torch.Tensor:
        """A persistent [m, n] staging tensor for the partial (any contiguous bf16 works)."""
        return self._input[:m * n].view(m, n)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """Sum of ``x`` (contiguous bf16, numel a multiple of 8) over the ranks."""
        out = torch.empty_like(x)
        self.C.allreduce_p2p(out, x, self.bases, self.rank, x.numel(), self.max_elems, self.ctas,
                             self.err)
        ops.launch_counter_add(1)
        self.calls += 1
        return out

    def allreduce_rmsnorm(self, y: torch.Tensor, residual: torch.Tensor, w: torch.Tensor,
                          eps: float) -> Optional[torch.Tensor]:
        """``residual += allreduce(y)``; returns ``rmsnorm(residual) * w`` in one launch, or
        None when the shape does not fit the receive buffers (the caller then composes)."""
        h = torch.empty_like(y)
        if not self.C.allreduce_rmsnorm_p2p(h, y, residual, w, self.bases, self.rank,
                                            self.max_elems, self.ctas, float(eps), self.err):
            return None
        ops.launch_counter_add(1)
        self.calls += 1
        return h

    def close(self):
        for r, b in enumerate(self.bases):
            if r != self.rank:
                self.C.ipc_close(b)
        self.C.ipc_free(self.base)
        self.bases = []


def selfcheck(argv=None) -> int:
    """``torchrun --nproc-per-node N -m lightbulb_b200.parallel.allreduce``: sums random partials
    of several sizes (both receive parities, sizes that do not divide by the world size, a lane
    holding the sentinel bit pattern) and compares with an fp32 reference; every rank's result
    must be bitwise identical.  Exit code 0 = pass."""
    from .comm import TPComm, init_distributed
    rank, world, local = init_distributed(timeout_s=60)
    dev = torch.device("cuda", local)
    comm = TPComm()
    ar = comm.enable_p2p_allreduce(512 * 4096, dev)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    bad = []
    for it, n in enumerate([8, 8 * 37, 4096, 3 * 4096 + 8 * world + 8, 256 * 4096, 8, 512 * 4096,
                            1000 * 8]):
        x = torch.randn(n, device=dev, generator=g).to(torch.bfloat16)
        if it == 1 and rank == 0:
            x.view(torch.int16)[5] = -1          # 0xFFFF: a NaN with the sentinel's bits
        y = ar(x.clone())
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x)
        ref = torch.stack([p.float() for p in parts]).sum(0)
        ys = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(ys, y)
        if not all(torch.equal(ys[0].view(torch.int16), t.view(torch.int16)) for t in ys):
            bad.append((n, "ranks differ"))
        fin = torch.isfinite(ref)
        err = (y.float()[fin] - ref[fin]).abs().max().item() if fin.any() else 0.0
        tol = 0.01 * ref[fin].abs().max().item() + 1e-2
        if err > tol or bool(torch.isnan(y.float()[~fin]).logical_not().any()):
            bad.append((n, err, tol))
    # fused residual add + RMSNorm, interleaved with plain calls (shared per-CTA epochs)
    for T, H in [(1, 4096), (3, 4096), (256, 4096), (255, 2048), (2, 8192), (129, 4096)]:
        y = (torch.randn(T, H, device=dev, generator=g) * 0.5).to(torch.bfloat16)
        x0 = torch.randn(T, H, device=dev, generator=torch.Generator(device=dev).manual_seed(7))
        x0 = x0.to(torch.bfloat16)
        wn = (1 + 0.1 * torch.randn(H, device=dev,
                                    generator=torch.Generator(device=dev).manual_seed(8)))
        wn = wn.to(torch.bfloat16)
        x = x0.clone()
        h = ar.allreduce_rmsnorm(y, x, wn, 1e-5)
        if h is None:
            bad.append((T, H, "not launched"))
            continue
        ar(y.view(-1).clone())                 # a plain call in between
        parts = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(parts, y)
        ysum = torch.stack([p.float() for p in parts]).sum(0).to(torch.bfloat16).float()
        xr = (x0.float() + ysum).to(torch.bfloat16).float()
        hr = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-5) * wn.float()
        if (x.float() - xr).abs().max().item() > 0.02 * xr.abs().max().item() + 1e-2 or \
                ((h.float() - hr).norm() / hr.norm()).item() > 1e-2:
            bad.append((T, H, "fused mismatch"))
        hs = [torch.empty_like(h) for _ in range(world)]
        dist.all_gather(hs, h)
        if not all(torch.equal(hs[0].view(torch.int16), t.view(torch.int16)) for t in hs):
            bad.append((T, H, "fused ranks differ"))
    ops.check_errors(dev)
    torch.cuda.synchronize()
    if rank == 0:
        print(f"p2p all-reduce world={world}: {'ok' if not bad else bad}", flush=True)
    ok = torch.tensor([int(not bad)], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    comm.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0 if int(ok.item()) == 1 else 1


if __name__ == "__main__":
    import sys
    sys.exit(selfcheck())
