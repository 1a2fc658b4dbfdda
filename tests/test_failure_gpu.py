"""Failure detection on the device without faulting the GPU: a peer that never signals.

The push all-reduce is launched once, as rank 0 of a 2-rank group whose "rank 1" receive
buffer is ordinary memory of this same GPU that nobody writes.  Rank 0's bounded poll for its
peer's slice must give up after the kernel's time budget (about 2 s), record the error code
the host reads, and leave the CUDA context usable.  One launch, one GPU: no kernel waits on
another launch."""
import time

import pytest
import torch

from lightbulb_b200 import ops

pytestmark = pytest.mark.gpu


def test_allreduce_peer_never_signals_reports_timeout():
    C = ops._need_c()
    dev = torch.device("cuda", 0)
    n = 4096 * 8
    nbytes = C.allreduce_buffer_bytes(n, 2)
    bufs = [torch.empty(nbytes, dtype=torch.uint8, device=dev) for _ in range(2)]
    for b in bufs:
        C.allreduce_prepare(b.data_ptr(), n, 2)         # sentinel-filled, epochs zero
    x = torch.randn(n, device=dev).to(torch.bfloat16)
    out = torch.empty_like(x)
    err = ops.scratch(dev).err
    err.zero_()
    t0 = time.perf_counter()
    C.allreduce_p2p(out, x, [b.data_ptr() for b in bufs], 0, n, n, 16, err)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    with pytest.raises(ops.KernelError, match="peer flag wait timed out"):
        ops.check_errors(dev)
    assert 1.0 < waited < 30.0
    # the context is still healthy: an ordinary kernel runs and is correct
    a = torch.randn(64, 256, device=dev).to(torch.bfloat16)
    w = torch.randn(128, 256, device=dev).to(torch.bfloat16)
    ref = a.float() @ w.float().T
    assert ((ops.gemm(a, w).float() - ref).norm() / ref.norm()).item() < 1e-2
    ops.check_errors(dev)
