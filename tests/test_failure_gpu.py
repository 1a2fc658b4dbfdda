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


@pytest.mark.parametrize("decode", [True, False])
@pytest.mark.parametrize("bad", [10_000, -7])
def test_corrupt_block_table_is_reported_not_faulted(decode, bad):
    # an out-of-range block id (a corrupted table) is caught in software before any load is
    # issued: both kernels report it through the error word, read nothing outside the KV pool
    # (the TMA-fed decode kernel never receives the bad coordinate) and leave the context usable
    from test_kernels_gpu import _paged_setup, _rel, _ref_paged
    from lightbulb_b200.models.llama import prefill_tiles
    dev = torch.device("cuda", 0)
    seq_lens = [40, 300, 17]
    q_lens = [1, 1, 1] if decode else [40, 20, 17]
    q, kc, vc, bt, sl, cu = _paged_setup(seq_lens, q_lens, 8, 2, seed=5)
    bt_bad = bt.clone()
    bt_bad[1, 3] = bad                               # sequence 1, its 4th block
    kw = {}
    if not decode:
        ts, tr = prefill_tiles(cu.tolist(), 0, 4)
        kw = dict(tile_seq=torch.tensor(ts, dtype=torch.int32, device=dev),
                  tile_row0=torch.tensor(tr, dtype=torch.int32, device=dev))
    out = torch.empty(q.shape, dtype=torch.bfloat16, device=dev)
    ops.scratch(dev).err.zero_()
    ops.paged_attention(q.to(dev), kc.to(dev), vc.to(dev), bt_bad.to(dev), sl.to(dev),
                        cu.to(dev), out, 4, decode=decode, **kw)
    torch.cuda.synchronize()
    with pytest.raises(ops.KernelError, match="index out of bounds"):
        ops.check_errors(dev)
    # the untouched sequences are still exact, and a clean call reports nothing
    ref = _ref_paged(q, kc, vc, bt, sl, cu)
    r0 = slice(int(cu[0]), int(cu[1]))
    assert _rel(out[r0].cpu(), ref[r0]) < 2e-2
    ops.paged_attention(q.to(dev), kc.to(dev), vc.to(dev), bt.to(dev), sl.to(dev), cu.to(dev),
                        out, 4, decode=decode, **kw)
    torch.cuda.synchronize()
    ops.check_errors(dev)
    assert _rel(out.cpu(), ref) < 2e-2
