"""Per-op timing of the tensor-parallel decode hot path (run under torchrun, one GPU per rank).

    torchrun --nproc-per-node N -m lightbulb_b200.parallel.tp_bench [--tokens 256]

For one Llama-3-8B layer shard it times, with CUDA events and the max over ranks:
  nccl : o_proj GEMM -> NCCL all_reduce -> fused add+RMSNorm -> gate_up GEMM
  fused: o_proj GEMM with scatter epilogue -> reduce+residual+RMSNorm+all-gather kernel ->
         gate_up GEMM waiting on the gather flag
and the pieces separately, so each collective's cost and the fused path's roofline fraction
(the slower of compute at peak and bytes over NVLink at the measured 770 GB/s) are visible.
"""
from __future__ import annotations

import argparse
import json
import sys

import torch
import torch.distributed as dist


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=256)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--ffn", type=int, default=14336)
    ap.add_argument("--heads", type=int, default=32)
    a = ap.parse_args(argv)
    from .. import ops
    from .comm import TPComm, init_distributed
    from .fused import enable_fused, ensure_fused
    rank, world, local = init_distributed(timeout_s=60)
    dev = torch.device("cuda", local)
    comm = TPComm()
    enable_fused(comm, max_rows=max(512, a.tokens))
    F = ensure_fused(comm, a.hidden, dev)
    T, H = a.tokens, a.hidden
    R = T // world
    g = torch.Generator(device=dev).manual_seed(rank + 1)
    qd = a.heads * 128 // world
    Wo = (torch.randn(H, qd, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    Wgu = (torch.randn(2 * a.ffn // world, H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    attn = torch.randn(T, qd, device=dev, generator=g).to(torch.bfloat16)
    x = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    lnw = torch.ones(H, device=dev, dtype=torch.bfloat16)

    def timed(fn, iters=a.iters, reps=10):
        """Device time per call: ``reps`` calls captured in one CUDA graph, replayed ``iters``
        times between CUDA events (no host launch overhead), max over ranks."""
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        comm.barrier()
        graph = torch.cuda.CUDAGraph()
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            fn()
        torch.cuda.current_stream().wait_stream(st)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph):
            for _ in range(reps):
                fn()
        torch.cuda.synchronize()
        comm.barrier()
        graph.replay()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            graph.replay()
        e.record()
        torch.cuda.synchronize()
        us = s.elapsed_time(e) / (iters * reps) * 1e3
        del graph
        return comm.max_float(us)

    res = {}
    res["gemm_o_local_us"] = timed(lambda: ops.gemm(attn, Wo))
    o = ops.gemm(attn, Wo)
    res["nccl_allreduce_us"] = timed(lambda: dist.all_reduce(o))
    res["rmsnorm_add_us"] = timed(lambda: ops.rmsnorm(o, lnw, 1e-5, residual=x))
    h = ops.rmsnorm(o, lnw, 1e-5)
    res["gemm_gateup_local_us"] = timed(lambda: ops.gemm(h, Wgu, mode=ops.EPI_SWIGLU))

    def nccl_chain():
        y = ops.gemm(attn, Wo)
        dist.all_reduce(y)
        hh = ops.rmsnorm(y, lnw, 1e-5, residual=x)
        ops.gemm(hh, Wgu, mode=ops.EPI_SWIGLU)

    res["nccl_chain_us"] = timed(nccl_chain)
    # two-shot peer-memory all-reduce (GEMM writes straight into its input)
    ar = comm.enable_p2p_allreduce(T * H, dev)
    xin = ar.input(T, H)
    xin.copy_(o)
    res["p2p_allreduce_us"] = timed(lambda: ar(xin))

    def p2p_chain():
        y = comm.gemm_all_reduce(attn, Wo)
        hh = ops.rmsnorm(y, lnw, 1e-5, residual=x)
        ops.gemm(hh, Wgu, mode=ops.EPI_SWIGLU)

    res["p2p_chain_us"] = timed(p2p_chain)
    xr = x.clone()
    res["p2p_allreduce_rmsnorm_us"] = timed(lambda: ar.allreduce_rmsnorm(o, xr, lnw, 1e-5))

    def p2p_norm_chain():
        hh = comm.gemm_all_reduce_rmsnorm(attn, Wo, xr, lnw, 1e-5)
        ops.gemm(hh, Wgu, mode=ops.EPI_SWIGLU)

    res["p2p_norm_chain_us"] = timed(p2p_norm_chain)
    # row-parallel exchange (default TP path): o_proj and down_proj, pushing GEMM epilogue or
    # local partial, each followed by reduce + residual + RMSNorm + all-gather in one kernel
    X = comm.enable_rowpar(max(512, T), H, dev)
    from .rowpar import owned_rows
    r0, nown = owned_rows(T, world, rank)
    xo = x.clone()[r0:r0 + nown].contiguous()
    hbuf = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    fd = a.ffn // world
    Wd = (torch.randn(H, fd, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    act = torch.randn(T, fd, device=dev, generator=g).to(torch.bfloat16)
    res["rowpar_norm_local_us"] = timed(lambda: X.norm(o, xo, lnw, T, 1e-5, out=hbuf))

    def rp_push(inp, w):
        X.gemm(inp, w)
        X.norm(None, xo, lnw, T, 1e-5, out=hbuf)

    def rp_local(inp, w):
        X.norm(ops.gemm(inp, w), xo, lnw, T, 1e-5, out=hbuf)

    res["rowpar_push_o_us"] = timed(lambda: rp_push(attn, Wo))
    res["rowpar_local_o_us"] = timed(lambda: rp_local(attn, Wo))
    res["rowpar_push_down_us"] = timed(lambda: rp_push(act, Wd))
    res["rowpar_local_down_us"] = timed(lambda: rp_local(act, Wd))
    res["gemm_down_local_us"] = timed(lambda: ops.gemm(act, Wd))

    def rp_chain():
        rp_push(attn, Wo)
        ops.gemm(hbuf, Wgu, mode=ops.EPI_SWIGLU)

    res["rowpar_chain_us"] = timed(rp_chain)

    def rp_layer():
        # one decode layer's comm-relevant chain: o_proj -> exchange -> gate_up -> down ->
        # exchange (local-partial mode, the default)
        rp_local(attn, Wo)
        a2 = ops.gemm(hbuf, Wgu, mode=ops.EPI_SWIGLU)
        X.norm(ops.gemm(a2, Wd), xo, lnw, T, 1e-5, out=hbuf)

    for mode in (1, 2, 0):
        X.C.set_comm_fence_mode(mode)
        res[f"rowpar_norm_local_fence{mode}_us"] = timed(lambda: X.norm(o, xo, lnw, T, 1e-5,
                                                                         out=hbuf))
        res[f"p2p_allreduce_fence{mode}_us"] = timed(lambda: ar(xin))
    X.C.set_comm_fence_mode(1)
    for on in (True, False):
        X.C.set_pdl(on)
        res[f"rowpar_layer_pdl{int(on)}_us"] = timed(rp_layer)
    X.C.set_pdl(True)
    # roofline of GEMM + exchange: the slower of tensor FLOPs at the measured GEMM peak,
    # HBM bytes (weights) at the measured copy bandwidth, and bytes leaving this rank over
    # NVLink (partials to owners + normalised rows to every peer) at 770 GB/s per direction
    from ..utils.microbench import peaks
    hbm, tflops, _src = peaks()
    nvl = 2 * (world - 1) / world * T * H * 2
    for name, k in (("o", qd), ("down", fd)):
        fl = 2 * T * k * H
        roof = max(fl / tflops, H * k * 2 / hbm, nvl / 770e9) * 1e6
        res[f"rowpar_{name}_roofline_us"] = roof
        res[f"rowpar_push_{name}_frac_of_roofline"] = roof / res[f"rowpar_push_{name}_us"]
    # one traced push + exchange (globaltimer ns relative to this rank's GEMM start): GEMM CTA
    # stamps [start, setup, acc ready, published, cluster synced, reduced+stored, done], exchange
    # CTA 0 [start, pushed, own rows done, gathered]
    tr_g = torch.zeros(4096 * 8, dtype=torch.int64, device=dev)
    tr_x = torch.zeros(8, dtype=torch.int64, device=dev)
    torch.cuda.synchronize()
    comm.barrier()
    X.C.gemm_bf16_rowpar(attn, Wo, X.err, X.recv1, rank, X.rp_max, X.epoch_ptr, X.ws, 0,
                         tr_g.data_ptr())
    X.C.rowpar_norm(hbuf, None, xo, lnw, X.bases, rank, T, X.max_tokens, 1e-5, X.ctas, X.err,
                    tr_x.data_ptr())
    torch.cuda.synchronize()
    gg = tr_g.view(-1, 8).cpu()
    used = gg[:, 0] > 0
    g0 = int(gg[used, 0].min())
    xx = tr_x.cpu().tolist()
    rtrace = {"gemm_last_start": int(gg[used, 0].max()) - g0,
              "gemm_acc_ready_max": int(gg[used, 2].max()) - g0,
              "gemm_synced_max": int(gg[used, 4].max()) - g0,
              "gemm_stored_max": int(gg[used, 5].max()) - g0,
              "gemm_done_max": int(gg[used, 6].max()) - g0,
              "x_start": xx[0] - g0, "x_pushed": xx[1] - g0, "x_own_done": xx[2] - g0,
              "x_gathered": xx[3] - g0}
    tall = [None] * world
    dist.all_gather_object(tall, rtrace)
    res["rowpar_trace_ns"] = tall
    o2 = ops.gemm(attn, Wo)               # o itself was all-reduced in place by the timing above
    ref = o2.float().clone()
    dist.all_reduce(ref)
    xin.copy_(o2)
    got = ar(xin).float()
    res["p2p_max_abs_err_vs_nccl"] = float((got - ref).abs().max())
    F.residual[:R].copy_(x[rank * R:(rank + 1) * R])

    def fused_chain():
        F.gemm_scatter(attn, Wo, R)
        F.norm_gather(lnw, R, 1e-5)
        F.gemm_consume(F.gather[:T], Wgu, mode=ops.EPI_SWIGLU)

    res["fused_chain_us"] = timed(fused_chain)
    # one traced chain (globaltimer stamps, ns relative to this rank's GEMM start)
    tr_g = torch.zeros(4096 * 8, dtype=torch.int64, device=dev)
    tr_n = torch.zeros(8, dtype=torch.int64, device=dev)
    torch.cuda.synchronize()
    comm.barrier()
    F.C.gemm_bf16_tp(attn, Wo, F._row_shape, ops.EPI_STORE, F.err, 0, F.rs_peers,
                     F.rs_flag_peers, R, rank, R * H, 0, 0, F.done, tr_g.data_ptr(), ws=F.ws)
    F.C.rs_norm_ag(F.rs_peers[rank], None, F.residual[:R], lnw, F.g_peers, F.g_flag_peers,
                   F.rs_flag, F.done, rank, R, R, 1e-5, True, F.err, tr_n.data_ptr())
    F.gemm_consume(F.gather[:T], Wgu, mode=ops.EPI_SWIGLU)
    torch.cuda.synchronize()
    g = tr_g.view(-1, 8).cpu()
    g0 = int(g[g[:, 0] > 0, 0].min())
    n = tr_n.cpu().tolist()
    trace = {"gemm_acc_ready_max": int(g[g[:, 2] > 0, 2].max()) - g0,
             "gemm_reduced_max": int(g[g[:, 5] > 0, 5].max()) - g0,
             "gemm_signal": int(g[-1, 7]) - g0,
             "norm_start": n[0] - g0, "norm_flag_seen": n[1] - g0, "norm_pushed": n[2] - g0,
             "norm_signal": n[3] - g0}
    res["trace_ns_rank%d" % rank] = trace
    tall = [None] * world
    dist.all_gather_object(tall, trace)
    res["trace_ns_all"] = tall
    ops.check_errors(dev)
    # roofline of the fused o_proj+RS: compute vs NVLink bytes leaving this rank
    flops = 2 * T * qd * H
    nvl = (world - 1) / world * T * H * 2 * 2   # scatter partials out + gathered rows out
    res["fused_roofline_us"] = max(flops / 1.6424e15, nvl / 770e9) * 1e6
    res["tokens"], res["world"] = T, world
    if rank == 0:
        print(json.dumps({k: (round(v, 2) if isinstance(v, float) else v) for k, v in res.items()}))
    F.close()
    comm.close()
    comm.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
