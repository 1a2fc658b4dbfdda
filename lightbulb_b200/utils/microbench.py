"""Per-op device microbenchmarks of the decode step (CUDA events, warm-up, L2-sized inputs).

    python -m lightbulb_b200.utils.microbench decode --batch 256 --ctx 1200 [--tp 1]
    python -m lightbulb_b200.utils.microbench gemm --m 256 --n 4096 --k 4096
    python -m lightbulb_b200.utils.microbench prefill --batch 4 --chunk 512 --ctx 4096
    python -m lightbulb_b200.utils.microbench small_ops --batch 256
    python -m lightbulb_b200.utils.microbench kv_ops --batch 16 --ctx 4096

Reports time, achieved bytes/s or FLOP/s and the fraction of the measured roofline
(``MEASURED_PEAKS.json`` when present: copy bandwidth and cuBLAS bf16 throughput).
Weights are distinct per repetition set and larger than L2 so weight streaming is from HBM.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

import torch

from .. import ops


def peaks():
    p = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d["hbm_gbs"] * 1e9, d["bf16_tflops"] * 1e12, "measured"
    except Exception:
        return 6.65e12, 1.59e15, "fallback"


def time_fn(fn, iters=20, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters * 1e3  # us


def time_graph(fn, calls: int, replays: int = 10) -> float:
    """Device time per call with host launch cost removed: ``calls`` invocations of ``fn``
    (each may use different, L2-busting operands) captured in one CUDA graph, replayed
    between CUDA events."""
    for _ in range(3):
        fn()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        fn()
    torch.cuda.current_stream().wait_stream(st)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(calls):
            fn()
    g.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(replays):
        g.replay()
    e.record()
    torch.cuda.synchronize()
    del g
    return s.elapsed_time(e) / (calls * replays) * 1e3


def bench_gemm(m, n, k, copies=None, mode=ops.EPI_STORE, bt=0, splits=0, iters=20):
    bw, fl, src = peaks()
    wbytes = n * k * 2
    copies = copies or max(1, math.ceil(512e6 / wbytes))  # > L2 worth of distinct weights
    ws = [torch.randn(n, k, device="cuda").to(torch.bfloat16) * 0.02 for _ in range(copies)]
    a = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    it = [0]

    def run():
        ops.gemm(a, ws[it[0] % copies], mode=mode, bt=bt, splits=splits)
        it[0] += 1

    us = time_graph(run, calls=max(copies, iters))
    it[0] = 0

    def run_cublas():
        torch.matmul(a, ws[it[0] % copies].T)
        it[0] += 1

    us_cublas = time_graph(run_cublas, calls=max(copies, iters))
    us_pair = None
    if m > 64:
        it[0] = 0

        def run_pair():
            ops.gemm_pair(a, ws[it[0] % copies], mode=mode)
            it[0] += 1

        us_pair = round(time_graph(run_pair, calls=max(copies, iters)), 2)
    flops = 2 * m * n * k
    byts = wbytes + m * k * 2 + m * n * (4 if mode == ops.EPI_F32 else 2)
    t_roof = max(flops / fl, byts / bw) * 1e6
    plan = ops.gemm_plan(m, n, k, bt, splits)
    return {"op": "gemm", "m": m, "n": n, "k": k, "us": round(us, 2),
            "tflops": round(flops / us / 1e6, 1), "gbs": round(byts / us / 1e3, 1),
            "roofline_us": round(t_roof, 2), "frac_of_" + src: round(t_roof / us, 3),
            "plan_bt_splits": plan[:2], "cublas_us": round(us_cublas, 2),
            "pair_us": us_pair}


def bench_gemm_quant(m, n, k, kind="awq", iters=20):
    """Dequant-fused GEMM on random quantized weights (> L2 of distinct copies)."""
    from ..formats.quant import QuantWeight
    bw, fl, src = peaks()
    bits, group = (8, 32) if kind == "q80" else (4, 128 if kind == "awq" else 32)
    wbytes = n * k * bits // 8 + 2 * 2 * n * (k // group)
    copies = max(1, math.ceil(512e6 / wbytes))
    ws = []
    for _ in range(copies):
        qw = torch.randint(0, 256, (n, k * bits // 8), device="cuda", dtype=torch.int32)
        sc = torch.rand(n, k // group, device="cuda").half() * 0.01
        ws.append(QuantWeight(qw.to(torch.uint8), sc, sc * 8, bits, group,
                              int_zero=kind == "awq"))
    a = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    it = [0]

    def run():
        ops.gemm(a, ws[it[0] % copies])
        it[0] += 1

    us = time_graph(run, calls=max(copies, iters))
    byts = wbytes + m * k * 2 + m * n * 2
    t_roof = max(2 * m * n * k / fl, byts / bw) * 1e6
    return {"op": f"gemm_{kind}", "m": m, "n": n, "k": k, "us": round(us, 2),
            "weight_bytes": wbytes, "gbs": round(byts / us / 1e3, 1),
            "roofline_us": round(t_roof, 2), "frac_of_" + src: round(t_roof / us, 3)}


def trace_gemm(m, n, k, bt=0, splits=0):
    """Per-CTA phase times (us) of one cluster split-K GEMM launch (globaltimer stamps)."""
    from .. import _C
    w = torch.randn(n, k, device="cuda").to(torch.bfloat16) * 0.02
    a = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    s = ops.scratch(a.device)
    tr = torch.zeros(4096 * 8, dtype=torch.int64, device="cuda")
    # warm the clocks first (a second of dense GEMMs), then three traced launches
    x = torch.randn(8192, 8192, device="cuda", dtype=torch.bfloat16)
    t_end = __import__("time").time() + 1.0
    while __import__("time").time() < t_end:
        x @ x
    for _ in range(3):
        _C.gemm_bf16(a, w, out, None, 0, s.gemm_ws, s.gemm_counters, s.err, bt, splits, tr)
    torch.cuda.synchronize()
    plan = ops.gemm_plan(m, n, k, bt, splits)
    grid = plan[2] * abs(plan[1])
    t_all = tr.view(-1, 8).cpu()
    t = t_all[:grid].double()
    t0 = t[:, 0].min()
    names = ["start", "prologue", "acc_ready", "published", "synced", "reduced_stored",
             "exit"]
    # second row (thread 0 of the epilogue): inside publish / reduce / store
    names2 = ["tmem_to_smem", "bar", "bulk_issued", "bulk_done", "fetched", "reduced",
              "tma_issue", "tma_done"]
    res = {"op": "gemm_trace", "m": m, "n": n, "k": k, "ctas": grid}
    t2 = t_all[grid:2 * grid].double()
    for tab, nms in ((t, names), (t2, names2)):
        for i, nm in enumerate(nms):
            col = tab[:, i]
            ok = col > 0
            if ok.any():
                res[nm + "_us"] = round(float((col[ok] - t0).mean()) / 1e3, 2)
    return res


def bench_decode_attn(batch, ctx, hq, hkv, bs=16, splits=None, iters=20):
    bw, fl, src = peaks()
    d = 128
    nb_per = (ctx + bs - 1) // bs
    nblocks = batch * nb_per + 8
    kc = torch.empty(nblocks, hkv, bs, d, device="cuda", dtype=torch.bfloat16).normal_()
    vc = torch.empty_like(kc).normal_()
    bt = torch.randperm(nblocks, device="cuda")[:batch * nb_per].view(batch, nb_per).int()
    sl = torch.full((batch,), ctx, dtype=torch.int32, device="cuda")
    cu = torch.arange(batch + 1, dtype=torch.int32, device="cuda")
    q = torch.randn(batch, hq, d, device="cuda").to(torch.bfloat16)
    out = torch.empty_like(q)
    sp = splits if splits is not None else ops.decode_splits(batch, hkv, ctx)

    def run():
        ops.paged_attention(q, kc, vc, bt, sl, cu, out, hq // hkv, decode=True, num_splits=sp)

    us = time_graph(run, calls=iters)
    byts = batch * ctx * hkv * d * 2 * 2
    return {"op": "attn_decode", "batch": batch, "ctx": ctx, "hq": hq, "hkv": hkv, "splits": sp,
            "us": round(us, 2), "gbs": round(byts / us / 1e3, 1),
            "frac_of_" + src: round(byts / bw * 1e6 / us, 3)}


def bench_prefill_attn(batch, chunk, ctx, hq, hkv, bs=16, iters=10):
    """Chunked-prefill attention: ``batch`` sequences, each a chunk of ``chunk`` new query
    tokens at the end of a ``ctx``-token paged context (causal)."""
    from ..models.llama import prefill_tiles
    bw, fl, src = peaks()
    d = 128
    nb_per = (ctx + bs - 1) // bs
    nblocks = batch * nb_per + 8
    kc = torch.empty(nblocks, hkv, bs, d, device="cuda", dtype=torch.bfloat16).normal_()
    vc = torch.empty_like(kc).normal_()
    bt = torch.randperm(nblocks, device="cuda")[:batch * nb_per].view(batch, nb_per).int()
    sl = torch.full((batch,), ctx, dtype=torch.int32, device="cuda")
    cu = [i * chunk for i in range(batch + 1)]
    q = torch.randn(batch * chunk, hq, d, device="cuda").to(torch.bfloat16)
    out = torch.empty_like(q)
    ts, tr = prefill_tiles(cu, 0, hq // hkv)
    tile_seq = torch.tensor(ts, dtype=torch.int32, device="cuda")
    tile_row0 = torch.tensor(tr, dtype=torch.int32, device="cuda")
    cu_t = torch.tensor(cu, dtype=torch.int32, device="cuda")
    sl_cpu, cu_cpu = sl.cpu(), torch.tensor(cu, dtype=torch.int32)

    def run():
        ops.paged_attention(q, kc, vc, bt, sl, cu_t, out, hq // hkv, decode=False,
                            tile_seq=tile_seq, tile_row0=tile_row0,
                            seq_lens_cpu=sl_cpu, cu_q_cpu=cu_cpu)

    us = time_graph(run, calls=iters)
    pairs = sum(ctx - chunk + i + 1 for i in range(chunk)) * batch   # causal (q, k) pairs
    flops = 4 * pairs * hq * d
    byts = batch * ctx * hkv * d * 2 * 2 + 2 * q.numel() * 2
    t_roof = max(flops / fl, byts / bw) * 1e6
    return {"op": "attn_prefill", "batch": batch, "chunk": chunk, "ctx": ctx, "hq": hq,
            "hkv": hkv, "us": round(us, 2), "tflops": round(flops / us / 1e6, 1),
            "roofline_us": round(t_roof, 2), "frac_of_" + src: round(t_roof / us, 3)}


def bench_small_ops(batch, model="llama3-8b"):
    """Elementwise / sampling kernels of one decode step at ``batch`` tokens."""
    from ..config import get_preset
    bw, fl, src = peaks()
    cfg = get_preset(model)
    h, d = cfg.hidden_size, 128
    hq, hkv = cfg.num_heads, cfg.num_kv_heads
    rows = []
    x = torch.randn(batch, h, device="cuda").to(torch.bfloat16)
    r = torch.randn(batch, h, device="cuda").to(torch.bfloat16)
    w = torch.ones(h, device="cuda", dtype=torch.bfloat16)
    us = time_graph(lambda: ops.rmsnorm(x, w, 1e-5, residual=r), 50)
    rows.append({"op": "rmsnorm_add", "us": round(us, 2),
                 "frac_of_" + src: round(batch * h * 2 * 4 / bw * 1e6 / us, 3)})
    emb = torch.randn(cfg.vocab_size, h, device="cuda").to(torch.bfloat16)
    ids = torch.randint(0, cfg.vocab_size, (batch,), device="cuda", dtype=torch.int32)
    us = time_graph(lambda: ops.embedding(ids, emb), 50)
    rows.append({"op": "embedding", "us": round(us, 2)})
    qkv = torch.randn(batch, (hq + 2 * hkv) * d, device="cuda").to(torch.bfloat16)
    pos = torch.randint(0, 4000, (batch,), dtype=torch.int32, device="cuda")
    slots = torch.randperm(batch * 16, device="cuda")[:batch].int()
    cs = ops.rope_table(4096, d, cfg.rope_theta, "cuda")
    kc = torch.zeros(batch, hkv, 16, d, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    us = time_graph(lambda: ops.rope_kv(qkv, pos, slots, cs, kc, vc, hq, hkv), 50)
    rows.append({"op": "rope_kv", "us": round(us, 2)})
    logits = torch.randn(batch, cfg.vocab_size, device="cuda")
    t = torch.full((batch,), 0.8, device="cuda")
    tk = torch.full((batch,), 50, dtype=torch.int32, device="cuda")
    tp = torch.full((batch,), 0.9, device="cuda")
    seeds = torch.arange(batch, dtype=torch.int64, device="cuda")
    us = time_graph(lambda: ops.sample(logits, t, tk, tp, seeds), 20)
    rows.append({"op": "sample_topk_topp", "us": round(us, 2),
                 "frac_of_" + src: round(logits.numel() * 4 / bw * 1e6 / us, 3)})
    z = torch.zeros(batch, device="cuda")
    zi = torch.zeros(batch, dtype=torch.int32, device="cuda")
    us = time_graph(lambda: ops.sample(logits, z, zi, z + 1, seeds), 20)
    rows.append({"op": "sample_greedy", "us": round(us, 2),
                 "frac_of_" + src: round(logits.numel() * 4 / bw * 1e6 / us, 3)})
    return rows


def bench_kv_ops(batch, ctx, hq=32, hkv=8, layers=32, bs=16):
    """H2O attention-mass accumulation (last layer) and KV compaction of ``ctx`` tokens."""
    from .. import _C
    bw, fl, src = peaks()
    d = 128
    nb_per = (ctx + bs - 1) // bs
    nblocks = batch * nb_per + 8
    kc = torch.empty(nblocks, hkv, bs, d, device="cuda", dtype=torch.bfloat16).normal_()
    bt = torch.randperm(nblocks, device="cuda")[:batch * nb_per].view(batch, nb_per).int()
    sl = torch.full((batch,), ctx, dtype=torch.int32, device="cuda")
    q = torch.randn(batch, hq, d, device="cuda").to(torch.bfloat16)
    score = torch.zeros(nblocks * bs, device="cuda")
    wl = torch.empty(batch, hq, nb_per * bs, device="cuda")
    wp = torch.empty(batch, hq, (nb_per * bs + 255) // 256, 2, device="cuda")
    us = time_graph(lambda: _C.h2o_accumulate(q, kc, bt, sl, score, 0.95, d ** -0.5, wl, wp), 10)
    rows = [{"op": "h2o_accumulate", "batch": batch, "ctx": ctx, "us": round(us, 2),
             "gbs": round(batch * ctx * hkv * d * 2 * 2 / us / 1e3, 1)}]
    storage = torch.zeros(layers, 2, nblocks, hkv, bs, d, device="cuda", dtype=torch.bfloat16)
    n = batch * (ctx // 2)
    src_s = torch.randperm(nblocks * bs, device="cuda")[:n].int()
    dst_s = torch.randperm(nblocks * bs, device="cuda")[:n].int()
    us = time_graph(lambda: _C.kv_compact(storage, src_s, dst_s, score), 5)
    byts = n * layers * 2 * hkv * d * 2 * 2
    rows.append({"op": "kv_compact", "tokens": n, "us": round(us, 2),
                 "gbs": round(byts / us / 1e3, 1), "frac_of_" + src: round(byts / bw * 1e6 / us, 3)})
    return rows


def bench_decode(batch, ctx, tp=1, model="llama3-8b"):
    from ..config import get_preset
    cfg = get_preset(model)
    h, f = cfg.hidden_size, cfg.intermediate_size // tp
    hq, hkv = cfg.num_heads // tp, max(1, cfg.num_kv_heads // tp)
    d = cfg.head_dim
    rows = []
    rows.append(bench_gemm(batch, (hq + 2 * hkv) * d, h))
    rows.append(bench_gemm(batch, h, hq * d))
    rows.append(bench_gemm(batch, 2 * f, h, mode=ops.EPI_SWIGLU))
    rows.append(bench_gemm(batch, h, f))
    rows.append(bench_gemm(batch, cfg.vocab_size // tp, h, mode=ops.EPI_F32, iters=5))
    rows.append(bench_decode_attn(batch, ctx, hq, hkv))
    x = torch.randn(batch, h, device="cuda").to(torch.bfloat16)
    r = torch.randn(batch, h, device="cuda").to(torch.bfloat16)
    w = torch.ones(h, device="cuda", dtype=torch.bfloat16)
    rows.append({"op": "rmsnorm_add", "us": round(time_graph(lambda: ops.rmsnorm(x, w, 1e-5, residual=r), 20), 2)})
    qkv = torch.randn(batch, (hq + 2 * hkv) * d, device="cuda").to(torch.bfloat16)
    pos = torch.arange(batch, dtype=torch.int32, device="cuda")
    slots = torch.arange(batch, dtype=torch.int32, device="cuda")
    cs = ops.rope_table(4096, d, cfg.rope_theta, "cuda")
    kc = torch.zeros(batch, hkv, 16, d, device="cuda", dtype=torch.bfloat16)
    rows.append({"op": "rope_kv", "us": round(time_graph(
        lambda: ops.rope_kv(qkv, pos, slots, cs, kc, kc, hq, hkv), 20), 2)})
    logits = torch.randn(batch, cfg.vocab_size, device="cuda")
    z = torch.zeros(batch, device="cuda")
    zi = torch.zeros(batch, dtype=torch.int32, device="cuda")
    seeds = torch.zeros(batch, dtype=torch.int64, device="cuda")
    rows.append({"op": "sample_greedy", "us": round(time_graph(
        lambda: ops.sample(logits, z, zi, z + 1, seeds), 20), 2)})
    per_layer = sum(r["us"] for r in rows[:4]) + rows[5]["us"] + 2 * rows[6]["us"] + rows[7]["us"]
    total = cfg.num_layers * per_layer + rows[4]["us"] + rows[8]["us"]
    rows.append({"op": "estimated_step_us", "us": round(total, 1),
                 "layers": cfg.num_layers, "per_layer_us": round(per_layer, 1)})
    return rows


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["decode", "gemm", "attn", "gemm_trace", "gemm_quant",
                                     "prefill", "small_ops", "kv_ops"])
    ap.add_argument("--chunk", type=int, default=512)
    ap.add_argument("--kind", default="awq", choices=["awq", "q4k", "q80"])
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--ctx", type=int, default=1200)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--m", type=int, default=256)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--bt", type=int, default=0)
    ap.add_argument("--splits", type=int, default=0)
    ap.add_argument("--hq", type=int, default=32)
    ap.add_argument("--hkv", type=int, default=8)
    ap.add_argument("--model", default="llama3-8b")
    a = ap.parse_args(argv)
    torch.cuda.set_device(0)
    if a.what == "decode":
        rows = bench_decode(a.batch, a.ctx, a.tp, a.model)
    elif a.what == "gemm_quant":
        rows = [bench_gemm_quant(a.m, a.n, a.k, a.kind)]
    elif a.what == "gemm_trace":
        rows = [trace_gemm(a.m, a.n, a.k, a.bt, a.splits)]
    elif a.what == "gemm":
        rows = [bench_gemm(a.m, a.n, a.k, bt=a.bt, splits=a.splits)]
    elif a.what == "prefill":
        rows = [bench_prefill_attn(a.batch, a.chunk, a.ctx, a.hq, a.hkv)]
    elif a.what == "small_ops":
        rows = bench_small_ops(a.batch, a.model)
    elif a.what == "kv_ops":
        rows = bench_kv_ops(a.batch, a.ctx, a.hq, a.hkv)
    else:
        rows = [bench_decode_attn(a.batch, a.ctx, a.hq, a.hkv,
                                  splits=a.splits if a.splits else None)]
    for r in rows:
        print(json.dumps(r))
    ops.check_errors()


if __name__ == "__main__":
    sys.exit(main())
