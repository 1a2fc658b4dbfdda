#!/usr/bin/env python
"""Headline benchmark: continuous-batching decode throughput (+ p50 TTFT / ITL).

Config: Llama-3-8B-shaped bf16, random-init weights, 256 requests with
random-id prompts of length U[128, 2048], 256 output tokens each, paged KV block 16,
tensor parallel over N GPUs (one process per GPU, torchrun).

Procedure (our arm):
  1. all 256 requests arrive at t=0; the engine runs continuous batching (chunked prefill +
     decode) until every request is decoding -> TTFT of each request;
  2. W warm-up decode steps, then K timed decode steps through ``LLMEngine.step()``:
     * value: decode tokens / sum of per-step DEVICE time (CUDA events around each step's
       CUDA-graph replay), max over ranks;
     * e2e:   the same steps by wall clock through the public API, including each step's
       H2D copy of its inputs from pinned memory and the D2H read of the sampled ids.
  Every timed step reads all weights (16 GB) and all resident KV (tens of GB), both far
  larger than the 126 MB L2, so no L2 flush is needed between steps.

``--impl reference`` runs the reference implementation (ciresnave/lightbulb); it is a Rust
crate that cannot be built on this image, so that arm prints an ``unavailable`` line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BASELINE_TOKS = None  # BASELINE.md publishes no number for this config


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--requests", type=int, default=256)
    ap.add_argument("--min-prompt", type=int, default=128)
    ap.add_argument("--max-prompt", type=int, default=2048)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--block-size", type=int, default=16)
    ap.add_argument("--max-batched-tokens", type=int, default=16384)
    ap.add_argument("--comm", default="nccl", choices=["nccl", "fused"])
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--seed", type=int, default=1234)
    return ap.parse_args()


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str):
        self.uuid = uuid
        self.proc = None
        self.path = os.path.join("/tmp", f"lb_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                p = [x.strip() for x in line.split(",")]
                if len(p) < 10 or (self.uuid and p[1] != self.uuid):
                    continue
                try:
                    sm.append(float(p[2]))
                    mx = float(p[3])
                except ValueError:
                    continue
                for n, v in zip(names, p[6:10]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def reference_arm(args):
    line = {"impl": "reference",
            "unavailable": "ciresnave/lightbulb is a Rust crate (cargo/rustc absent from the image, "
                           "git dependencies candlelight/fuel need network, CI documents Linux "
                           "builds failing); pip install of /root/reference fails: no setup.py "
                           "or pyproject.toml"}
    rank = int(os.environ.get("RANK", "0"))
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    import random

    import torch
    import torch.distributed as dist

    from lightbulb_b200 import ops
    from lightbulb_b200.config import (CacheConfig, EngineConfig, SchedulerConfig, get_preset)
    from lightbulb_b200.engine.llm_engine import LLMEngine
    from lightbulb_b200.engine.sampling import SamplingParams
    from lightbulb_b200.models.weights import random_packed_model
    from lightbulb_b200.parallel.comm import TPComm, init_distributed

    rank, world, local = init_distributed()
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = TPComm() if world > 1 else None
    if comm is not None and args.comm == "fused":
        from lightbulb_b200.parallel.fused import enable_fused
        enable_fused(comm)

    mcfg = get_preset(args.model)
    out_len = max(args.output_len, args.warmup + args.steps + 2)
    max_len = args.max_prompt + out_len + 16
    ecfg = EngineConfig(
        model=mcfg,
        cache=CacheConfig(block_size=args.block_size, gpu_memory_utilization=0.92),
        scheduler=SchedulerConfig(max_num_seqs=args.requests,
                                  max_num_batched_tokens=args.max_batched_tokens,
                                  chunk_size=args.max_batched_tokens, max_model_len=max_len),
        use_cuda_graphs=not args.no_graphs)
    t0 = time.perf_counter()
    packed = random_packed_model(mcfg, seed=args.seed, rank=rank, world=world, device=dev)
    torch.cuda.synchronize()
    eng = LLMEngine(ecfg, packed, None, comm=comm, tp_rank=rank, tp_size=world)
    load_s = time.perf_counter() - t0

    rng = random.Random(args.seed)
    prompts = []
    for _ in range(args.requests):
        L = rng.randint(args.min_prompt, args.max_prompt)
        prompts.append([rng.randrange(mcfg.vocab_size) for _ in range(L)])
    sp = SamplingParams(temperature=0.0, max_tokens=out_len, ignore_eos=True, detokenize=False)

    # Capture the decode graph for the full batch before any request arrives.
    if not args.no_graphs:
        eng.runner.capture_all(up_to=args.requests)
    ops.launch_counter_reset()
    # ---- phase 1: arrival + continuous batching until everyone decodes (TTFT) ----
    t_arr = time.perf_counter()
    seqs = [eng.add_request(f"req{i}", prompt_token_ids=p, params=sp) for i, p in enumerate(prompts)]
    while any(s.first_token_time is None for s in seqs):
        eng.step()
    prefill_s = time.perf_counter() - t_arr
    ttfts = sorted(s.first_token_time - s.arrival_time for s in seqs)

    # ---- phase 2: warm-up decode steps ----
    for _ in range(args.warmup):
        eng.step()
    ops.check_errors(dev)
    n_active = sum(1 for s in seqs if not s.finished)

    # ---- phase 3: timed decode steps ----
    if comm is not None:
        comm.barrier()
    torch.cuda.synchronize()
    uuid = ""
    try:
        uuid = str(torch.cuda.get_device_properties(local).uuid)
        uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    except Exception:
        pass
    clocks = ClockSampler(uuid)
    clocks.start()
    ev = eng.runner.enable_step_events()
    ops.launch_counter_reset()
    tokens = 0
    h2d = d2h = 0
    w0 = time.perf_counter()
    for _ in range(args.steps):
        outs = eng.step()
        tokens += len(outs)
        a, b = eng.last_step_io()
        h2d += a
        d2h += b
    torch.cuda.synchronize()
    wall = time.perf_counter() - w0
    launches = ops.launch_counter_value()
    dev_ms = eng.runner.step_events_total_ms()
    eng.runner.disable_step_events()
    clk = clocks.stop()
    ops.check_errors(dev)
    if comm is not None:
        comm.barrier()
        dev_ms = comm.max_float(dev_ms)
        wall = comm.max_float(wall)
    itls = sorted(eng.stats.itls) if eng.stats.itls else [0.0]

    value = tokens / (dev_ms / 1e3)
    e2e = tokens / wall
    if rank == 0:
        line = {
            "metric": "decode tok/s, p50 TTFT/ITL; Llama-3-8B shape, TP=1/2/4/8 B200, max over ranks",
            "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 4),
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": (value / BASELINE_TOKS) if BASELINE_TOKS else None,
            "dtype": "bf16", "data": "synthetic (random-id prompts, random-init N(0,0.02) weights)",
            "impl": "ours",
            "config": {"model": f"{args.model} (32L, h4096, 32/8 heads, FFN 14336, vocab 128256)",
                       "global_batch": args.requests, "seq_len": f"prompt U[{args.min_prompt},"
                       f"{args.max_prompt}] + {out_len} out", "parallelism": f"tp{world}",
                       "kv_block": args.block_size, "comm": args.comm if world > 1 else "none",
                       "l2": "inputs larger than L2 (16 GB weights + KV per step)",
                       "cuda_graphs": not args.no_graphs},
            "ttft_p50_ms": round(1e3 * ttfts[len(ttfts) // 2], 2),
            "itl_p50_ms": round(1e3 * itls[len(itls) // 2], 3),
            "prefill_phase_s": round(prefill_s, 3),
            "active_seqs": n_active,
            "e2e": {"value": round(e2e, 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d // max(1, args.steps),
                    "d2h_bytes_per_step": d2h // max(1, args.steps),
                    "api": "LLMEngine.step()"},
            "gpu_launches": launches,
            "clocks": clk,
            "load_s": round(load_s, 1),
        }
        print(json.dumps(line), flush=True)
    eng.runner.release_graphs()
    if comm is not None:
        comm.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
