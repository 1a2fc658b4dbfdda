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

Other reference configs (``--config``; the default is the headline above):
  local-gen       config 1: CPU fp32 TinyLlama shape from a random N(0,0.02) safetensors
                  checkpoint through ``local_llama_generate``; 8 seeded prompt ids, greedy 16
  prefill-prefix  config 3: Phi-3-mini shape, 64 x 8192-token prompts sharing a 1024-token
                  prefix (prefix-cache hits), chunked prefill 512, 128 outputs
  spec            config 4: Llama-3-70B shape target + Llama-3.2-1B shape draft, k = 4,
                  batch 32, prompt 1024, 512 outputs (value: emitted tokens / device second)
  awq-h2o         config 5: Llama-3-8B shape AWQ int4 (group 128), 32k-token prompts, H2O
                  budget 2048 + 4 sinks, batch 16, 256 outputs
Sizes can be reduced with --requests / --max-prompt / --output-len / --model for smoke runs.

``--impl reference`` runs the reference implementation (ciresnave/lightbulb); it is a Rust
crate that cannot be built on this image, so that arm prints an ``unavailable`` line.

``--impl ref-algorithm`` (decode config) runs the reference's serving algorithm on this
engine's kernels for comparison: one request at a time to completion (the job loop of
``src/engine/model_runner.rs:383-398``), synchronous steps, NCCL-only tensor parallelism; it
times the decode steps of ``--ref-requests`` requests on the device (max over ranks).
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

BASELINE_TOKS = None  # the reference publishes no B200 figure for this metric and config


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "ref-algorithm"])
    ap.add_argument("--ref-requests", type=int, default=2,
                    help="ref-algorithm arm: requests run one after another")
    ap.add_argument("--config", default="decode",
                    choices=["decode", "local-gen", "prefill-prefix", "spec", "awq-h2o"])
    ap.add_argument("--model", default=None, help="preset (default: the config's model)")
    ap.add_argument("--draft-model", default="llama3.2-1b")
    ap.add_argument("--requests", type=int, default=None)
    ap.add_argument("--min-prompt", type=int, default=None)
    ap.add_argument("--max-prompt", type=int, default=None)
    ap.add_argument("--output-len", type=int, default=None)
    ap.add_argument("--prefix-len", type=int, default=1024)
    ap.add_argument("--chunk", type=int, default=512)
    ap.add_argument("--spec-k", type=int, default=4)
    ap.add_argument("--spec-fallback", dest="spec_no_fallback", action="store_false",
                    help="spec config: keep the engine's auto-fallback to plain decoding")
    ap.add_argument("--h2o-budget", type=int, default=2048)
    ap.add_argument("--h2o-sinks", type=int, default=4)
    ap.add_argument("--block-size", type=int, default=16)
    ap.add_argument("--max-batched-tokens", type=int, default=16384)
    ap.add_argument("--comm", default="p2p", choices=["nccl", "fused", "p2p", "allreduce"],
                    help="TP partial-sum collective (engine option parallel.comm)")
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--seed", type=int, default=1234)
    a = ap.parse_args()
    d = CONFIG_DEFAULTS[a.config]
    for k, v in d.items():
        if getattr(a, k) is None:
            setattr(a, k, v)
    return a


# per-config defaults
CONFIG_DEFAULTS = {
    "decode": dict(model="llama3-8b", requests=256, min_prompt=128, max_prompt=2048,
                   output_len=256),
    "local-gen": dict(model="tinyllama", requests=1, min_prompt=8, max_prompt=8, output_len=16),
    "prefill-prefix": dict(model="phi3-mini", requests=64, min_prompt=8192, max_prompt=8192,
                           output_len=128),
    "spec": dict(model="llama3-70b", requests=32, min_prompt=1024, max_prompt=1024,
                 output_len=512),
    "awq-h2o": dict(model="llama3-8b", requests=16, min_prompt=32768, max_prompt=32768,
                    output_len=256),
}


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

    def _count(self) -> int:
        try:
            with open(self.path) as f:
                return sum(1 for ln in f if not self.uuid or self.uuid in ln)
        except OSError:
            return 0

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        # a short timed region can end before the sampler's first line: wait for one
        t0 = time.time()
        while self._count() == 0 and time.time() - t0 < 1.0:
            time.sleep(0.05)
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
        if not sm:
            # one synchronous query as the last resort
            try:
                out = subprocess.run(["nvidia-smi", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True,
                                     text=True, timeout=10).stdout
                for line in out.splitlines():
                    p = [x.strip() for x in line.split(",")]
                    if len(p) >= 10 and (not self.uuid or p[1] == self.uuid):
                        sm.append(float(p[2]))
                        mx = float(p[3])
                        for n, v in zip(names, p[6:10]):
                            if v.lower().startswith("active"):
                                reasons.add(n)
            except Exception:
                pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def reference_arm(args):
    line = {"impl": "reference",
            "unavailable": "ciresnave/lightbulb is a Rust crate (cargo/rustc absent from the image, "
                           "git dependencies candlelight/fuel need network, CI documents Linux "
                           "builds failing); pip install of the reference source fails: no setup.py "
                           "or pyproject.toml"}
    rank = int(os.environ.get("RANK", "0"))
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def describe(c) -> str:
    return (f"{c.name} ({c.num_layers}L, h{c.hidden_size}, {c.num_heads}/{c.num_kv_heads} heads, "
            f"FFN {c.intermediate_size}, vocab {c.vocab_size})")


def bench_decode(args):
    import random

    import torch
    import torch.distributed as dist

    from lightbulb_b200 import ops
    from lightbulb_b200.config import (CacheConfig, EngineConfig, ParallelConfig, SchedulerConfig,
                                       get_preset)
    from lightbulb_b200.engine.llm_engine import LLMEngine
    from lightbulb_b200.engine.sampling import SamplingParams
    from lightbulb_b200.models.weights import random_packed_model
    from lightbulb_b200.parallel.comm import TPComm, init_distributed

    rank, world, local = init_distributed()
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = TPComm() if world > 1 else None

    mcfg = get_preset(args.model)
    out_len = max(args.output_len, args.warmup + args.steps + 2)
    max_len = args.max_prompt + out_len + 16
    ecfg = EngineConfig(
        model=mcfg,
        cache=CacheConfig(block_size=args.block_size, gpu_memory_utilization=0.92),
        scheduler=SchedulerConfig(max_num_seqs=args.requests,
                                  max_num_batched_tokens=args.max_batched_tokens,
                                  chunk_size=args.max_batched_tokens, max_model_len=max_len),
        use_cuda_graphs=not args.no_graphs, parallel=ParallelConfig(comm=args.comm))
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

    # ---- phase 2: warm-up decode steps (the clock sampler starts here: same kind of steps,
    # so a short timed region still has samples under load) ----
    uuid = ""
    try:
        uuid = str(torch.cuda.get_device_properties(local).uuid)
        uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    except Exception:
        pass
    clocks = ClockSampler(uuid)
    clocks.start()
    eng.runner.enable_step_events()
    gen_tokens = 0
    gen_w0 = time.perf_counter()
    for _ in range(args.warmup):
        gen_tokens += len(eng.step())
    ops.check_errors(dev)
    gen_dev_ms = eng.runner.step_events_total_ms()
    eng.runner.disable_step_events()
    n_active = sum(1 for s in seqs if not s.finished)

    # ---- phase 3: timed decode steps ----
    if comm is not None:
        comm.barrier()
    torch.cuda.synchronize()
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
    # ---- phase 4 (not part of the timed K steps): the rest of the generation, so the line
    # also carries decode throughput over every output token, not only the early window ----
    gen_tokens += tokens
    gen_dev_ms += dev_ms
    eng.runner.enable_step_events()
    while eng.has_unfinished():
        gen_tokens += len(eng.step())
    gen_dev_ms += eng.runner.step_events_total_ms()
    gen_wall = time.perf_counter() - gen_w0
    eng.runner.disable_step_events()
    ops.check_errors(dev)
    if comm is not None:
        comm.barrier()
        dev_ms = comm.max_float(dev_ms)
        wall = comm.max_float(wall)
        gen_dev_ms = comm.max_float(gen_dev_ms)
        gen_wall = comm.max_float(gen_wall)
    itls = sorted(x for s in seqs for x in s.itls()) or [0.0]

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
            "config": {"model": describe(mcfg),
                       "global_batch": args.requests, "seq_len": f"prompt U[{args.min_prompt},"
                       f"{args.max_prompt}] + {out_len} out", "parallelism": f"tp{world}",
                       "kv_block": args.block_size, "comm": args.comm if world > 1 else "none",
                       "l2": "inputs larger than L2 (16 GB weights + KV per step)",
                       "cuda_graphs": not args.no_graphs},
            "ttft_p50_ms": round(1e3 * ttfts[len(ttfts) // 2], 2),
            "itl_p50_ms": round(1e3 * itls[len(itls) // 2], 3),
            "prefill_phase_s": round(prefill_s, 3),
            "active_seqs": n_active,
            "whole_generation": {"decode_tok_s": round(gen_tokens / (gen_dev_ms / 1e3), 2),
                                 "e2e_tok_s": round(gen_tokens / gen_wall, 2),
                                 "tokens": gen_tokens, "device_ms": round(gen_dev_ms, 2),
                                 "note": "every decode step after the last first token, "
                                         "warm-up and timed steps included"},
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





# ======================================================================================
# Shared helpers for the other configs
# ======================================================================================
def _dist():
    import torch
    from lightbulb_b200.parallel.comm import TPComm, init_distributed
    rank, world, local = init_distributed()
    torch.cuda.set_device(local)
    return rank, world, local, torch.device("cuda", local), (TPComm() if world > 1 else None)


def _prompts(args, vocab, prefix=None):
    import random
    rng = random.Random(args.seed)
    out = []
    for _ in range(args.requests):
        L = rng.randint(args.min_prompt, args.max_prompt)
        body = [rng.randrange(vocab) for _ in range(L - (len(prefix) if prefix else 0))]
        out.append((list(prefix) if prefix else []) + body)
    return out


def _run_until_first_token(eng, seqs):
    while any(s.first_token_time is None for s in seqs):
        eng.step()


def _emit(rank, line):
    if rank == 0:
        print(json.dumps(line), flush=True)


def _finish(eng, comm):
    import torch.distributed as dist
    eng.runner.release_graphs()
    spec = getattr(eng, "spec", None)
    if spec is not None:
        spec.draft.release_graphs()
    if comm is not None:
        comm.barrier()
        comm.close()
        comm.barrier()
        dist.destroy_process_group()


# ======================================================================================
# Config 1: CPU local-llama-gen
# ======================================================================================
def bench_local_gen(args):
    import random
    import shutil
    import tempfile

    import torch
    from lightbulb_b200.cli.local_gen import local_llama_generate
    from lightbulb_b200.config import get_preset
    from lightbulb_b200.models.weights import random_weights, save_checkpoint
    rank = int(os.environ.get("RANK", "0"))
    cfg = get_preset(args.model)
    d = tempfile.mkdtemp(prefix="lb_localgen_")
    try:
        t0 = time.perf_counter()
        w = random_weights(cfg, seed=args.seed, std=0.02, dtype=torch.float32)
        save_checkpoint(d, cfg, w)
        del w
        write_s = time.perf_counter() - t0
        rng = random.Random(args.seed)
        ids = [rng.randrange(cfg.vocab_size) for _ in range(args.max_prompt)]
        for _ in range(max(1, args.warmup)):
            local_llama_generate(d, "", sample_len=args.output_len, prompt_ids=ids)
        runs = []
        for _ in range(max(1, args.steps)):
            t = time.perf_counter()
            r = local_llama_generate(d, "", sample_len=args.output_len, prompt_ids=ids)
            runs.append((time.perf_counter() - t, r))
        secs = sum(t for t, _ in runs)
        toks = sum(len(r["tokens"]) for _, r in runs)
        value = toks / secs
        _emit(rank, {
            "metric": "local-llama-gen tokens/s (CPU fp32, greedy)", "value": round(value, 3),
            "unit": "tokens/s", "n_gpus": 0, "steps": len(runs), "warmup": max(1, args.warmup),
            "ms_per_step": round(1e3 * secs / len(runs), 2), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (seeded prompt ids, random-init N(0,0.02) safetensors)",
            "impl": "ours",
            "config": {"model": describe(cfg), "prompt_ids": args.max_prompt,
                       "new_tokens": args.output_len, "device": "cpu",
                       "threads": torch.get_num_threads()},
            "ms_per_token": round(statistics.median(r["ms_per_token"] for _, r in runs), 2),
            "tokens": runs[-1][1]["tokens"],
            "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0, "api": "local_llama_generate (loads the checkpoint "
                    "each run)"},
            "gpu_launches": 0, "checkpoint_write_s": round(write_s, 1)})
    finally:
        shutil.rmtree(d, ignore_errors=True)
    return 0


# ======================================================================================
# Config 3: chunked prefill with a shared prefix (prefix-cache hits)
# ======================================================================================
def bench_prefill_prefix(args):
    import random

    import torch
    from lightbulb_b200 import ops
    from lightbulb_b200.config import (CacheConfig, EngineConfig, ParallelConfig, SchedulerConfig,
                                       get_preset)
    from lightbulb_b200.engine.llm_engine import LLMEngine
    from lightbulb_b200.engine.sampling import SamplingParams
    from lightbulb_b200.models.weights import random_packed_model
    rank, world, local, dev, comm = _dist()
    mcfg = get_preset(args.model)
    max_len = args.max_prompt + args.output_len + 16
    ecfg = EngineConfig(model=mcfg,
                        cache=CacheConfig(block_size=args.block_size, gpu_memory_utilization=0.92,
                                          enable_prefix_caching=True),
                        scheduler=SchedulerConfig(max_num_seqs=args.requests,
                                                  max_num_batched_tokens=args.chunk,
                                                  chunk_size=args.chunk, max_model_len=max_len),
                        use_cuda_graphs=not args.no_graphs, parallel=ParallelConfig(comm=args.comm))
    packed = random_packed_model(mcfg, seed=args.seed, rank=rank, world=world, device=dev)
    eng = LLMEngine(ecfg, packed, None, comm=comm, tp_rank=rank, tp_size=world)
    rng = random.Random(args.seed + 1)
    prefix = [rng.randrange(mcfg.vocab_size) for _ in range(args.prefix_len)]
    prompts = _prompts(args, mcfg.vocab_size, prefix)
    sp = SamplingParams(temperature=0.0, max_tokens=args.output_len, ignore_eos=True,
                        detokenize=False)
    if not args.no_graphs:
        eng.runner.capture_all(up_to=args.requests)
    # warm-up: one short request through the same path (kernels, allocator)
    eng.generate(prompt_token_ids=[prompts[0][:args.chunk + 7]],
                 params=SamplingParams(temperature=0.0, max_tokens=2, ignore_eos=True,
                                       detokenize=False))
    torch.cuda.synchronize()
    if comm is not None:
        comm.barrier()
    ev = eng.runner.enable_step_events()
    ops.launch_counter_reset()
    steps = 0
    w0 = time.perf_counter()
    seqs = [eng.add_request(f"p{i}", prompt_token_ids=p, params=sp) for i, p in enumerate(prompts)]
    while any(s.first_token_time is None for s in seqs):
        eng.step()
        steps += 1
    torch.cuda.synchronize()
    pre_wall = time.perf_counter() - w0
    pre_dev = eng.runner.step_events_total_ms()
    eng.runner.enable_step_events()
    dec_tokens = 0
    d0 = time.perf_counter()
    dsteps = 0
    while eng.has_unfinished():
        dec_tokens += len(eng.step())
        dsteps += 1
    torch.cuda.synchronize()
    dec_wall = time.perf_counter() - d0
    dec_dev = eng.runner.step_events_total_ms()
    launches = ops.launch_counter_value()
    eng.runner.disable_step_events()
    ops.check_errors(dev)
    if comm is not None:
        pre_dev, dec_dev = comm.max_float(pre_dev), comm.max_float(dec_dev)
        pre_wall, dec_wall = comm.max_float(pre_wall), comm.max_float(dec_wall)
    ttfts = sorted(s.first_token_time - s.arrival_time for s in seqs)
    prompt_tokens = sum(len(p) for p in prompts)
    cached = sum(s.num_cached_prefix for s in seqs)
    value = prompt_tokens / (pre_dev / 1e3)
    _emit(rank, {
        "metric": "prompt tok/s (chunked prefill 512, shared-prefix cache hits), p50 TTFT",
        "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": 1, "ms_per_step": round(pre_dev / max(1, steps), 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-id prompts with a shared prefix, random-init weights)",
        "impl": "ours",
        "config": {"model": describe(mcfg), "global_batch": args.requests,
                   "seq_len": f"{args.max_prompt} prompt ({args.prefix_len} shared) + "
                              f"{args.output_len} out", "parallelism": f"tp{world}",
                   "chunk": args.chunk, "kv_block": args.block_size,
                   "head_dim": f"{mcfg.head_dim} (zero-padded to {mcfg.head_dim_padded})",
                   "l2": "inputs larger than L2 (weights + KV per step)"},
        "prompt_tokens": prompt_tokens, "prefix_cache_hit_tokens": cached,
        "ttft_p50_ms": round(1e3 * ttfts[len(ttfts) // 2], 1),
        "decode_tok_s": round(dec_tokens / max(1e-9, dec_dev / 1e3), 1),
        "decode_steps": dsteps,
        "e2e": {"value": round(prompt_tokens / pre_wall, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": None, "d2h_bytes_per_step": None,
                "api": "LLMEngine.add_request + step() until every request has its first token",
                "decode_tok_s": round(dec_tokens / dec_wall, 1)},
        "gpu_launches": launches})
    _finish(eng, comm)
    return 0


# ======================================================================================
# Config 4: speculative decoding (target + draft)
# ======================================================================================
def bench_spec(args):
    import torch
    from lightbulb_b200 import ops
    from lightbulb_b200.config import (CacheConfig, EngineConfig, ParallelConfig, SchedulerConfig,
                                       get_preset)
    from lightbulb_b200.engine.llm_engine import LLMEngine
    from lightbulb_b200.engine.sampling import SamplingParams
    from lightbulb_b200.models.weights import random_packed_model
    rank, world, local, dev, comm = _dist()
    mcfg = get_preset(args.model)
    dcfg = get_preset(args.draft_model)
    k = args.spec_k
    max_len = args.max_prompt + args.output_len + k + 32
    nb = args.requests * ((max_len + args.block_size - 1) // args.block_size) + 64
    ecfg = EngineConfig(model=mcfg, cache=CacheConfig(block_size=args.block_size, num_blocks=nb),
                        scheduler=SchedulerConfig(max_num_seqs=args.requests,
                                                  max_num_batched_tokens=args.max_batched_tokens,
                                                  chunk_size=args.max_batched_tokens,
                                                  max_model_len=max_len),
                        use_cuda_graphs=not args.no_graphs, parallel=ParallelConfig(comm=args.comm))
    t0 = time.perf_counter()
    packed = random_packed_model(mcfg, seed=args.seed, rank=rank, world=world, device=dev)
    eng = LLMEngine(ecfg, packed, None, comm=comm, tp_rank=rank, tp_size=world)
    dpacked = random_packed_model(dcfg, seed=args.seed + 7, rank=rank, world=world, device=dev)
    # the engine's auto-fallback (off below an acceptance of 0.3 after 10 rounds) stays off
    # here, so every timed step is a speculative round: unrelated random-init models accept
    # almost nothing, and the number shows the cost of the draft + verify machinery
    spec = eng.attach_draft(dpacked, dcfg, k=k, num_blocks=nb,
                            min_acceptance=0.0 if args.spec_no_fallback else 0.3)
    load_s = time.perf_counter() - t0
    prompts = _prompts(args, min(mcfg.vocab_size, dcfg.vocab_size))
    out_len = max(args.output_len, 8)
    sp = SamplingParams(temperature=0.0, max_tokens=out_len, ignore_eos=True, detokenize=False)
    seqs = [eng.add_request(f"s{i}", prompt_token_ids=p, params=sp) for i, p in enumerate(prompts)]
    _run_until_first_token(eng, seqs)
    for _ in range(args.warmup):
        eng.step()
    ops.check_errors(dev)
    if comm is not None:
        comm.barrier()
    torch.cuda.synchronize()
    eng.runner.enable_step_events()
    spec.draft.enable_step_events()
    ops.launch_counter_reset()
    p0, a0 = spec.stats.proposed, spec.stats.accepted
    tokens = 0
    w0 = time.perf_counter()
    steps = 0
    for _ in range(args.steps):
        if not eng.has_unfinished():
            break
        tokens += len(eng.step())
        steps += 1
    torch.cuda.synchronize()
    wall = time.perf_counter() - w0
    dev_ms = eng.runner.step_events_total_ms() + spec.draft.step_events_total_ms()
    launches = ops.launch_counter_value()
    eng.runner.disable_step_events()
    spec.draft.disable_step_events()
    ops.check_errors(dev)
    if comm is not None:
        dev_ms, wall = comm.max_float(dev_ms), comm.max_float(wall)
    prop, acc = spec.stats.proposed - p0, spec.stats.accepted - a0
    value = tokens / (dev_ms / 1e3)
    _emit(rank, {
        "metric": "speculative decode tok/s (emitted tokens / device second), acceptance",
        "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(dev_ms / max(1, steps), 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-id prompts, random-init target and draft: acceptance is "
                "that of unrelated models)",
        "impl": "ours",
        "config": {"model": describe(mcfg), "draft": describe(dcfg), "k": k,
                   "global_batch": args.requests,
                   "seq_len": f"{args.max_prompt} prompt + {out_len} out",
                   "parallelism": f"tp{world}",
                   "l2": "inputs larger than L2 (weights + KV per step)"},
        "acceptance_rate": round(acc / prop, 4) if prop else None,
        "speculation_active": spec.active, "spec_rounds": spec.stats.rounds,
        "auto_fallback": not args.spec_no_fallback,
        "e2e": {"value": round(tokens / wall, 2), "unit": "tokens/s",
                "h2d_bytes_per_step": None, "d2h_bytes_per_step": None,
                "api": "LLMEngine.step() with SpeculativeDecoder attached"},
        "gpu_launches": launches, "load_s": round(load_s, 1)})
    _finish(eng, comm)
    return 0


# ======================================================================================
# Config 5: AWQ int4 + H2O KV compression on long prompts
# ======================================================================================
def bench_awq_h2o(args):
    import torch
    from lightbulb_b200 import ops
    from lightbulb_b200.config import (CacheConfig, EngineConfig, ParallelConfig, SchedulerConfig,
                                       get_preset)
    from lightbulb_b200.engine.llm_engine import LLMEngine
    from lightbulb_b200.engine.sampling import SamplingParams
    from lightbulb_b200.models.weights import random_packed_awq_model
    rank, world, local, dev, comm = _dist()
    mcfg = get_preset(args.model, max_position_embeddings=max(
        131072, args.max_prompt + args.output_len + 64))
    out_len = max(args.output_len, args.warmup + args.steps + 2)
    max_len = args.max_prompt + out_len + 64
    ecfg = EngineConfig(model=mcfg,
                        cache=CacheConfig(block_size=args.block_size, gpu_memory_utilization=0.9),
                        scheduler=SchedulerConfig(max_num_seqs=args.requests,
                                                  max_num_batched_tokens=args.max_batched_tokens,
                                                  chunk_size=args.max_batched_tokens,
                                                  max_model_len=max_len),
                        use_cuda_graphs=not args.no_graphs, parallel=ParallelConfig(comm=args.comm))
    t0 = time.perf_counter()
    packed = random_packed_awq_model(mcfg, seed=args.seed, rank=rank, world=world, device=dev)
    eng = LLMEngine(ecfg, packed, None, comm=comm, tp_rank=rank, tp_size=world)
    eng.enable_kv_compression("h2o", budget=args.h2o_budget, sinks=args.h2o_sinks)
    load_s = time.perf_counter() - t0
    prompts = _prompts(args, mcfg.vocab_size)
    sp = SamplingParams(temperature=0.0, max_tokens=out_len, ignore_eos=True, detokenize=False)
    if not args.no_graphs:
        eng.runner.capture_all(up_to=args.requests)
    t_arr = time.perf_counter()
    seqs = [eng.add_request(f"a{i}", prompt_token_ids=p, params=sp) for i, p in enumerate(prompts)]
    _run_until_first_token(eng, seqs)
    prefill_s = time.perf_counter() - t_arr
    for _ in range(args.warmup):
        eng.step()
    ops.check_errors(dev)
    if comm is not None:
        comm.barrier()
    torch.cuda.synchronize()
    eng.runner.enable_step_events()
    ops.launch_counter_reset()
    tokens = 0
    h2d = d2h = 0
    w0 = time.perf_counter()
    for _ in range(args.steps):
        tokens += len(eng.step())
        a, b = eng.last_step_io()
        h2d += a
        d2h += b
    torch.cuda.synchronize()
    wall = time.perf_counter() - w0
    dev_ms = eng.runner.step_events_total_ms()
    launches = ops.launch_counter_value()
    eng.runner.disable_step_events()
    ops.check_errors(dev)
    if comm is not None:
        dev_ms, wall = comm.max_float(dev_ms), comm.max_float(wall)
    kv_lens = [s.num_computed_tokens for s in seqs if not s.finished]  # KV-resident tokens
    ttfts = sorted(s.first_token_time - s.arrival_time for s in seqs)
    value = tokens / (dev_ms / 1e3)
    _emit(rank, {
        "metric": "decode tok/s with H2O KV compression (AWQ int4 weights), p50 TTFT",
        "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 activations, int4 weights (group 128)",
        "data": "synthetic (random-id prompts, random uint4 weights, fp16 scales U[0.001,0.02], "
                "zeros U{0..15})",
        "impl": "ours",
        "config": {"model": describe(mcfg) + " AWQ int4", "global_batch": args.requests,
                   "seq_len": f"{args.max_prompt} prompt + {out_len} out",
                   "parallelism": f"tp{world}",
                   "h2o": {"budget": args.h2o_budget, "sinks": args.h2o_sinks},
                   "l2": "inputs larger than L2 (weights + KV per step)"},
        "ttft_p50_ms": round(1e3 * ttfts[len(ttfts) // 2], 1),
        "prefill_phase_s": round(prefill_s, 2),
        "kv_tokens_per_seq_max": max(kv_lens) if kv_lens else None,
        "h2o_compactions": eng.kv_policy.compactions,
        "e2e": {"value": round(tokens / wall, 2), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d // max(1, args.steps),
                "d2h_bytes_per_step": d2h // max(1, args.steps), "api": "LLMEngine.step()"},
        "gpu_launches": launches, "load_s": round(load_s, 1)})
    _finish(eng, comm)
    return 0


def bench_ref_algorithm(args):
    """The reference's serving algorithm on this engine: requests run serially, batch 1."""
    import torch
    import torch.distributed as dist
    from lightbulb_b200.config import (CacheConfig, EngineConfig, ParallelConfig,
                                       SchedulerConfig, get_preset)
    from lightbulb_b200.engine.llm_engine import LLMEngine
    from lightbulb_b200.engine.sampling import SamplingParams
    from lightbulb_b200.models.weights import random_packed_model
    rank, world, local, dev, comm = _dist()
    mcfg = get_preset(args.model)
    steps = max(1, args.steps)
    out_len = args.warmup + steps + 1
    ecfg = EngineConfig(model=mcfg, cache=CacheConfig(block_size=args.block_size,
                                                      gpu_memory_utilization=0.9),
                        scheduler=SchedulerConfig(max_num_seqs=1, max_num_batched_tokens=2048,
                                                  chunk_size=2048,
                                                  max_model_len=args.max_prompt + out_len + 16),
                        use_cuda_graphs=not args.no_graphs, overlap_decode=False,
                        parallel=ParallelConfig(comm="nccl"))
    packed = random_packed_model(mcfg, seed=args.seed, rank=rank, world=world, device=dev)
    eng = LLMEngine(ecfg, packed, None, comm=comm, tp_rank=rank, tp_size=world)
    prompts = _prompts(args, mcfg.vocab_size)[:max(1, args.ref_requests)]
    sp = SamplingParams(temperature=0.0, max_tokens=out_len, ignore_eos=True, detokenize=False)
    dev_ms, tokens = 0.0, 0
    for i, p in enumerate(prompts):
        s = eng.add_request(f"ref{i}", prompt_token_ids=p, params=sp)
        _run_until_first_token(eng, [s])
        for _ in range(args.warmup):
            eng.step()
        if comm is not None:
            comm.barrier()
        torch.cuda.synchronize()
        eng.runner.enable_step_events()
        for _ in range(steps):
            tokens += len(eng.step())
        dev_ms += eng.runner.step_events_total_ms()
        eng.runner.disable_step_events()
        while eng.has_unfinished():
            eng.step()
    if comm is not None:
        dev_ms = comm.max_float(dev_ms)
    value = tokens / (dev_ms / 1e3)
    _emit(rank, {
        "impl": "ref-algorithm",
        "metric": "decode tok/s, p50 TTFT/ITL; Llama-3-8B shape, TP=1/2/4/8 B200, max over ranks",
        "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_token": round(dev_ms / max(1, tokens), 4),
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"model": describe(mcfg), "requests_timed": len(prompts),
                   "parallelism": f"tp{world}", "comm": "nccl", "batch": 1,
                   "cuda_graphs": not args.no_graphs},
        "note": "reference serving algorithm (one request at a time, NCCL-only TP) on this "
                "engine's kernels; not the reference build"})
    _finish(eng, comm)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    if args.impl == "ref-algorithm":
        return bench_ref_algorithm(args)
    return {"decode": bench_decode, "local-gen": bench_local_gen,
            "prefill-prefix": bench_prefill_prefix, "spec": bench_spec,
            "awq-h2o": bench_awq_h2o}[args.config](args)


if __name__ == "__main__":
    sys.exit(main())
