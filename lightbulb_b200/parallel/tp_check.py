"""Tensor-parallel self-check (run under torchrun, one process per GPU).

    torchrun --nproc-per-node N -m lightbulb_b200.parallel.tp_check [--comm nccl|fused|p2p|allreduce]

Every rank builds the same random-init model sharded over the ranks and greedily generates;
rank 0 also runs the unsharded model on its own GPU and compares.  Exit code 0 = match.
"""
from __future__ import annotations

import argparse
import sys

import torch
import torch.distributed as dist


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--comm", default="nccl", choices=["nccl", "fused", "p2p", "allreduce"])
    ap.add_argument("--graphs", type=int, default=1)
    args = ap.parse_args(argv)
    from ..config import CacheConfig, EngineConfig, ParallelConfig, SchedulerConfig, get_preset
    from ..engine.llm_engine import LLMEngine
    from ..engine.sampling import SamplingParams
    from ..models.weights import pack_model, random_weights
    from .comm import TPComm, init_distributed

    rank, world, local = init_distributed(timeout_s=60)
    dev = torch.device("cuda", local)
    cfg = get_preset("tiny-test", hidden_size=1024, intermediate_size=2048, num_heads=8,
                     num_kv_heads=8, head_dim=128, vocab_size=2048, num_layers=2)
    w = random_weights(cfg, seed=11, std=0.05)
    w = {k: v.to(torch.bfloat16).float() for k, v in w.items()}
    comm = TPComm()

    def engine(r, n, c):
        packed = pack_model(cfg, w, rank=r, world=n, dtype=torch.bfloat16, device=dev)
        ecfg = EngineConfig(model=cfg, cache=CacheConfig(num_blocks=128, block_size=16),
                            scheduler=SchedulerConfig(max_num_seqs=8, max_num_batched_tokens=128,
                                                      chunk_size=64, max_model_len=512),
                            use_cuda_graphs=bool(args.graphs),
                            parallel=ParallelConfig(comm=args.comm))
        return LLMEngine(ecfg, packed, comm=c, tp_rank=r, tp_size=n)

    prompts = [list(range(3, 80)), [5, 6, 7], [100] * 40]
    sp = SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True)
    eng = engine(rank, world, comm)
    out = [s.output_token_ids for s in eng.generate(prompt_token_ids=prompts, params=sp)]
    eng.runner.release_graphs()
    from .. import ops
    ops.check_errors(dev)
    ok = torch.tensor([1], device=dev)
    if rank == 0:
        # Teacher-forced oracle (tolerance covers bf16 partial sums under TP): every token must be the fp32 argmax along the
        # emitted trajectory unless the oracle's top-2 logits are within bf16 noise.
        from ..models.reference import ReferenceLlama
        ref = ReferenceLlama(cfg, w)
        bad = []
        for p, o in zip(prompts, out):
            ref.reset()
            lg = ref.forward(torch.tensor(p + o[:-1]))[len(p) - 1:]
            for i, t in enumerate(o):
                v, ix = torch.topk(lg[i], 2)
                if int(ix[0]) != t and float(v[0] - v[1]) > 0.15:
                    bad.append((i, t, ix.tolist(), float(v[0] - v[1])))
        print(f"tp{world} {args.comm}: {out}\nmismatches vs fp32 oracle: {bad}", flush=True)
        ok[0] = int(not bad)
    dist.broadcast(ok, 0)
    dist.barrier()
    comm.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0 if int(ok.item()) == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
