"""Tensor parallelism on CPU ranks (gloo, world size 2): sharded weights + collectives must
reproduce the single-process tokens (greedy)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _engine(cfg, w, rank, world, comm):
    from lightbulb_b200.config import CacheConfig, EngineConfig, SchedulerConfig
    from lightbulb_b200.engine.llm_engine import LLMEngine
    from lightbulb_b200.models.weights import pack_model
    packed = pack_model(cfg, w, rank=rank, world=world, dtype=torch.bfloat16, device="cpu")
    ecfg = EngineConfig(model=cfg, cache=CacheConfig(num_blocks=64, block_size=16),
                        scheduler=SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=64,
                                                  chunk_size=32, max_model_len=256),
                        use_cuda_graphs=False)
    return LLMEngine(ecfg, packed, comm=comm, tp_rank=rank, tp_size=world)


def _setup():
    from lightbulb_b200.config import get_preset
    from lightbulb_b200.models.weights import random_weights
    cfg = get_preset("tiny-test")
    w = random_weights(cfg, seed=5, std=0.05)
    return cfg, {k: v.to(torch.bfloat16).float() for k, v in w.items()}


PROMPTS = [list(range(5, 45)), [9, 8, 7]]


def _worker(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from lightbulb_b200.engine.sampling import SamplingParams
    from lightbulb_b200.parallel.comm import TPComm
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        cfg, w = _setup()
        eng = _engine(cfg, w, rank, world, TPComm())
        seqs = eng.generate(prompt_token_ids=PROMPTS,
                            params=SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
        out_q.put((rank, [s.output_token_ids for s in seqs]))
    except Exception as e:  # report instead of leaving the parent waiting
        out_q.put((rank, f"error: {e!r}"))
    finally:
        dist.destroy_process_group()


def test_tp2_matches_single_process():
    from lightbulb_b200.engine.sampling import SamplingParams
    cfg, w = _setup()
    single = _engine(cfg, w, 0, 1, None)
    ref = [s.output_token_ids for s in single.generate(
        prompt_token_ids=PROMPTS,
        params=SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    assert not any(isinstance(v, str) for v in res.values()), res
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0] == res[1]
    # bf16 partial sums reduce in a different order under TP: allow a near-tie flip late on
    for a, b in zip(res[0], ref):
        assert a[:4] == b[:4]


def _argmax_worker(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from datetime import timedelta
    from lightbulb_b200.parallel.comm import TPComm
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(3)
        full = torch.randn(5, 40, generator=g)
        full[1, 7] = full[1, 27] = 9.0        # tie across shards: first (global 7) wins
        full[2, 30] = 8.0
        full[3, 12] = full[3, 13] = 7.0       # tie inside a shard
        shard = full[:, rank * 20:(rank + 1) * 20].contiguous()
        out = torch.zeros(5, dtype=torch.int32)
        TPComm().argmax_vocab_parallel(shard, out)
        out_q.put((rank, out.tolist(), full.argmax(1).tolist()))
    except Exception as e:
        out_q.put((rank, f"error: {e!r}", None))
    finally:
        dist.destroy_process_group()


def test_argmax_vocab_parallel_first_max():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_argmax_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, got, ref in res:
        assert not isinstance(got, str), got
        assert got == ref and got[1] == 7 and got[3] == 12


def test_rowpar_owned_rows_partition():
    # token rows are owned in contiguous ranges of ceil(T / world); every row exactly once,
    # ranks past the end own nothing (e.g. 3 tokens on 8 ranks)
    from lightbulb_b200.parallel.rowpar import owned_rows
    for world in (2, 3, 4, 8):
        for T in (1, 3, 7, 8, 255, 256, 257, 640):
            seen = []
            for r in range(world):
                r0, n = owned_rows(T, world, r)
                assert n >= 0 and (n == 0 or r0 + n <= T)
                seen += list(range(r0, r0 + n))
            assert seen == list(range(T))
