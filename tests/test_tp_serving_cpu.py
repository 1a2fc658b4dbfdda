"""Tensor-parallel serving on CPU ranks (gloo, world size 2): rank 0 serves requests through
the asynchronous engine, rank 1 follows through the control plane; the streamed tokens must
equal the single-process engine's (greedy), and the worker must stop when rank 0 shuts down."""
import os
import socket

import torch
import torch.multiprocessing as mp

from test_tp_cpu import PROMPTS, _engine, _free_port, _setup


def _serve_rank(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import asyncio
    from datetime import timedelta

    import torch.distributed as dist

    from lightbulb_b200.engine.sampling import SamplingParams
    from lightbulb_b200.parallel.comm import TPComm
    from lightbulb_b200.parallel.serving import ControlPlane, run_worker
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        cfg, w = _setup()
        eng = _engine(cfg, w, rank, world, TPComm())
        plane = ControlPlane(timeout_s=120)
        if rank == 0:
            from lightbulb_b200.engine.async_engine import AsyncEngine
            ae = AsyncEngine(eng)
            ae.attach_control_plane(plane)
            sp = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True)

            async def one(p):
                toks = []
                async for it in ae.generate(prompt_token_ids=p, params=sp):
                    toks += list(it.token_ids or [])
                return toks

            async def both():
                return await asyncio.gather(*(one(p) for p in PROMPTS))
            outs = asyncio.new_event_loop().run_until_complete(both())
            ae.shutdown()                      # publishes stop to the worker
            out_q.put(("served", outs))
        else:
            out_q.put(("worker_steps", run_worker(eng, plane)))
        dist.barrier()
    except Exception as e:  # report instead of leaving the parent waiting
        out_q.put(("served" if rank == 0 else "worker_steps", f"error: {e!r}"))
    finally:
        dist.destroy_process_group()


def test_tp_serving_matches_single_process():
    from lightbulb_b200.engine.sampling import SamplingParams
    cfg, w = _setup()
    single = _engine(cfg, w, 0, 1, None)
    ref = [s.output_token_ids for s in single.generate(
        prompt_token_ids=PROMPTS,
        params=SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_serve_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert not any(isinstance(v, str) for v in got.values()), got
    # bf16 partial sums reduce in a different order under TP: allow a near-tie flip late on
    for a, b in zip(got["served"], ref):
        assert len(a) == 8 and a[:4] == b[:4]
    assert got["worker_steps"] > 0
