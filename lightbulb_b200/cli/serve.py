"""Server bootstrap (reference ``src/main.rs:12-77`` and ``ApiServer::new/serve``,
``src/api/mod.rs:166-470``).

    python -m lightbulb_b200.cli.serve [--model PATH] [--bind 127.0.0.1:8080]
    torchrun --nproc-per-node N -m lightbulb_b200.cli.serve --model PATH   # tensor parallel

Environment (same names as the reference): ``LIGHTBULB_BIND_ADDRESS``,
``LIGHTBULB_MODELS_DIR`` + ``LIGHTBULB_DEFAULT_MODEL`` (model = models_dir/default_model when
it exists), ``DATABASE_URL`` (sqlite:///path enables API keys / rate limit / audit),
``LIGHTBULB_TLS_CERT`` + ``LIGHTBULB_TLS_KEY`` (HTTPS) or ``LIGHTBULB_TLS_SELF_SIGNED=1``.
Without a model the server still starts and answers with the reference's no-model replies.
"""
from __future__ import annotations

import argparse
import logging
import os
import sys


def build_state(model_path, engine_overrides=None, random_model=None, comm=None, rank=0,
                world=1, start_engine=True):
    from ..config import EngineConfig, SchedulerConfig, ServerConfig, get_preset
    from ..engine.async_engine import AsyncEngine
    from ..engine.llm_engine import LLMEngine
    from ..server.app import AppState
    from ..templates.chat_template import resolve_for_model
    sc = ServerConfig.from_env()
    engine = None
    template = None
    name = "lightbulb-default"
    if random_model:
        cfg = get_preset(random_model)
        ecfg = EngineConfig(scheduler=SchedulerConfig(max_model_len=sc.max_context))
        eng = LLMEngine.random_init(cfg, ecfg, comm=comm, tp_rank=rank, tp_size=world)
        engine = AsyncEngine(eng) if start_engine else eng
        name = random_model
        template = resolve_for_model(None, eng.tokenizer)
    elif model_path and os.path.exists(model_path):
        ecfg = EngineConfig(scheduler=SchedulerConfig(max_model_len=sc.max_context))
        eng = LLMEngine.from_pretrained(model_path, ecfg, comm=comm, tp_rank=rank, tp_size=world)
        engine = AsyncEngine(eng) if start_engine else eng
        template = resolve_for_model(model_path, eng.tokenizer)
        name = os.path.basename(os.path.normpath(model_path))
        logging.getLogger("lightbulb_b200").info("chat template resolved by %s",
                                                 template.resolved_by.value)
    return AppState(engine, template, model_name=name, database_url=sc.database_url), sc


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="lightbulb-serve")
    ap.add_argument("--model", default=None)
    ap.add_argument("--random-model", default=None, help="preset name: random-init weights")
    ap.add_argument("--bind", default=None)
    a = ap.parse_args(argv)
    logging.basicConfig(level=os.environ.get("LIGHTBULB_LOG", "INFO"))
    from ..config import ServerConfig
    sc = ServerConfig.from_env()
    model = a.model or os.path.join(sc.models_dir, sc.default_model)
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        return _serve_tp(a, model)
    state, sc = build_state(model, random_model=a.random_model)
    from ..server.app import create_app
    from ..server.tls import ssl_kwargs
    import uvicorn
    host, port = (a.bind or sc.bind_address).rsplit(":", 1)
    uvicorn.run(create_app(state), host=host, port=int(port), log_level="info",
                **ssl_kwargs(sc))
    return 0


def _serve_tp(a, model) -> int:
    """One process per GPU (torchrun): every rank holds its shard of the engine; rank 0 serves
    HTTP and drives the others through the control plane; a heartbeat watchdog over the
    process group's store turns a dead rank into 503s on rank 0."""
    import torch.distributed as dist
    from ..parallel.comm import TPComm, init_distributed
    from ..parallel.serving import ControlPlane, run_worker
    from ..parallel.watchdog import Watchdog, attach
    rank, world, _ = init_distributed(timeout_s=600)
    comm = TPComm()
    state, sc = build_state(model, random_model=a.random_model, comm=comm, rank=rank,
                            world=world, start_engine=(rank == 0))
    if state.engine is None:
        raise SystemExit("tensor-parallel serving needs --model or --random-model")
    plane = ControlPlane()
    store = dist.distributed_c10d._get_default_store()
    wd = Watchdog(store, rank, world).start()
    if rank != 0:
        try:
            run_worker(state.engine, plane)
        finally:
            wd.stop()
        return 0
    state.engine.attach_control_plane(plane)
    attach(state.engine, wd)
    from ..server.app import create_app
    from ..server.tls import ssl_kwargs
    import uvicorn
    host, port = (a.bind or sc.bind_address).rsplit(":", 1)
    try:
        uvicorn.run(create_app(state), host=host, port=int(port), log_level="info",
                    **ssl_kwargs(sc))
    finally:
        state.engine.shutdown()            # tells the workers to stop
        wd.stop()
    return 0


if __name__ == "__main__":
    sys.exit(main())
