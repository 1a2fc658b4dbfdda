"""Tensor-parallel serving: rank 0 runs the HTTP server and the asynchronous engine, the other
ranks run the same engine without a front end and follow rank 0 step by step.

Every engine step is a collective (the sharded layers all-reduce), so all ranks must admit the
same requests in the same order and step together.  Rank 0 publishes, over a gloo group with a
long timeout (idle servers wait indefinitely), the adds and aborts it applies in each loop
iteration in which it applies any or steps; a worker applies the same list and steps iff its
engine has work, which is then exactly when rank 0 steps (identical state on every rank).
``None`` tells the workers to stop (shutdown, or rank 0's engine failed).

The reference runs tensor parallelism inside one process (``src/multi_gpu/``); here it is one
process per GPU, and this module is what keeps their schedulers identical.
"""
from __future__ import annotations

import datetime
import logging
from typing import Any, List, Optional

import torch.distributed as dist

log = logging.getLogger(__name__)


class ControlPlane:
    def __init__(self, timeout_s: float = 7 * 24 * 3600.0):
        # collective over every rank of the default group
        self.group = dist.new_group(backend="gloo",
                                    timeout=datetime.timedelta(seconds=timeout_s))
        self.rank = dist.get_rank()

    def publish(self, msgs: Optional[List[tuple]]) -> None:
        """Rank 0: send this iteration's submissions (``None`` = stop)."""
        obj: List[Any] = [msgs]
        dist.broadcast_object_list(obj, src=0, group=self.group)

    def receive(self) -> Optional[List[tuple]]:
        obj: List[Any] = [None]
        dist.broadcast_object_list(obj, src=0, group=self.group)
        return obj[0]


def run_worker(engine, plane: ControlPlane) -> int:
    """Follow rank 0 until it says stop; returns the number of steps taken."""
    steps = 0
    while True:
        msgs = plane.receive()
        if msgs is None:
            return steps
        for kind, payload in msgs:
            if kind == "add":
                rid, kw = payload
                try:
                    engine.add_request(request_id=rid, **kw)
                except Exception:      # rank 0 rejected the same request the same way
                    pass
            elif kind == "abort":
                engine.abort(payload)
                engine.release(payload)
        if engine.has_unfinished():
            for o in engine.step():
                if o.finished:
                    engine.release(o.request_id)      # mirrors rank 0's bookkeeping
            steps += 1
