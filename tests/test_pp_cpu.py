"""Pipeline parallelism on CPU ranks (gloo): stages on separate processes, micro-batches in
flight, greedy tokens identical to the fp32 oracle."""
import os
import socket
import subprocess
import sys

import pytest

from lightbulb_b200.parallel.pp import HybridConfig, split_layers


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_split_layers_and_hybrid_layout():
    assert split_layers(32, 3) == [(0, 10), (10, 20), (20, 32)]   # last stage: remainder
    assert split_layers(80, 8)[-1] == (70, 80)
    h = HybridConfig(tensor_world_size=4, pipeline_stages=2)
    assert h.world() == 8 and h.coords(5) == (1, 1) and h.stage_group_ranks(1) == [4, 5, 6, 7]


@pytest.mark.parametrize("world,mb", [(2, 2), (3, 1)])
def test_pipeline_matches_oracle(world, mb):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="2")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           f"--master-port={_free_port()}", "-m", "lightbulb_b200.parallel.pp",
           "--micro-batches", str(mb), "--tokens", "5"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=240)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert r.stdout.count("pp [") == 3
