"""Multi-GPU checks (one process per GPU under torchrun, NCCL + CUDA IPC peer memory).

Skipped unless the box has at least two GPUs.  Each check is a module's self-check entry point,
run as child processes with a process-group timeout and an outer time limit."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _ngpus() -> int:
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _torchrun(module: str, *args: str, n: int = 2, port: int = 29631) -> subprocess.CompletedProcess:
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={n}", "--master-addr", "127.0.0.1",
           "--master-port", str(port), "-m", module, *args]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    return subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)


@pytest.mark.skipif(_ngpus() < 2, reason="needs 2 GPUs")
def test_p2p_allreduce_two_ranks():
    r = _torchrun("lightbulb_b200.parallel.allreduce", port=29631)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "ok" in r.stdout


@pytest.mark.skipif(_ngpus() < 2, reason="needs 2 GPUs")
def test_rowpar_exchange_two_ranks():
    r = _torchrun("lightbulb_b200.parallel.rowpar", port=29633)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "ok" in r.stdout


@pytest.mark.skipif(_ngpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("comm", ["p2p", "allreduce", "nccl"])
def test_tp2_generation_matches_oracle(comm):
    r = _torchrun("lightbulb_b200.parallel.tp_check", "--comm", comm, port=29632)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
