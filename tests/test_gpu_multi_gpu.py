"""The slot-sharded RepEncoder on 2 (and, where the box has them, 4) GPUs,
one process per GPU over NCCL, each rank checked against the oracle and the
single-GPU forward (tests/multi_gpu_worker.py).  Skipped with fewer GPUs."""

import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_slot_sharded_ranks_against_oracle(cuda_device, world):
    import torch

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", OMP_NUM_THREADS="4")
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "multi_gpu_worker.py")]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=500)
    lines = [json.loads(l) for l in res.stdout.splitlines() if l.startswith("{")]
    assert res.returncode == 0, res.stdout[-4000:] + res.stderr[-4000:]
    assert sorted(l["rank"] for l in lines) == list(range(world))
    assert all(l["ok"] for l in lines), lines
    assert sum(l["items"] for l in lines) > 0
