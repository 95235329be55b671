"""Multi-GPU parity (needs >= 2 visible GPUs; skipped otherwise).

Runs ``tests/multigpu_worker.py`` under torchrun with one process per GPU
(NCCL), which checks context-parallel decode (eager and CUDA-graph replay
with the all-gather inside the graph) and batch / KV-head sharding against
the single-GPU result.
"""
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs at least 2 GPUs")
@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_decode_matches_single_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), str(ROOT / "tests" / "multigpu_worker.py")]
    proc = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=300)
    lines = [l for l in proc.stdout.splitlines() if l.startswith("{")]
    assert proc.returncode == 0 and lines, proc.stdout[-2000:] + proc.stderr[-4000:]
    report = json.loads(lines[-1])
    assert report["all_ranks_ok"], report
