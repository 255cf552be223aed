"""Fused GEMM + all-gather across real GPUs (2 or more): runs
tests/mgpu_peer_worker.py with one process per GPU under
torch.distributed.run.  Skipped with fewer than two GPUs."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_sharded_gemm_multi_gpu():
    world = min(torch.cuda.device_count(), 8)
    root = Path(__file__).resolve().parent.parent
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           str(root / "tests" / "mgpu_peer_worker.py")]
    res = subprocess.run(cmd, cwd=root, env=env, capture_output=True, text=True)
    out = res.stdout + res.stderr
    assert res.returncode == 0, out[-4000:]
    assert "PEER_MGPU OK" in out, out[-4000:]
