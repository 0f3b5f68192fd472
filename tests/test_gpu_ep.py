"""Expert parallelism on all visible GPUs (NCCL), bit-exact against one GPU.

Needs 2+ GPUs; launched as a torchrun job on 127.0.0.1 with a short NCCL
timeout and an outer process timeout, so a rank that fails ends the job
instead of hanging it.
"""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2+ GPUs")
def test_ep_matches_single_gpu(tmp_path):
    n = min(torch.cuda.device_count(), 8)
    out = tmp_path / "ep.txt"
    here = os.path.dirname(os.path.abspath(__file__))
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={n}", "--master-addr", "127.0.0.1",
           "--master-port", str(_port()), os.path.join(here, "ep_worker_gpu.py"), str(out)]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    res = subprocess.run(cmd, env=env, capture_output=True, text=True)
    lines = out.read_text().splitlines() if out.exists() else []
    assert res.returncode == 0, res.stderr[-3000:] + "\n" + "\n".join(lines)
    assert len(lines) == n and all(" OK " in l for l in lines), "\n".join(lines)
