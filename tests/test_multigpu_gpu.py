"""Multi-GPU gathers on device memory (one process per GPU): the copy-engine
gather into rank 0's HBM (PeerGather) and the NCCL point-to-point gather
(gather_to_root), each checked against the CPU oracle.  Needs two or more
visible GPUs; skipped otherwise."""

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _gpus() -> int:
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(_gpus() < 2, reason="needs two or more GPUs")
def test_peer_gather_and_nccl_gather_match_oracle():
    n = min(_gpus(), 8)
    env = dict(os.environ)
    env["NCCL_DEBUG"] = "WARN"
    env["NCCL_NVLS_ENABLE"] = "0"
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(ROOT / "tests" / "multigpu_worker.py")]
    out = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT, timeout=660)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-4000:]
    line = [l for l in out.stdout.splitlines() if l.startswith("{")][-1]
    res = json.loads(line)
    assert res["world"] == n
    assert res["ok"], res
