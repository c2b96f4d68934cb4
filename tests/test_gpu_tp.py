"""KV-head tensor-parallel WCA on 2 GPUs: ``ShardedWCAState`` (per-rank head
shards, row sums all-reduced over NCCL) against the unsharded ``WCAState``.
Runs tests/tp_worker.py as 2 ranks; skipped with fewer than 2 GPUs."""

from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

HERE = Path(__file__).resolve().parent


@pytest.mark.gpu
def test_sharded_wca_matches_the_unsharded_state_on_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node",
           "2", "--master-addr", "127.0.0.1", "--master-port", str(port),
           str(HERE / "tp_worker.py")]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "selections agree" in res.stdout
