"""The pushed exchange across real ranks: tests/push_ranks.py on two GPUs (or all, up to eight, with
PUSH_RANKS=all), one process each, NVLS off; skipped when fewer than two GPUs are visible."""

import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_pushed_exchange_across_gpus():
    """Two ranks, or every visible GPU up to eight with PUSH_RANKS=all."""
    gpus = torch.cuda.device_count()
    if gpus < 2:
        pytest.skip("needs two GPUs")
    ranks = min(gpus, 8) if os.environ.get("PUSH_RANKS") == "all" else 2
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(ranks), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "push_ranks.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0, (r.stdout[-3000:], r.stderr[-3000:])
    assert r.stdout.count("pushed exchange equals the all-gather") == ranks
