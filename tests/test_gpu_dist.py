"""Multi-GPU row-sharded iteration through NCCL (needs 2 GPUs; skipped on a
single-GPU box). Each rank runs tests/dist_worker.py."""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_iteration_matches_oracle():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    out = subprocess.run(["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                          "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
                          os.path.join(ROOT, "tests", "dist_worker.py")], env=env, capture_output=True, text=True,
                         timeout=400)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    assert out.stdout.count(": ok") == 12, out.stdout[-3000:]
