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
    assert out.stdout.count(": ok") == 20, out.stdout[-3000:]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_wait_gives_up_when_a_rank_skips_a_step():
    """Failure detection over peer memory without a GPU fault: a rank that
    skips a step makes the other rank's bounded barrier wait give up after
    one second with SPMVB_ERR_TIMEOUT (status 7), and both ranks close
    cleanly."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", SPMVB_PEER_TIMEOUT_MS="1000")
    out = subprocess.run(["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                          "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
                          os.path.join(ROOT, "tests", "dist_worker.py"), "peer-timeout"], env=env,
                         capture_output=True, text=True, timeout=400)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    assert "rank 0 status 7" in out.stdout
