"""The command-line driver (spmvbench_b200/driver.py): --stats on the CPU,
--validate / --auto / --profile on the GPU."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

from conftest import ROOT


def run(*args, timeout=900):
    return subprocess.run([sys.executable, "-m", "spmvbench_b200.driver", *args], cwd=ROOT, capture_output=True,
                          text=True, timeout=timeout)


def test_stats_runs_without_a_gpu():
    out = run("--stats", "--workload", "1", "4")
    assert out.returncode == 0, out.stderr
    assert "banded_100k_hb4" in out.stdout and "dense_share_of_stored_4x4=1" in out.stdout


@pytest.mark.gpu
def test_validate_all_workloads(tmp_path):
    out = run("--validate")
    assert out.returncode == 0, out.stdout + out.stderr
    assert "validate: ok" in out.stdout


@pytest.mark.gpu
def test_auto_and_profile(tmp_path):
    out = run("--auto", "--workload", "1", "--iters", "5", "--warmup", "2")
    assert out.returncode == 0, out.stdout + out.stderr
    assert "heuristic-vs-oracle" in out.stdout
    out = run("--profile", "ell", "--workload", "1", "--steps", "2")
    assert out.returncode == 0 and "per launch" in out.stdout, out.stdout + out.stderr
    out = run("--profile", "spmm", "--workload", "1", "--k", "16", "--steps", "2")
    assert out.returncode == 0 and "per launch" in out.stdout, out.stdout + out.stderr


@pytest.mark.gpu
def test_spmm_timings(tmp_path):
    out = run("--spmm", "--k", "8", "--iters", "3", "--warmup", "1", "--dtype", "f32")
    assert out.returncode == 0, out.stdout + out.stderr
    assert out.stdout.count("GFLOP/s") == 6 and "wrote results/spmm.csv" in out.stdout
