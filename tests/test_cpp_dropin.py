"""The C++ drop-in API (include/spmvbench: CsrMatrix, csr_to_ell,
csr_to_bcsr, compute_row_stats, choose_spmv, SpmvRunner, spmm_csr_tiled_*)
exercised by a C++ program written like the reference's own tests
(tests/cpp/dropin_test.cpp), built against libspmvb.so."""
from __future__ import annotations

import os
import subprocess

import pytest

from conftest import ROOT

BIN = os.path.join(ROOT, "_build", "tests", "dropin_test")


def _build():
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "tests", "cpp")], check=True)


def test_dropin_cpu_cases():
    _build()
    out = subprocess.run([BIN, "cpu"], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert " 0 failed" in out.stdout


@pytest.mark.gpu
def test_dropin_gpu_cases():
    _build()
    out = subprocess.run([BIN, "gpu"], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stdout + out.stderr
    assert " 0 failed" in out.stdout
