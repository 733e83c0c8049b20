"""Shared fixtures. Tests marked `gpu` need a CUDA device (a B200) and call
the CUDA kernels through the C ABI; everything else runs on the CPU."""
from __future__ import annotations

import glob
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")
GOLDEN_NAMES = sorted(os.path.splitext(os.path.basename(p))[0]
                      for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU; calls the CUDA kernels through the C ABI")


def load_golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN_DIR, name + ".npz"), allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def golden_B(g: dict, k: int) -> np.ndarray:
    """The dense operand the fixture generator drew for SpMM width k."""
    rng = np.random.default_rng(11)
    for kk in g["spmm_ks"]:
        B = rng.uniform(-1.0, 1.0, size=(int(g["n"]), int(kk)))
        if int(kk) == k:
            return B
    raise KeyError(k)


def mixed_x(n: int, seed: int = 1234) -> np.ndarray:
    """x with magnitudes 1e-6..1e6 and random signs, the shape of the
    reference GPU test's make_x (tests/test_cuda_correctness.cpp:58-70)."""
    rng = np.random.default_rng(seed)
    sign = np.where(rng.random(n) < 0.5, -1.0, 1.0)
    return sign * 10.0 ** rng.uniform(-6.0, 6.0, size=n)


@pytest.fixture(scope="session")
def ctx():
    """A library context on device 0; fails loudly without a GPU."""
    import spmvbench_b200 as S
    if not S.gpu_available():
        pytest.fail("gpu-marked test run without a CUDA device")
    c = S.Context(0)
    yield c
    c.close()
