"""Helpers for the GPU parity tests: run a kernel through the C ABI and
compare with the oracle.

Tolerance (stated once, used everywhere): a row passes when
    |y_gpu - y_ref| <= max(tol * |y_ref|, 2 * gamma_n(u) * sum_j |a_ij x_j|)
with tol = 1e-12 (fp64 accumulation) or 1e-5 (fp32), n = the row's length,
gamma_n = n*u / (1 - n*u), u = 2^-53 or 2^-24: the per-row relative bound
set for this path, widened to the reference GPU test's own gamma_n criterion
(tests/test_cuda_correctness.cpp:1-11,53-56,88) for rows where cancellation
makes |y| tiny. Kernels that keep csr_omp's summation order must match
bit for bit instead."""
from __future__ import annotations

import numpy as np
import torch

import oracle
import spmvbench_b200 as S

NP = {S.F64: np.float64, S.F32: np.float32}
TORCH = {S.F64: torch.float64, S.F32: torch.float32}
DTYPE_PAIRS = [(S.F64, S.F64), (S.F32, S.F32), (S.F32, S.F64)]
TOL = {S.F64: 1e-12, S.F32: 1e-5}


def run_spmv(M: S.DeviceMatrix, x: np.ndarray, kernel: int, lanes: int = 4, block: int = 4,
             acc: int | None = None) -> np.ndarray:
    acc = M.dtype if acc is None else acc
    xt = torch.from_numpy(np.ascontiguousarray(x, NP[M.dtype])).cuda()
    yt = torch.full((max(M.m, 1),), float("nan"), dtype=TORCH[acc], device="cuda")
    M.spmv(xt, yt, kernel=kernel, lanes=lanes, block=block, acc=acc)
    torch.cuda.synchronize()
    return yt.cpu().numpy()[:M.m]


def oracle_y(A: S.CsrMatrix, x: np.ndarray, dtype: int, acc: int) -> np.ndarray:
    return oracle.spmv_csr(A.m, A.rowptr, A.colind, np.ascontiguousarray(A.values, NP[dtype]),
                           np.ascontiguousarray(x, NP[dtype]), NP[acc])


def assert_rows_within_bound(A: S.CsrMatrix, x, ref, got, dtype: int, acc: int, label: str = ""):
    assert got.shape == ref.shape
    assert not np.isnan(got).any(), f"{label}: unwritten rows"
    m = A.m
    if m == 0:
        return
    vals = np.ascontiguousarray(A.values, NP[dtype]).astype(np.float64)
    xx = np.ascontiguousarray(x, NP[dtype]).astype(np.float64)
    u = 2.0 ** -53 if acc == S.F64 else 2.0 ** -24
    lens = np.diff(A.rowptr).astype(np.int64)
    rows = np.repeat(np.arange(m), lens)
    abs_sum = np.bincount(rows, weights=np.abs(vals * xx[A.colind]), minlength=m)
    nu = lens * u
    gamma_bound = 2.0 * (nu / (1.0 - nu)) * abs_sum
    diff = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    allowed = np.maximum(TOL[acc] * np.abs(ref.astype(np.float64)), gamma_bound)
    bad = np.flatnonzero(diff > allowed)
    assert bad.size == 0, (f"{label}: {bad.size} rows out of bound, first row {bad[0]}: "
                           f"|d|={diff[bad[0]]:.3e} allowed={allowed[bad[0]]:.3e}")


def assert_bitwise(ref, got, label: str = ""):
    assert got.shape == ref.shape
    if not np.array_equal(got, ref):
        d = np.flatnonzero(got != ref)
        raise AssertionError(f"{label}: {d.size} entries differ, first {d[0]}: {got[d[0]]!r} vs {ref[d[0]]!r}")
