"""SpMM parity on the GPU: tiles 16/32/64, uniform and bucketed, every
(T, Acc) pair. The tiled kernel keeps spmm_csr_cpu's per-column summation
order, so it must match the reference's own Y bit for bit; the bucketed
variant splits rows longer than 64 entries across warps and is held to the
gamma_n bound on those rows."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import spmvbench_b200 as S
from conftest import GOLDEN_NAMES, golden_B, load_golden
from gpu_util import DTYPE_PAIRS, NP, TOL, TORCH, assert_bitwise

pytestmark = pytest.mark.gpu


def run_spmm(M, B, k, tile, bucketed, acc=None):
    acc = M.dtype if acc is None else acc
    Bt = torch.from_numpy(np.ascontiguousarray(B, NP[M.dtype])).cuda()
    Yt = torch.full((max(M.m, 1), max(k, 1)), float("nan"), dtype=TORCH[acc], device="cuda")
    M.spmm(Bt, Yt, k, tile=tile, bucketed=bucketed, acc=acc)
    torch.cuda.synchronize()
    return Yt.cpu().numpy()[:M.m, :k]


def check_spmm(A, B, k, dtype, acc, got, label):
    vals = np.ascontiguousarray(A.values, NP[dtype])
    Bc = np.ascontiguousarray(B, NP[dtype])
    ref = oracle.spmm_csr(A.m, k, A.rowptr, A.colind, vals, Bc, NP[acc])
    lens = np.diff(A.rowptr)
    short = lens <= 64
    assert_bitwise(ref[short], got[short], label + " (rows <= 64)")
    if (~short).any():
        r, where = oracle.gamma_ratio_spmm(A.rowptr, A.colind, vals, Bc, k, ref, got, NP[acc])
        rel = np.abs(got - ref) <= TOL[acc] * np.abs(ref)
        assert r <= 1.0 or rel[where], f"{label}: gamma ratio {r} at {where}"


@pytest.mark.parametrize("name", GOLDEN_NAMES)
@pytest.mark.parametrize("dtype,acc", DTYPE_PAIRS)
def test_golden_spmm(ctx, name, dtype, acc):
    g = load_golden(name)
    A = S.CsrMatrix(int(g["m"]), int(g["n"]), g["rowptr"], g["colind"], g["values"])
    M = S.DeviceMatrix(ctx, A, dtype)
    for k in g["spmm_ks"]:
        k = int(k)
        B = golden_B(g, k)
        for tile in (16, 32, 64):
            for bucketed in (False, True):
                got = run_spmm(M, B, k, tile, bucketed, acc)
                check_spmm(A, B, k, dtype, acc, got, f"{name} k={k} t={tile} b={bucketed}")
                if not bucketed and dtype == S.F64:
                    assert_bitwise(g[f"Y{k}_dd"], got, f"{name} vs reference Y")
                if not bucketed and dtype == S.F32 and acc == S.F32:
                    assert_bitwise(g[f"Y{k}_ff"], got, f"{name} vs reference Y")


@pytest.mark.parametrize("k", [1, 15, 16, 33, 64, 65, 100])
def test_k_edges(ctx, k):
    A = S.generate(3, seed=61, scale_rows=20000)
    B = S.generate_vector(62, A.n * k).reshape(A.n, k)
    for dtype, acc in DTYPE_PAIRS:
        M = S.DeviceMatrix(ctx, A, dtype)
        for tile in (16, 32, 64):
            for bucketed in (False, True):
                check_spmm(A, B, k, dtype, acc, run_spmm(M, B, k, tile, bucketed, acc),
                           f"k={k} t={tile} b={bucketed} {dtype}/{acc}")


@pytest.mark.parametrize("dtype,acc", DTYPE_PAIRS)
def test_spmm_workload_scaled(ctx, dtype, acc):
    A = S.generate(5, seed=63, scale_rows=100000)
    k = 64
    B = S.generate_vector(64, A.n * k).reshape(A.n, k)
    M = S.DeviceMatrix(ctx, A, dtype)
    for tile in (16, 32, 64):
        for bucketed in (False, True):
            check_spmm(A, B, k, dtype, acc, run_spmm(M, B, k, tile, bucketed, acc), f"C5 t={tile} b={bucketed}")


def test_spmm_full_size_fp64(ctx):
    A = S.generate(5, seed=65)
    k = 64
    B = S.generate_vector(66, A.n * k).reshape(A.n, k)
    M = S.DeviceMatrix(ctx, A, S.F64)
    ref = oracle.spmm_csr(A.m, k, A.rowptr, A.colind, A.values, B, np.float64)
    assert_bitwise(ref, run_spmm(M, B, k, 64, False), "C5 full t=64")
    Y = M.spmm_host(B, k, tile=64)
    assert_bitwise(ref, Y, "C5 full host entry")


def test_spmm_full_size_fp32(ctx):
    """The k = 64 SpMM workload (uniform 1M x 1M, 16 nnz/row) in fp32: Y equals
    spmm_csr_cpu's fp32 output bit for bit, on the device and host entries."""
    A = S.generate(5, seed=67)
    k = 64
    B = S.generate_vector(68, A.n * k).reshape(A.n, k).astype(np.float32)
    M = S.DeviceMatrix(ctx, A, S.F32)
    vals = np.ascontiguousarray(A.values, np.float32)
    ref = oracle.spmm_csr(A.m, k, A.rowptr, A.colind, vals, B, np.float32)
    assert_bitwise(ref, run_spmm(M, B, k, 64, False), "C5 fp32 full t=64")
    assert_bitwise(ref, run_spmm(M, B, k, 32, False), "C5 fp32 full t=32")


def test_spmm_with_more_elements_than_int32(ctx):
    """Y and X of 600,000 x 4,096 fp64 (2.46e9 elements, 19.7 GB each): the
    element offsets row * k pass 2^31 from row 524,288 on, so X and Y are
    addressed with 64-bit offsets. X is built on the device from exact
    binary fractions; the last 2,000 rows of Y equal spmm_csr_cpu's order
    (0 + a0*X[c0] + a1*X[c1], each step rounded) bit for bit."""
    import torch
    free, _ = torch.cuda.mem_get_info()
    if free < 60e9:
        pytest.skip("needs 60 GB of free device memory")
    m = n = 600_000
    k = 4096
    rng = np.random.default_rng(73)
    colind = np.sort(rng.integers(0, n, (m, 2), dtype=np.int32), axis=1).ravel()
    rowptr = (np.arange(m + 1, dtype=np.int64) * 2).astype(np.int32)
    values = rng.standard_normal(2 * m)
    A = S.CsrMatrix(m, n, rowptr, colind, values)
    M = S.DeviceMatrix(ctx, A, S.F64)
    X = torch.arange(n * k, dtype=torch.float64, device="cuda").remainder_(1021).sub_(510).mul_(2.0 ** -7)
    X = X.view(n, k)
    Y = torch.full((m, k), float("nan"), dtype=torch.float64, device="cuda")
    for tile in (64, 32):
        M.spmm(X, Y, k, tile=tile, bucketed=False)
        torch.cuda.synchronize()
        r0 = m - 2000
        got = Y[r0:].cpu().numpy()
        cols = torch.from_numpy(colind[2 * r0:].astype(np.int64)).cuda()
        xr = X.index_select(0, cols).cpu().numpy().reshape(2000, 2, k)
        a = values[2 * r0:].reshape(2000, 2, 1)
        ref = (np.zeros((2000, k)) + a[:, 0] * xr[:, 0]) + a[:, 1] * xr[:, 1]
        assert_bitwise(ref, got, f"rows past 2^31 elements, tile {tile}")
    M.close()
    del X, Y
    torch.cuda.empty_cache()


@pytest.mark.parametrize("bands", ["2", "3", "5", "8"])
@pytest.mark.parametrize("dtype,acc", DTYPE_PAIRS)
def test_spmm_column_band_sweep_is_bit_identical(ctx, bands, dtype, acc):
    """The plain SpMM swept in column bands (spmvb_matrix_set_spmm_bands): each output
    element still gets its terms in CSR order, so Y equals spmm_csr_cpu bit
    for bit; rows with no entry in a band, empty rows, a long row and an
    unsorted row (which sends the matrix back to the one-pass kernel) are
    covered, and a rerun with a different band count reuses nothing stale."""
    bands = int(bands)
    A = S.generate(2, seed=71, scale_rows=30000)
    k = 64
    B = S.generate_vector(72, A.n * k).reshape(A.n, k)
    M = S.DeviceMatrix(ctx, A, dtype)
    M.set_spmm_bands(bands)
    vals = np.ascontiguousarray(A.values, NP[dtype])
    ref = oracle.spmm_csr(A.m, k, A.rowptr, A.colind, vals, np.ascontiguousarray(B, NP[dtype]), NP[acc])
    assert_bitwise(ref, run_spmm(M, B, k, 64, False, acc), f"bands {bands}")
    M.set_spmm_bands(4)
    assert_bitwise(ref, run_spmm(M, B, k, 64, False, acc), "bands 4 after another count")
    M.close()
    # Empty rows, a 3,000-entry row and one unsorted row.
    rng = np.random.default_rng(73)
    n = 9000
    rows = [[] if i % 7 == 0 else sorted(rng.choice(n, size=int(rng.integers(1, 30)), replace=False).tolist())
            for i in range(2000)]
    rows[5] = sorted(rng.choice(n, size=3000, replace=False).tolist())
    for unsorted in (False, True):
        rr = [list(r) for r in rows]
        if unsorted:
            rr[9] = rr[9][::-1] if len(rr[9]) > 1 else [3, 1]
        rp = np.zeros(len(rr) + 1, np.int32)
        rp[1:] = np.cumsum([len(r) for r in rr])
        ci = np.array([c for r in rr for c in r], np.int32)
        C = S.CsrMatrix(len(rr), n, rp, ci, rng.uniform(-1, 1, ci.size))
        Bc = rng.uniform(-1, 1, (n, k))
        MC = S.DeviceMatrix(ctx, C, dtype)
        cv = np.ascontiguousarray(C.values, NP[dtype])
        refc = oracle.spmm_csr(C.m, k, C.rowptr, C.colind, cv, np.ascontiguousarray(Bc, NP[dtype]), NP[acc])
        MC.set_spmm_bands(bands)
        assert_bitwise(refc, run_spmm(MC, Bc, k, 64, False, acc), f"skewed bands {bands} unsorted={unsorted}")
        MC.close()
