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
