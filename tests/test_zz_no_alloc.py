"""The merge-path SpMV entry point that allocates nothing.

Some callers cannot call cudaMalloc: their device memory belongs to another
allocator (a framework's caching allocator, a pool sized at start-up), or
their latency rules forbid allocating after start-up because cudaMalloc and
cudaFree can synchronize the device. spmvb_spmv_merge_noalloc serves them:
the caller passes its own device arrays and the kernels' scratch sits in a
fixed device array inside the library. This test calls it through the C ABI
twice in a row on caller-owned buffers and checks each result against the
oracle (csr_omp restated on the CPU) and against the existing merge-path
entry point (spmvb_spmv, SPMVB_CSR_MERGE), within the tolerance every GPU
parity test here uses. One case fills the fixed scratch almost to its limit
(65,458 of 65,536 tiles), so the last tile start and carry sit near the end
of the array. It runs last (file name), and passes alone in a fresh process
or after the other tests.
"""
from __future__ import annotations

import ctypes as C

import pytest
import torch

import spmvbench_b200 as S
from gpu_util import NP, TORCH, assert_rows_within_bound, oracle_y, run_spmv

pytestmark = pytest.mark.gpu


def _noalloc(A, dev, x, y, dtype, acc):
    lib = S.load()
    return lib.spmvb_spmv_merge_noalloc(dtype, A.m, A.n, A.nnz, C.c_void_p(dev["rowptr"].data_ptr()),
                                        C.c_void_p(dev["colind"].data_ptr()),
                                        C.c_void_p(dev["values"].data_ptr()), C.c_void_p(x.data_ptr()),
                                        C.c_void_p(y.data_ptr()), acc,
                                        C.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("which,rows,dtype,acc", [(3, 300000, S.F64, S.F64), (2, 200000, S.F32, S.F32),
                                                  (1, 0, S.F32, S.F64)])
def test_noalloc_merge_matches_existing_entry_point(which, rows, dtype, acc):
    ctx = S.Context(0)
    A = S.generate(which, seed=81, scale_rows=rows)
    dev = {"rowptr": torch.from_numpy(A.rowptr.copy()).cuda(),
           "colind": torch.from_numpy(A.colind.copy()).cuda(),
           "values": torch.from_numpy(A.values.astype(NP[dtype])).cuda()}
    M = S.DeviceMatrix(ctx, A, dtype)
    for call in range(2):  # two calls in a row share the scratch array
        xh = S.generate_vector(82 + call, A.n)
        x = torch.from_numpy(xh.astype(NP[dtype])).cuda()
        y = torch.full((A.m,), float("nan"), dtype=TORCH[acc], device="cuda")
        assert _noalloc(A, dev, x, y, dtype, acc) == 0, S.load().spmvb_last_error()
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        assert_rows_within_bound(A, xh, oracle_y(A, xh, dtype, acc), got, dtype, acc, f"no-alloc call {call} vs oracle")
        ref = run_spmv(M, xh, S.CSR_MERGE, acc=acc)
        assert_rows_within_bound(A, xh, ref, got, dtype, acc, f"no-alloc call {call} vs SPMVB_CSR_MERGE")
    M.close()
    ctx.close()


def test_noalloc_near_the_scratch_limit():
    """m + nnz = 117,300,000 (6.9M rows of 16 entries): 65,458 merge tiles of
    the 65,536 the fixed scratch holds, two calls in a row, each within the
    gamma_n bound of the oracle."""
    import numpy as np

    import oracle
    ctx = S.Context(0)
    A = S.generate(2, seed=83, scale_rows=6_900_000)
    assert A.m + A.nnz == 117_300_000
    dev = {"rowptr": torch.from_numpy(A.rowptr).cuda(), "colind": torch.from_numpy(A.colind).cuda(),
           "values": torch.from_numpy(A.values).cuda()}
    for call in range(2):
        xh = S.generate_vector(84 + call, A.n)
        x = torch.from_numpy(xh).cuda()
        y = torch.full((A.m,), float("nan"), dtype=torch.float64, device="cuda")
        assert _noalloc(A, dev, x, y, S.F64, S.F64) == 0, S.load().spmvb_last_error()
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        assert not np.isnan(got).any(), f"call {call}: unwritten rows"
        ref = oracle.spmv_csr(A.m, A.rowptr, A.colind, A.values, xh, np.float64)
        r, row = oracle.gamma_ratio(A.rowptr, A.colind, A.values, xh, ref, got, np.float64)
        assert r <= 1.0, f"call {call}: row {row} outside the gamma_n bound (ratio {r})"
    del dev
    ctx.close()


def test_noalloc_rejects_oversize_request():
    lib = S.load()
    y = torch.zeros(4, dtype=torch.float64, device="cuda")
    # m + nnz beyond the fixed scratch: refused before anything is read
    st = lib.spmvb_spmv_merge_noalloc(S.F64, 100_000_000, 10, 50_000_000, C.c_void_p(y.data_ptr()),
                                      C.c_void_p(y.data_ptr()), C.c_void_p(y.data_ptr()),
                                      C.c_void_p(y.data_ptr()), C.c_void_p(y.data_ptr()), S.F64, None)
    assert st == 3 and b"no-allocation limit" in lib.spmvb_last_error()
