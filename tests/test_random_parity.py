"""Randomised host-side parity against the reference's own code (oracle/_ref).

Several hundred small matrices with adversarial structure - empty rows and
columns, m = 0 or n = 0, dense rows, unsorted columns, repeated (row, column)
entries, tails that cut 2x2 / 4x4 blocks - each checked for:
  * spmvb_compute_row_stats against compute_row_stats, every field bit for
    bit, and the histogram;
  * spmvb_choose_spmv_reference against choose_spmv on those statistics;
  * the oracle's csr_omp, spmm_csr_cpu, ELL and BCSR conversions and kernels
    against the reference's, bit for bit.
CPU only; skipped where oracle/_ref is absent.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import oracle
import spmvbench_b200 as S

pytestmark = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")


def random_csr(rng):
    m = int(rng.integers(0, 40))
    n = int(rng.integers(0, 50))
    kind = rng.integers(0, 4)
    if n == 0:
        lens = np.zeros(m, np.int64)
    elif kind == 0:   # uniform short rows
        lens = rng.integers(0, min(n, 6) + 1, m)
    elif kind == 1:   # skewed: a few long rows
        lens = np.where(rng.random(m) < 0.1, rng.integers(0, 3 * n + 1, m), rng.integers(0, 3, m))
    elif kind == 2:   # dense block rows
        lens = np.full(m, n)
    else:             # many empty rows
        lens = np.where(rng.random(m) < 0.6, 0, rng.integers(1, n + 1, m))
    rowptr = np.zeros(m + 1, np.int32)
    rowptr[1:] = np.cumsum(lens)
    nnz = int(rowptr[-1])
    colind = rng.integers(0, max(n, 1), nnz).astype(np.int32) if n else np.zeros(0, np.int32)
    values = rng.uniform(-1, 1, nnz)
    if kind == 2 and n:   # keep dense rows sorted and distinct where they fit
        for i in range(m):
            s, e = rowptr[i], rowptr[i + 1]
            if e - s <= n:
                colind[s:e] = rng.permutation(n)[: e - s] if rng.random() < 0.5 else np.arange(e - s)
    return m, n, rowptr, colind, values


def ref_stats(m, n, rp, ci):
    st = np.zeros(13)
    mx = int(np.diff(rp).max()) if m else 0
    hist = np.zeros(mx + 1, np.int64)
    nnz = int(rp[m]) if m else 0
    oracle.ref().ref_row_stats(oracle._p(rp), oracle._p(ci) if nnz else None, m, n, nnz, oracle._p(st),
                               oracle._p(hist), hist.size)
    return st, hist


def ref_choice(st):
    out = np.zeros(4, np.int32)
    reason = C.create_string_buffer(512)
    oracle.ref().ref_choose_spmv(oracle._p(st), oracle._p(out), reason, 512)
    return out.tolist()


@pytest.mark.parametrize("seed", range(12))
def test_random_matrices_match_reference(seed):
    rng = np.random.default_rng(1000 + seed)
    lib = oracle.ref()
    for _ in range(30):
        m, n, rp, ci, va = random_csr(rng)
        nnz = int(rp[m]) if m else 0
        A = S.CsrMatrix(m, n, rp, ci, va)
        st, hist = ref_stats(m, n, rp, ci)
        mine = S.row_stats(A, histogram=True)
        np.testing.assert_array_equal(np.array([mine[f] for f in oracle.STAT_FIELDS]), st)
        if m:
            np.testing.assert_array_equal(mine["row_nnz_histogram"], hist)
        got = S.choose_spmv_reference(mine)
        assert [got["kernel"], got["lanes"], got["block_r"], got["block_c"]] == ref_choice(st)
        if nnz == 0 or n == 0:
            continue
        x = rng.uniform(-1, 1, n)
        R = oracle.RefCsr(m, n, rp, ci, va)
        np.testing.assert_array_equal(oracle.spmv_csr(m, rp, ci, va, x, np.float64), R.spmv(x))
        k = int(rng.integers(1, 9))
        B = rng.uniform(-1, 1, (n, k))
        np.testing.assert_array_equal(oracle.spmm_csr(m, k, rp, ci, va, B, np.float64), R.spmm(B, k))
        w, ecol, ev, rl = oracle.csr_to_ell(m, rp, ci, va)
        assert w == lib.ref_ell_width_d(R.h)
        recol = np.zeros(max(m * w, 1), np.int32)
        rev = np.zeros(max(m * w, 1), np.float64)
        rrl = np.zeros(max(m, 1), np.int32)
        lib.ref_csr_to_ell_d(R.h, oracle._p(recol), oracle._p(rev), oracle._p(rrl))
        np.testing.assert_array_equal(ecol, recol[:m * w])
        np.testing.assert_array_equal(ev, rev[:m * w])
        np.testing.assert_array_equal(rl, rrl[:m])
        for b in (2, 4):
            brp, bci, bva = oracle.csr_to_bcsr(m, n, b, rp, ci, va)
            mb, bn = C.c_int32(), C.c_int64()
            lib.ref_bcsr_shape_d(R.h, b, C.byref(mb), C.byref(bn))
            rbrp = np.zeros(mb.value + 1, np.int32)
            rbci = np.zeros(max(bn.value, 1), np.int32)
            rbva = np.zeros(max(bn.value, 1) * b * b, np.float64)
            lib.ref_csr_to_bcsr_d(R.h, b, oracle._p(rbrp), oracle._p(rbci), oracle._p(rbva))
            np.testing.assert_array_equal(brp, rbrp)
            np.testing.assert_array_equal(bci, rbci[:bn.value])
            np.testing.assert_array_equal(bva, rbva[:bn.value * b * b])
            yb = np.empty(m)
            lib.ref_spmv_bcsr_dd(R.h, b, oracle._p(x), oracle._p(yb), 0)
            np.testing.assert_array_equal(oracle.spmv_bcsr(m, n, b, b, brp, bci, bva, x, np.float64), yb)
        R.close()
