"""The reference's own benchmark matrices, end to end on the host.

banded_100k, uniform_random and powerlaw_skew are written by the reference's
generator (tools/gen_matrices.py, imported from the SpMVBench tree and pointed
at a temporary data directory) and read back. On each:
  * spmvb_read_matrix_market gives the CSR of the reference's
    read_matrix_market (oracle/_ref, compiled from the same tree), bit for bit;
  * spmvb_compute_row_stats equals the reference's compute_row_stats and
    spmvb_choose_spmv_reference picks what its choose_spmv picks;
  * the oracle's csr_omp equals the reference's csr_omp, and the reference's
    validate gate holds: csr_omp equals SciPy's y = A x for tools/reference.py's
    x (max_rel 0);
  * the oracle's BCSR (and, where it fits, ELL) conversions equal the
    reference's.
CPU only; skipped where the reference tree or oracle/_ref is absent.
"""
from __future__ import annotations

import importlib.util
import os

import numpy as np
import pytest

import oracle
import spmvbench_b200 as S

REF = oracle.reference_tree() or ""

pytestmark = pytest.mark.skipif(
    not (oracle.ref_available() and os.path.exists(os.path.join(REF, "tools", "gen_matrices.py"))),
    reason="the reference tree or oracle/_ref is absent")


def _ref_module(name, rel):
    spec = importlib.util.spec_from_file_location(name, os.path.join(REF, rel))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def ref_files(tmp_path_factory):
    gen = _ref_module("spmvbench_gen_matrices_t", "tools/gen_matrices.py")
    gen.DATA_DIR = str(tmp_path_factory.mktemp("data"))
    return {"banded_100k": gen.gen_banded_100k(), "uniform_random": gen.gen_uniform_random(),
            "powerlaw_skew": gen.gen_powerlaw_skew()}


@pytest.mark.parametrize("name", ["banded_100k", "uniform_random", "powerlaw_skew"])
def test_reference_matrix_end_to_end(ref_files, name):
    path = ref_files[name]
    m, n, rp, ci, va = oracle.ref_read_matrix_market(path)
    A = S.read_matrix_market(path)
    assert (A.m, A.n) == (m, n)
    np.testing.assert_array_equal(A.rowptr, rp)
    np.testing.assert_array_equal(A.colind, ci)
    np.testing.assert_array_equal(A.values, va)

    mine = S.row_stats(A, histogram=True)
    st = np.zeros(13)
    oracle.ref().ref_row_stats(oracle._p(rp), oracle._p(ci), m, n, int(rp[m]), oracle._p(st), None, 0)
    np.testing.assert_array_equal(np.array([mine[f] for f in oracle.STAT_FIELDS]), st)
    ref_choice = oracle.choose_spmv(dict(zip(oracle.STAT_FIELDS, st.tolist())))
    got = S.choose_spmv_reference(mine)
    assert [got[k] for k in ("kernel", "lanes", "block_r", "block_c")] == \
           [ref_choice[k] for k in ("kernel", "lanes", "block_r", "block_c")]

    x = _ref_module("spmvbench_reference_t", "tools/reference.py").make_x(n)
    R = oracle.RefCsr(m, n, rp, ci, va)
    y = oracle.spmv_csr(m, rp, ci, va, x, np.float64)
    np.testing.assert_array_equal(y, R.spmv(x))
    import scipy.sparse as sp
    np.testing.assert_array_equal(y, sp.csr_matrix((va, ci, rp), shape=(m, n)).dot(x))

    lib = oracle.ref()
    for b in (2, 4):
        brp, bci, bva = oracle.csr_to_bcsr(m, n, b, rp, ci, va)
        mb, bn = oracle.C.c_int32(), oracle.C.c_int64()
        lib.ref_bcsr_shape_d(R.h, b, oracle.C.byref(mb), oracle.C.byref(bn))
        rbrp = np.zeros(mb.value + 1, np.int32)
        rbci = np.zeros(max(bn.value, 1), np.int32)
        rbva = np.zeros(max(bn.value, 1) * b * b, np.float64)
        lib.ref_csr_to_bcsr_d(R.h, b, oracle._p(rbrp), oracle._p(rbci), oracle._p(rbva))
        np.testing.assert_array_equal(brp, rbrp)
        np.testing.assert_array_equal(bci, rbci[:bn.value])
        np.testing.assert_array_equal(bva, rbva[:bn.value * b * b])
    width = int(np.diff(rp).max())
    if m * width <= 20_000_000:  # powerlaw_skew's ELL would hold 30,000 x 8,000 slots
        w, ecol, ev, rl = oracle.csr_to_ell(m, rp, ci, va)
        rw = lib.ref_ell_width_d(R.h)
        recol = np.zeros(max(m * rw, 1), np.int32)
        rev = np.zeros(max(m * rw, 1), np.float64)
        rrl = np.zeros(max(m, 1), np.int32)
        lib.ref_csr_to_ell_d(R.h, oracle._p(recol), oracle._p(rev), oracle._p(rrl))
        assert w == rw
        np.testing.assert_array_equal(ecol, recol[:m * w])
        np.testing.assert_array_equal(ev, rev[:m * w])
        np.testing.assert_array_equal(rl, rrl[:m])
