"""Pins the oracle (oracle/oracle.c) before it is trusted as the checker.

1. Golden fixtures produced by the reference itself (tests/golden/, made by
   tests/golden/make_golden.py from SpMVBench's generator, reader and CPU
   kernels): every output must match bit for bit.
2. The known answers written into the reference's own GoogleTest suite.
3. When oracle/_ref (the reference compiled from its sources) is present,
   oracle and reference must agree bit for bit on the seeded workloads.
"""
from __future__ import annotations

import math
import os

import numpy as np
import pytest

import oracle
from conftest import GOLDEN_NAMES, golden_B, load_golden


def _csr(g):
    return int(g["m"]), int(g["n"]), g["rowptr"].astype(np.int32), g["colind"].astype(np.int32), g["values"]


@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_spmv_matches_reference_bitwise(name):
    g = load_golden(name)
    m, n, rp, ci, va = _csr(g)
    x = g["x"]
    np.testing.assert_array_equal(oracle.spmv_csr(m, rp, ci, va, x, np.float64), g["y_dd"])
    vf, xf = va.astype(np.float32), x.astype(np.float32)
    np.testing.assert_array_equal(oracle.spmv_csr(m, rp, ci, vf, xf, np.float32), g["y_ff"])
    np.testing.assert_array_equal(oracle.spmv_csr(m, rp, ci, vf, xf, np.float64), g["y_fd"])
    if "y_scipy" in g:  # the reference's validate gate: csr_omp == SciPy (max_rel 0)
        np.testing.assert_array_equal(g["y_dd"], g["y_scipy"])


@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_spmm_matches_reference_bitwise(name):
    g = load_golden(name)
    m, n, rp, ci, va = _csr(g)
    for k in g["spmm_ks"]:
        k = int(k)
        B = golden_B(g, k)
        np.testing.assert_array_equal(oracle.spmm_csr(m, k, rp, ci, va, B, np.float64), g[f"Y{k}_dd"])
        got = oracle.spmm_csr(m, k, rp, ci, va.astype(np.float32), B.astype(np.float32), np.float32)
        np.testing.assert_array_equal(got, g[f"Y{k}_ff"])


@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_formats_match_reference_bitwise(name):
    g = load_golden(name)
    m, n, rp, ci, va = _csr(g)
    w, ecol, ev, rl = oracle.csr_to_ell(m, rp, ci, va)
    assert w == int(g["ell_width"])
    np.testing.assert_array_equal(ecol, g["ell_colind"])
    np.testing.assert_array_equal(ev, g["ell_values"])
    np.testing.assert_array_equal(rl, g["ell_row_lengths"])
    np.testing.assert_array_equal(oracle.spmv_ell(m, ecol, ev, rl, g["x"], np.float64), g["y_ell_dd"])
    for b in (2, 4):
        brp, bci, bva = oracle.csr_to_bcsr(m, n, b, rp, ci, va)
        np.testing.assert_array_equal(brp, g[f"bcsr{b}_rowptr"])
        np.testing.assert_array_equal(bci, g[f"bcsr{b}_colind"])
        np.testing.assert_array_equal(bva, g[f"bcsr{b}_values"])
        y = oracle.spmv_bcsr(m, n, b, b, brp, bci, bva, g["x"], np.float64)
        np.testing.assert_array_equal(y, g[f"y_bcsr{b}_dd"])


@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_stats_and_choice_match_reference(name):
    g = load_golden(name)
    m, n, rp, ci, va = _csr(g)
    st = oracle.row_stats(m, n, rp, ci if ci.size else None)
    got = np.array([st[f] for f in oracle.STAT_FIELDS])
    np.testing.assert_array_equal(got, g["stats"])
    np.testing.assert_array_equal(st["row_nnz_histogram"], g["histogram"])
    ch = oracle.choose_spmv(st)
    assert [ch["kernel"], ch["lanes"], ch["block_r"], ch["block_c"]] == g["choice"].tolist()


# ---- known answers of the reference's test suite ------------------------------
def test_ell_padding_math_known_answers():
    # tests/test_formats.cpp:23-46
    g = load_golden("formats_sample")
    m, n, rp, ci, va = _csr(g)
    w, ecol, ev, rl = oracle.csr_to_ell(m, rp, ci, va)
    assert (m, n, w, m * w, int(rp[-1])) == (3, 4, 4, 12, 7)
    assert rl.tolist() == [2, 1, 4]
    for j in range(1, 4):
        assert ecol[j * 3 + 1] == 0 and ev[j * 3 + 1] == 0.0
    assert math.isclose((m * w) / 7.0, 12.0 / 7.0)
    # padding only adds zeros (test_formats.cpp:58-63)
    assert ev.sum() == va.sum()


def test_bcsr_known_answers():
    # tests/test_formats.cpp:66-107
    g = load_golden("formats_sample")
    m, n, rp, ci, va = _csr(g)
    b2 = oracle.csr_to_bcsr(m, n, 2, rp, ci, va)
    assert (b2[0].size - 1, b2[1].size, b2[2].size) == (2, 4, 16)
    b4 = oracle.csr_to_bcsr(m, n, 4, rp, ci, va)
    assert (b4[0].size - 1, b4[1].size) == (1, 1)
    assert int(rp[-1]) / (b4[1].size * 16) == 7.0 / 16.0


def test_spmv_known_answers():
    # tests/test_spmv_correctness.cpp:57-67: single unsorted row sums to 10
    g = load_golden("single_row_unsorted")
    m, n, rp, ci, va = _csr(g)
    assert oracle.spmv_csr(m, rp, ci, va, np.ones(4), np.float64)[0] == 10.0
    # all-zero matrix gives zeros (test_spmv_correctness.cpp:91-95)
    g = load_golden("all_zero")
    m, n, rp, ci, va = _csr(g)
    assert oracle.spmv_csr(m, rp, ci, va, np.array([1.0, 2.0, 3.0]), np.float64).tolist() == [0.0] * 3


def test_stats_known_answers():
    # tests/test_stats.cpp:10-75
    g = load_golden("stats_1234")
    m, n, rp, ci, _ = _csr(g)
    s = oracle.row_stats(m, n, rp, ci)
    assert (s["rows"], s["cols"], s["nnz"]) == (4, 4, 10)
    assert s["mean_row_nnz"] == 2.5 and s["median_row_nnz"] == 2.5
    assert (s["min_row_nnz"], s["max_row_nnz"]) == (1, 4)
    assert math.isclose(s["stddev_row_nnz"], math.sqrt(1.25), abs_tol=1e-12)
    assert math.isclose(s["cv_row_nnz"], math.sqrt(1.25) / 2.5, abs_tol=1e-12)
    assert math.isclose(s["max_over_mean"], 1.6, abs_tol=1e-12)
    assert s["density"] == 10.0 / 16.0 and s["ell_padding_overhead"] == 16.0 / 10.0
    assert s["row_nnz_histogram"].tolist() == [0, 1, 1, 1, 1]
    g = load_golden("stats_const8")
    s = oracle.row_stats(*_csr(g)[:2], g["rowptr"], g["colind"])
    assert s["cv_row_nnz"] == 0.0 and s["ell_padding_overhead"] == 1.0 and s["median_row_nnz"] == 8.0
    g = load_golden("stats_skew")
    s = oracle.row_stats(*_csr(g)[:2], g["rowptr"], g["colind"])
    assert s["mean_row_nnz"] == 1003.0 / 4.0 and s["cv_row_nnz"] > 1.5 and s["max_over_mean"] > 2.0
    g = load_golden("stats_dense4")
    s = oracle.row_stats(*_csr(g)[:2], g["rowptr"], g["colind"])
    assert s["frac_dense_blocks_4x4"] == 1.0


SELECT_CASES = [
    # tests/test_select.cpp:11-83 (stats given, expected kernel id / lanes / block)
    (dict(nnz=1000, mean_row_nnz=10, cv_row_nnz=0.0), 0, None),
    (dict(nnz=1_000_000, mean_row_nnz=2.0, cv_row_nnz=0.3), 0, None),
    (dict(nnz=1_000_000, mean_row_nnz=8.0, cv_row_nnz=0.1, frac_dense_blocks_4x4=0.9), 5, None),
    (dict(nnz=1_000_000, mean_row_nnz=27.0, cv_row_nnz=5.0, max_over_mean=200.0), 3, None),
    (dict(nnz=1_000_000, mean_row_nnz=40.0, cv_row_nnz=0.1, max_over_mean=1.1,
          ell_padding_overhead=1.05), 4, None),
    (dict(nnz=1_000_000, mean_row_nnz=10.0, cv_row_nnz=0.2, max_over_mean=2.0,
          ell_padding_overhead=2.5), 1, 16),
    (dict(nnz=1_000_000, mean_row_nnz=20.0, cv_row_nnz=0.2, max_over_mean=2.0,
          ell_padding_overhead=2.5), 1, 32),
]


@pytest.mark.parametrize("stats,kernel,lanes", SELECT_CASES)
def test_choose_known_answers(stats, kernel, lanes):
    c = oracle.choose_spmv(stats)
    assert c["kernel"] == kernel
    if lanes is not None:
        assert c["lanes"] == lanes
    if kernel == 5:
        assert (c["block_r"], c["block_c"]) == (4, 4)


# ---- oracle vs the reference itself on the seeded workloads ---------------------
@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built (no reference tree)")
@pytest.mark.parametrize("which,rows", [(1, 0), (2, 20000), (3, 20000), (4, 20000)])
def test_oracle_matches_reference_on_workloads(which, rows):
    import spmvbench_b200 as S
    A = S.generate(which, seed=7, scale_rows=rows)
    x = S.generate_vector(8, A.n)
    R = oracle.RefCsr(A.m, A.n, A.rowptr, A.colind, A.values)
    np.testing.assert_array_equal(oracle.spmv_csr(A.m, A.rowptr, A.colind, A.values, x), R.spmv(x))
    Rf = oracle.RefCsr(A.m, A.n, A.rowptr, A.colind, A.values.astype(np.float32))
    vf, xf = A.values.astype(np.float32), x.astype(np.float32)
    np.testing.assert_array_equal(oracle.spmv_csr(A.m, A.rowptr, A.colind, vf, xf, np.float64),
                                  Rf.spmv(xf, np.float64))
    k = 8
    B = S.generate_vector(9, A.n * k).reshape(A.n, k)
    np.testing.assert_array_equal(oracle.spmm_csr(A.m, k, A.rowptr, A.colind, A.values, B), R.spmm(B, k))
    lib = oracle.ref()
    st = np.zeros(13)
    lib.ref_row_stats(oracle._p(A.rowptr), oracle._p(A.colind), A.m, A.n, A.nnz, oracle._p(st), None, 0)
    mine = oracle.row_stats(A.m, A.n, A.rowptr, A.colind)
    np.testing.assert_array_equal(np.array([mine[f] for f in oracle.STAT_FIELDS]), st)


@pytest.mark.skipif(not oracle.ref_cuda_available(), reason="the reference's GPU path was not built")
def test_reference_gpu_path_loads():
    """The reference's src/cuda compiled for sm_100a in place
    (oracle/_ref/libspmvref_cuda.so, `make -C oracle ref_cuda`) loads, and its
    gpu_available() answers without aborting where there is no GPU."""
    assert oracle.ref_cuda().refcuda_available() in (0, 1)


@pytest.mark.skipif(not (oracle.ref_available() and oracle.reference_tree() and os.path.exists(
    os.path.join(oracle.reference_tree(), "tools", "gen_matrices.py"))),
    reason="the reference tree or oracle/_ref is absent")
def test_golden_fixtures_regenerate_identically(tmp_path):
    """tests/golden/make_golden.py, run again from the reference, writes the
    committed fixtures array for array."""
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    subprocess.run([sys.executable, os.path.join(here, "golden", "make_golden.py"), "--out", str(tmp_path)],
                   check=True, capture_output=True, timeout=600)
    for name in GOLDEN_NAMES:
        g = np.load(os.path.join(here, "golden", f"{name}.npz"))
        h = np.load(os.path.join(tmp_path, f"{name}.npz"))
        assert sorted(g.files) == sorted(h.files), name
        for k in g.files:
            np.testing.assert_array_equal(g[k], h[k], err_msg=f"{name}:{k}")


@pytest.mark.parametrize("which,rows", [(1, 0), (1, 333), (2, 4096), (4, 8192), (5, 1000)])
def test_oracle_generator_equals_library_generator(which, rows):
    """The oracle's own statement of the seeded workloads (used by the CPU
    timing of the reference, which must not load the CUDA library) gives the
    library's matrices and vectors bit for bit."""
    import spmvbench_b200 as S
    m, n, rp, ci, va = oracle.generate(which, 2024, rows)
    A = S.generate(which, seed=2024, scale_rows=rows)
    assert (m, n) == (A.m, A.n)
    np.testing.assert_array_equal(rp, A.rowptr)
    np.testing.assert_array_equal(ci, A.colind)
    np.testing.assert_array_equal(va, A.values)
    np.testing.assert_array_equal(oracle.generate_vector(999, m), S.generate_vector(999, m))


def test_oracle_generator_full_uniform_workload():
    """The full 1M x 1M, 16-per-row workload the reference arm times: equal to
    the library's, array for array."""
    import spmvbench_b200 as S
    m, n, rp, ci, va = oracle.generate(2, 2024)
    A = S.generate(2, seed=2024)
    assert m == n == 1_000_000 and ci.size == 16_000_000
    assert np.array_equal(rp, A.rowptr) and np.array_equal(ci, A.colind) and np.array_equal(va, A.values)
