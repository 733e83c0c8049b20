"""The command-line driver (spmvbench_b200/driver.py): --stats on the CPU,
--validate / --auto / --profile on the GPU."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

from conftest import ROOT


def run(*args, timeout=900, env=None):
    e = dict(os.environ, **(env or {}))
    return subprocess.run([sys.executable, "-m", "spmvbench_b200.driver", *args], cwd=ROOT, capture_output=True,
                          text=True, timeout=timeout, env=e)


MTX = """%%MatrixMarket matrix coordinate real general
% {name}
4 4 6
1 1 2.0
1 3 -1.0
2 2 4.0
3 1 0.5
3 4 1.5
4 4 3.0
"""


def test_stats_runs_without_a_gpu():
    out = run("--stats", "--workload", "1", "4")
    assert out.returncode == 0, out.stderr
    assert "banded_100k_hb4" in out.stdout and "dense_share_of_stored_4x4=1" in out.stdout
    out = run("--stats", "--workload", "banded_100k_hb4")
    assert out.returncode == 0 and "=== banded_100k_hb4 ===" in out.stdout, out.stderr
    out = run("--stats", "--workload", "nine")
    assert out.returncode != 0 and "unknown workload" in out.stderr


def test_stats_on_matrix_files_and_data_dir(tmp_path):
    """--matrix FILE and --all ($SPMVBENCH_DATA) take .mtx files, as the
    reference's bench does (bench_main.cpp:77-96,102-139); a CSR cache file
    works too; names are the file stems."""
    import spmvbench_b200 as S
    for name in ("b_mat", "a_mat"):
        (tmp_path / f"{name}.mtx").write_text(MTX.format(name=name))
    (tmp_path / "notes.txt").write_text("not a matrix")
    out = run("--stats", "--matrix", str(tmp_path / "a_mat.mtx"))
    assert out.returncode == 0, out.stderr
    assert "=== a_mat ===" in out.stdout and "nnz=6" in out.stdout and "max_row_nnz=2" in out.stdout
    out = run("--stats", "--all", env={"SPMVBENCH_DATA": str(tmp_path)})
    assert out.returncode == 0, out.stderr
    assert out.stdout.index("=== a_mat ===") < out.stdout.index("=== b_mat ===")
    assert "notes" not in out.stdout
    A = S.read_matrix_market(str(tmp_path / "a_mat.mtx"))
    S.write_csr_cache(str(tmp_path / "a_mat.csrbin"), A)
    out = run("--stats", "--matrix", str(tmp_path / "a_mat.csrbin"))
    assert out.returncode == 0 and "nnz=6" in out.stdout, out.stderr
    empty = tmp_path / "empty"
    empty.mkdir()
    out = run("--stats", "--all", env={"SPMVBENCH_DATA": str(empty)})
    assert out.returncode != 0 and "no .mtx files found" in out.stderr


def test_bench_row_has_the_reference_columns_first():
    """results/bench.csv keeps the reference's columns in its order
    (bench_main.cpp:873-886) and its definitions: GFLOP/s from 2*nnz, bw_lo
    (x read once) and bw_hi (x per nonzero) in GB/s, bw_pct_peak from bw_hi."""
    from spmvbench_b200 import driver as D
    t = {"median_ms": 0.5, "min_ms": 0.4, "mean_ms": 0.55, "max_ms": 0.7, "iters": 20, "cold_ms": 0.6}
    r = D.bench_row("m", "fp64", "ell", 1, 4, t, 2e6, 1e9, 3e9, 8000.0, 0.25, gather=1e12, nnz=1e6)
    ref = ["device", "matrix", "precision", "kernel", "is_baseline", "iters", "median_ms", "min_ms", "mean_ms",
           "max_ms", "gflops", "bw_lo_gbs", "bw_hi_gbs", "bw_pct_peak", "transfer_ms", "speedup", "baseline"]
    assert list(r)[:len(ref)] == ref
    assert r["device"] == "cuda" and r["is_baseline"] == 0 and r["iters"] == 20
    assert r["gflops"] == pytest.approx(2e6 / 0.5e-3 / 1e9)
    assert r["bw_lo_gbs"] == pytest.approx(2000.0) and r["bw_hi_gbs"] == pytest.approx(6000.0)
    assert r["bw_pct_peak"] == pytest.approx(75.0) and r["roofline_frac"] == pytest.approx(0.25)
    assert r["gather_frac"] == pytest.approx(1e6 / 0.5e-3 / 1e12)
    assert D.HEURISTIC_COLUMNS[:8] == ["matrix", "device", "chosen", "oracle_best", "chosen_ms", "best_ms",
                                       "hit", "slowdown"]


def test_byte_models_follow_the_reference():
    """ByteModel lo / hi of bench_main.cpp:443-457 for CSR; ELL counts only the
    real entries (:661-667)."""
    from spmvbench_b200 import driver as D

    class A:
        m, n, nnz = 10, 20, 50
    lo, hi = D._models(D.CSR_SCALAR, 4, None, A, 8)
    assert lo == 50 * 12 + 11 * 4 + 20 * 8 + 10 * 8
    assert hi == 50 * 12 + 11 * 4 + 50 * 8 + 10 * 8
    lo, hi = D._models(D.ELL, 4, None, A, 8)
    assert lo == 50 * 12 + 10 * 4 + 10 * 8 + 20 * 8 and hi == 50 * 12 + 10 * 4 + 10 * 8 + 50 * 8


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
def test_bench_writes_reference_schema(tmp_path):
    out = run("--bench", "--workload", "1", "--iters", "3", "--warmup", "1")
    assert out.returncode == 0, out.stdout + out.stderr
    import csv as _csv
    with open(os.path.join(ROOT, "results", "bench.csv")) as f:
        rows = list(_csv.DictReader(f))
    assert rows and rows[0]["device"] == "cuda" and rows[0]["matrix"] == "banded_100k_hb4"
    assert {r["kernel"] for r in rows} >= {"csr_scalar", "csr_vector_l4", "csr_warp", "csr_merge", "ell", "bcsr_4x4"}
    assert all(float(r["median_ms"]) > 0 and float(r["transfer_ms"]) > 0 for r in rows)
    base = [r for r in rows if r["is_baseline"] == "1"]
    assert [r["kernel"] for r in base] == ["cusparse_spmv"] and base[0]["speedup"] == ""
    assert all(r["baseline"] == "cusparse_spmv" and float(r["speedup"]) > 0 for r in rows if r["is_baseline"] == "0")
    info = open(os.path.join(ROOT, "results", "gpu_info.txt")).read()
    assert "name=" in info and "compute_capability=10.0" in info


@pytest.mark.gpu
def test_auto_and_validate_on_a_matrix_file(tmp_path):
    (tmp_path / "small.mtx").write_text(MTX.format(name="small"))
    out = run("--validate", "--matrix", str(tmp_path / "small.mtx"))
    assert out.returncode == 0 and "validate: ok" in out.stdout, out.stdout + out.stderr
    out = run("--auto", "--matrix", str(tmp_path / "small.mtx"), "--iters", "3", "--warmup", "1")
    assert out.returncode == 0 and "small" in out.stdout, out.stdout + out.stderr


@pytest.mark.gpu
def test_spmm_timings(tmp_path):
    out = run("--spmm", "--k", "8", "--iters", "3", "--warmup", "1", "--dtype", "f32")
    assert out.returncode == 0, out.stdout + out.stderr
    assert out.stdout.count("GFLOP/s") == 7 and "wrote results/spmm.csv" in out.stdout
    assert "cusparse_spmm" in out.stdout and out.stdout.count("x cuSPARSE") == 6


def test_validate_criterion_against_scipy_catches_a_perturbed_y():
    """--validate's checks on the CPU: SciPy's product is the reference
    (independent of this library and of the oracle), an unchanged copy
    passes, and one row moved by more than the gamma_n bound - or a NaN, or a
    last-bit change where bit equality is required - is reported."""
    import numpy as np

    import spmvbench_b200 as S
    from spmvbench_b200 import driver as D
    A = S.generate(3, seed=5, scale_rows=20000)
    x = S.generate_vector(6, A.n)
    ref = D.scipy_product(A, A.values, x)
    assert D.row_bound_failures(A.rowptr, A.colind, A.values, x, ref, ref.copy(), 2.0 ** -53, 1e-12).size == 0
    bad = ref.copy()
    i = int(np.argmax(np.diff(A.rowptr)))
    bad[i] += 1e-9 * (abs(ref[i]) + 1.0)
    assert D.row_bound_failures(A.rowptr, A.colind, A.values, x, ref, bad, 2.0 ** -53, 1e-12).tolist() == [i]
    nan = ref.copy()
    nan[7] = np.nan
    assert 7 in D.row_bound_failures(A.rowptr, A.colind, A.values, x, ref, nan, 2.0 ** -53, 1e-12).tolist()
    ulp = ref.copy()
    ulp[3] = np.nextafter(ulp[3], np.inf)
    assert not np.array_equal(ulp, ref)  # what the bit-exact kernels are held to
    st = D.err_stats(bad, ref)
    assert st["max_abs_err"] > 0 and st["max_rel_err"] > 0 and st["l2_rel_err"] > 0
    assert D.err_stats(ref, ref) == {"max_rel_err": 0.0, "l2_rel_err": 0.0, "max_abs_err": 0.0}


def test_scipy_product_is_csr_omp_bitwise():
    """SciPy's float64 CSR product adds each row left to right like csr_omp,
    so the bit-exact GPU kernels are held to equality with it (the reference's
    own validate gate found max_rel 0 against SciPy)."""
    import numpy as np

    import oracle
    import spmvbench_b200 as S
    from spmvbench_b200 import driver as D
    for which, rows in ((1, 0), (2, 30000), (4, 8000)):
        A = S.generate(which, seed=9, scale_rows=rows)
        x = S.generate_vector(10, A.n)
        assert np.array_equal(D.scipy_product(A, A.values, x),
                              oracle.spmv_csr(A.m, A.rowptr, A.colind, A.values, x, np.float64))
