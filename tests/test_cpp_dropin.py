"""The C++ drop-in API (include/spmvbench: CsrMatrix, csr_to_ell,
csr_to_bcsr, compute_row_stats, choose_spmv, SpmvRunner, spmm_csr_tiled_*,
the cuSPARSE baselines) exercised by C++ programs written like the
reference's own tests (tests/cpp/dropin_test.cpp, cusparse_check.cpp), built
against libspmvb.so; and, where the reference tree is present, the
reference's own bench program built unmodified against the drop-in."""
from __future__ import annotations

import os
import shutil
import subprocess

import pytest

import oracle
from conftest import ROOT

BIN = os.path.join(ROOT, "_build", "tests", "dropin_test")


def _build():
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "tests", "cpp")], check=True)


def test_dropin_cpu_cases():
    _build()
    out = subprocess.run([BIN, "cpu"], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert " 0 failed" in out.stdout


def test_dropin_conversions_match_reference_on_random_matrices():
    """The drop-in's header-only csr_to_ell and csr_to_bcsr<2,2> / <4,4> on 400
    random matrices (empty rows, unsorted and repeated columns, partial blocks)
    against the reference's own conversions (oracle/_ref), bit for bit."""
    import oracle
    if not oracle.ref_available():
        pytest.skip("oracle/_ref not built")
    _build()
    out = subprocess.run([BIN, "fuzz", oracle.REF_PATH], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert " 0 failed" in out.stdout


@pytest.mark.gpu
def test_dropin_gpu_cases():
    _build()
    out = subprocess.run([BIN, "gpu"], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stdout + out.stderr
    assert " 0 failed" in out.stdout


@pytest.mark.gpu
def test_cusparse_baselines_agree_with_the_library():
    """cusparse_spmv_csr_f32/f64 and cusparse_spmm_f32/f64 (the reference
    bench's comparison rows, as the drop-in provides them) run and agree with
    SpmvRunner / spmm_csr_tiled within the gamma_n bound."""
    _build()
    out = subprocess.run([os.path.join(ROOT, "_build", "tests", "cusparse_check")], capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert " 0 failed" in out.stdout


REF = oracle.reference_tree() or ""
REF_BENCH = os.path.join(ROOT, "oracle", "_ref", "bench_dropin", "bench")

SMALL_MTX = ("%%MatrixMarket matrix coordinate real general\n"
             "4 4 6\n1 1 2.0\n1 3 -1.0\n2 2 4.0\n3 1 0.5\n3 4 1.5\n4 4 3.0\n")


def _write_mtx(path, m, n, rows, cols, vals):
    with open(path, "w") as f:
        f.write("%%MatrixMarket matrix coordinate real general\n")
        f.write(f"{m} {n} {len(rows)}\n")
        for r, c, v in zip(rows, cols, vals):
            f.write(f"{r + 1} {c + 1} {v!r}\n")


@pytest.mark.skipif(not os.path.exists(os.path.join(REF, "bench", "bench_main.cpp")),
                    reason="the reference tree is absent")
def test_reference_bench_builds_against_dropin(tmp_path):
    """The reference's bench_main.cpp, unmodified, with its reader, validator
    and CPU kernels, compiles and links against include/spmvbench and
    libspmvb (its src/cuda, formats, stats and select replaced); its --stats
    and CPU --auto run on a Matrix Market file."""
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "tests", "cpp"), "ref_bench", f"REF={REF}"], check=True)
    data = tmp_path / "data"
    data.mkdir()
    (data / "small.mtx").write_text(SMALL_MTX)
    out = subprocess.run([REF_BENCH, "--stats", str(data / "small.mtx")], capture_output=True, text=True,
                         timeout=120, cwd=tmp_path)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "=== small ===" in out.stdout and "rows=4 cols=4 nnz=6" in out.stdout
    out = subprocess.run([REF_BENCH, "--auto", "--all", "--cpu"], capture_output=True, text=True, timeout=300,
                         cwd=tmp_path, env=dict(os.environ, SPMVBENCH_DATA=str(data)))
    assert out.returncode == 0, out.stdout + out.stderr
    assert "small" in out.stdout and (tmp_path / "results" / "heuristic.csv").exists()
    shutil.rmtree(tmp_path / "results")


@pytest.mark.gpu
@pytest.mark.skipif(not os.path.exists(REF_BENCH), reason="the reference bench was not built against the drop-in")
def test_reference_bench_gpu_paths_run_through_dropin(tmp_path):
    """The reference's own GPU callers, unmodified, on the B200 through the
    drop-in: `--bench --gpu-only` (bench_gpu_type, bench/bench_main.cpp:605-772:
    every SpmvRunner kernel, SpMM tiles and the cuSPARSE comparison rows in
    fp64 and fp32) and `--auto` (evaluate_matrix_gpu, :265-301: choose_spmv
    against every kernel measured). Both exit 0 and write the reference's
    CSV files with a row per kernel."""
    import numpy as np
    data = tmp_path / "data"
    data.mkdir()
    (data / "small.mtx").write_text(SMALL_MTX)
    rng = np.random.default_rng(5)
    m = 3000  # a skewed random matrix: one long row, many short ones, an empty row
    rows, cols = [], []
    for i in range(m):
        k = 400 if i == 7 else (0 if i == 11 else int(rng.integers(1, 12)))
        c = np.sort(rng.choice(m, size=k, replace=False))
        rows += [i] * k
        cols += c.tolist()
    _write_mtx(data / "skewed.mtx", m, m, rows, cols, rng.uniform(-1, 1, len(rows)).tolist())
    env = dict(os.environ, SPMVBENCH_DATA=str(data))
    out = subprocess.run([REF_BENCH, "--bench", "--gpu-only", "--iters", "5", "--warmup", "2"],
                         capture_output=True, text=True, timeout=600, cwd=tmp_path, env=env)
    assert out.returncode == 0, out.stdout + out.stderr
    csv = (tmp_path / "results" / "bench.csv").read_text().splitlines()
    kernels = {line.split(",")[3] for line in csv[1:] if line.startswith("cuda")}
    for k in ("csr_scalar", "csr_merge", "ell", "cusparse_spmv"):
        assert any(k in name for name in kernels), (k, sorted(kernels))
    out = subprocess.run([REF_BENCH, "--auto", "--all"], capture_output=True, text=True, timeout=600,
                         cwd=tmp_path, env=env)
    assert out.returncode == 0, out.stdout + out.stderr
    heur = (tmp_path / "results" / "heuristic.csv").read_text()
    assert "skewed" in heur and "small" in heur
