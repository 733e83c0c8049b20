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


REF = os.environ.get("SPMVBENCH_REF", "/root/reference")


@pytest.mark.skipif(not os.path.exists(os.path.join(REF, "bench", "bench_main.cpp")),
                    reason="the reference tree is absent")
def test_reference_bench_builds_against_dropin(tmp_path):
    """The reference's bench_main.cpp, unmodified, with its reader, validator
    and CPU kernels, compiles and links against include/spmvbench and
    libspmvb (its src/cuda, formats, stats and select replaced); its --stats
    and CPU --auto run on a Matrix Market file."""
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "tests", "cpp"), "ref_bench", f"REF={REF}"], check=True)
    bench = os.path.join(ROOT, "_build", "tests", "ref_bench", "bench")
    data = tmp_path / "data"
    data.mkdir()
    (data / "small.mtx").write_text("%%MatrixMarket matrix coordinate real general\n"
                                    "4 4 6\n1 1 2.0\n1 3 -1.0\n2 2 4.0\n3 1 0.5\n3 4 1.5\n4 4 3.0\n")
    out = subprocess.run([bench, "--stats", str(data / "small.mtx")], capture_output=True, text=True, timeout=120,
                         cwd=tmp_path)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "=== small ===" in out.stdout and "rows=4 cols=4 nnz=6" in out.stdout
    out = subprocess.run([bench, "--auto", "--all", "--cpu"], capture_output=True, text=True, timeout=300,
                         cwd=tmp_path, env=dict(os.environ, SPMVBENCH_DATA=str(data)))
    assert out.returncode == 0, out.stdout + out.stderr
    assert "small" in out.stdout and (tmp_path / "results" / "heuristic.csv").exists()
    shutil.rmtree(tmp_path / "results")
