"""Host-side logic of libspmvb through its C ABI, on the CPU: the library
loads and exports every entry point include/spmvb.h declares; validation,
statistics, kernel selection, partitioning, sharding and the seeded
generators behave as specified. No kernel is launched here."""
from __future__ import annotations

import os
import re
import subprocess

import numpy as np
import pytest

import oracle
import spmvbench_b200 as S
from conftest import GOLDEN_NAMES, ROOT, load_golden
from spmvbench_b200 import _lib


def header_functions():
    text = open(os.path.join(ROOT, "include", "spmvb.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(spmvb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = S.load()
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.split()}
    declared = header_functions()
    assert len(declared) >= 30
    missing = [f for f in declared if f not in exported]
    assert not missing, missing
    for f in declared:
        assert hasattr(lib, f)
    assert set(_lib.SIGNATURES) <= set(declared)


def test_status_strings_and_version():
    lib = S.load()
    assert b"sm_100a" in lib.spmvb_version()
    for code, text in _lib.STATUS.items():
        assert lib.spmvb_status_string(code).decode() == text
    assert S.kernel_name(S.HYB) == "hyb" and S.kernel_name(99) == "unknown"
    assert [S.kernel_name(i) for i in range(7)] == _lib.KERNEL_NAMES


@pytest.mark.skipif(S.gpu_available(), reason="a GPU is present")
def test_no_device_is_reported_not_crashed():
    with pytest.raises(S.SpmvbError) as e:
        S.Context(0)
    assert e.value.status == 8


# ---- validation ------------------------------------------------------------------
def _bad(rowptr, colind, m, n):
    return S.CsrMatrix(m, n, np.array(rowptr, np.int32), np.array(colind, np.int32), np.ones(len(colind)))


@pytest.mark.parametrize("A,what", [
    (_bad([1, 2], [0, 0], 1, 2), "rowptr[0]"),
    (_bad([0, 2, 1], [0, 1], 2, 2), "decreases"),
    (_bad([0, 1, 2], [0, 2], 2, 2), "out of range"),
    (_bad([0, 1, 2], [0, -1], 2, 2), "out of range"),
])
def test_validation_rejects_bad_csr(A, what):
    with pytest.raises(S.SpmvbError) as e:
        S.csr_validate(A)
    assert e.value.status == 2 and what in str(e.value)


def test_short_or_out_of_range_arrays_are_refused_before_the_c_call():
    """The C ABI reads m + 1 rowptr and rowptr[m] colind / values entries
    through plain pointers; the Python layer refuses shorter arrays (and
    integer indices outside int32) before handing them over."""
    cases = [
        S.CsrMatrix(3, 4, np.array([0, 1, 2], np.int32), np.array([0, 1], np.int32), np.ones(2)),   # rowptr short
        S.CsrMatrix(2, 4, np.array([0, 2, 5], np.int32), np.array([0, 1, 2], np.int32), np.ones(5)),  # colind short
        S.CsrMatrix(2, 4, np.array([0, 1, 2], np.int64), np.array([0, 2**33], np.int64), np.ones(2)),  # > int32
    ]
    for A in cases:
        with pytest.raises(ValueError):
            S.csr_validate(A)
        with pytest.raises(ValueError):
            S.row_stats(A)
    A = S.CsrMatrix(2, 4, np.array([0, 1, 2], np.int32), np.array([0, 1], np.int32), np.ones(1))  # values short
    with pytest.raises(ValueError):
        S.write_csr_cache("/nonexistent/never.csrbin", A)


def test_c_abi_returns_errors_on_null_and_bad_arguments():
    """The boundary's contract: a status code, never a crash or an abort,
    for null pointers, negative sizes and bad ids on every entry point that
    runs without a GPU, and on the device entry points' handle checks."""
    import ctypes as C
    lib = S.load()
    rp = np.array([0, 1, 2], np.int32)
    ci = np.array([0, 1], np.int32)
    one = np.ones(2)
    out = C.c_void_p()
    i32, i64 = C.c_int32(), C.c_int64()
    st = S._lib.RowStats()
    calls = [
        lambda: lib.spmvb_query_gpu(0, None),
        lambda: lib.spmvb_context_create(0, None),
        lambda: lib.spmvb_compute_row_stats(None, None, 2, 2, 2, C.byref(st), None, 0),
        lambda: lib.spmvb_compute_row_stats(rp.ctypes.data, ci.ctypes.data, 2, 2, 2, None, None, 0),
        lambda: lib.spmvb_compute_row_stats(rp.ctypes.data, ci.ctypes.data, -1, 2, 2, C.byref(st), None, 0),
        lambda: lib.spmvb_compute_row_stats(rp.ctypes.data, ci.ctypes.data, 2, 2, 2, C.byref(st),
                                            np.zeros(1, np.int64).ctypes.data, 1),
        lambda: lib.spmvb_choose_spmv(None, None),
        lambda: lib.spmvb_choose_spmv_reference(None, None),
        lambda: lib.spmvb_generate(99, 1, 0, C.byref(i32), C.byref(i32), C.byref(i64), None, None, None),
        lambda: lib.spmvb_generate(1, 1, 0, None, None, None, None, None, None),
        lambda: lib.spmvb_generate(1, 1, -5, C.byref(i32), C.byref(i32), C.byref(i64), None, None, None),
        lambda: lib.spmvb_generate_vector(1, 10, None),
        lambda: lib.spmvb_generate_vector(1, -10, None),
        lambda: lib.spmvb_read_matrix_market(None, 0, C.byref(out)),
        lambda: lib.spmvb_read_matrix_market(b"/nonexistent.mtx", 0, None),
        lambda: lib.spmvb_csr_cache_write(None, 2, 2, 2, rp.ctypes.data, ci.ctypes.data, one.ctypes.data),
        lambda: lib.spmvb_csr_cache_write(b"/nonexistent/x.csrbin", 2, 2, 2, None, None, None),
        lambda: lib.spmvb_csr_cache_read(None, None),
        lambda: lib.spmvb_host_csr_get(None, None, None, None, None, None, None),
        lambda: lib.spmvb_partition_rows(None, 2, 2, None),
        lambda: lib.spmvb_partition_rows(rp.ctypes.data, 2, 0, np.zeros(3, np.int32).ctypes.data),
        lambda: lib.spmvb_partition_rows(rp.ctypes.data, -1, 2, np.zeros(3, np.int32).ctypes.data),
        lambda: lib.spmvb_shard_csr(2, rp.ctypes.data, ci.ctypes.data, 2, 5, rp.ctypes.data, C.byref(i32),
                                    C.byref(i64), None, None),
        lambda: lib.spmvb_shard_csr(2, rp.ctypes.data, ci.ctypes.data, 2, 0, None, C.byref(i32), C.byref(i64),
                                    None, None),
        lambda: lib.spmvb_shard_csr(2, rp.ctypes.data, ci.ctypes.data, 2, 0, np.array([0, 3, 2], np.int32).ctypes.data,
                                    C.byref(i32), C.byref(i64), None, None),
        lambda: lib.spmvb_matrix_create_csr(None, 1, 2, 2, 2, rp.ctypes.data, ci.ctypes.data, one.ctypes.data,
                                            C.byref(out)),
        lambda: lib.spmvb_spmv(None, 0, 4, 4, None, None, 1, None),
        lambda: lib.spmvb_spmv_host(None, 0, 4, 4, None, None, 1, None),
        lambda: lib.spmvb_spmm(None, 32, 0, 4, None, None, 1, None),
        lambda: lib.spmvb_spmv_merge_noalloc(1, 2, 2, 2, None, None, None, None, None, 1, None),
        # entries but no columns: refused before any pointer is used
        lambda: lib.spmvb_spmv_merge_noalloc(1, 2, 0, 2, rp.ctypes.data, ci.ctypes.data, one.ctypes.data,
                                             one.ctypes.data, one.ctypes.data, 1, None),
        lambda: lib.spmvb_pipeline_create(None, 3, C.byref(out)),
        lambda: lib.spmvb_pipeline_submit(None, 0, 4, 4, None, None, 1),
        lambda: lib.spmvb_dist_create(None, 2, 0, None, 1, 2, 2, None, None, None, None, C.byref(out)),
        lambda: lib.spmvb_context_check(None),
        lambda: lib.spmvb_selftest_wait_timeout(None),
        lambda: lib.spmvb_probe_gather_rate(None, 10, 100, None),
    ]
    for i, f in enumerate(calls):
        status = f()
        assert status != 0, i
        assert lib.spmvb_last_error(), i
    for destroy in (lib.spmvb_matrix_destroy, lib.spmvb_pipeline_destroy, lib.spmvb_dist_destroy):
        assert destroy(None) == 0
    lib.spmvb_host_csr_free(None)
    assert lib.spmvb_kernel_name(-1) == b"unknown" and lib.spmvb_status_string(99) == b"unknown status"


def test_noalloc_size_limit_boundary():
    """The no-allocation entry point's fixed scratch holds 65,536 merge tiles
    of 1,792 items (m + nnz <= 117,440,512). One item past that is refused
    with SPMVB_ERR_UNSUPPORTED; exactly at it the size check passes and the
    call goes on to fail on its null pointers (no device is touched)."""
    lib = S.load()
    limit = 65536 * 1792
    m = 1_000_000
    st = lib.spmvb_spmv_merge_noalloc(S.F64, m, m, limit + 1 - m, None, None, None, None, None, S.F64, None)
    assert st == 3 and b"no-allocation limit" in lib.spmvb_last_error()
    st = lib.spmvb_spmv_merge_noalloc(S.F64, m, m, limit - m, None, None, None, None, None, S.F64, None)
    assert st == 1 and b"null device pointer" in lib.spmvb_last_error()


def test_host_buffer_checks():
    """Host inputs shorter than what the C ABI reads, and outputs of the wrong
    type, layout or length, are refused by the Python layer."""
    from spmvbench_b200 import _host_in, _host_out
    assert _host_in([1, 2, 3], np.float64, 3, "x").dtype == np.float64
    with pytest.raises(ValueError, match="x holds 2 entries"):
        _host_in(np.ones(2), np.float64, 3, "x")
    y = np.empty(4)
    assert _host_out(y, np.float64, 4, "y") is y
    for bad in (np.empty(3), np.empty(4, np.float32), np.empty((4, 2))[:, 0], [0.0] * 4):
        with pytest.raises(ValueError):
            _host_out(bad, np.float64, 4, "y")
    ro = np.empty(4)
    ro.flags.writeable = False
    with pytest.raises(ValueError):
        _host_out(ro, np.float64, 4, "y")


def test_validation_agrees_with_the_csr_rules_on_random_damage():
    """spmvb_csr_validate accepts exactly the CSRs that satisfy rowptr[0] = 0,
    non-decreasing rowptr, rowptr[m] entries in colind, and every column in
    [0, n) (longer arrays are allowed; the tail is not read)."""
    rng = np.random.default_rng(11)
    for t in range(3000):
        m, n = int(rng.integers(0, 8)), int(rng.integers(0, 8))
        rp = np.zeros(m + 1, np.int64)
        rp[1:] = np.cumsum(rng.integers(0, 4, m))
        ci = rng.integers(0, max(n, 1), int(rp[-1])).astype(np.int64)
        k = t % 6
        if k == 1 and m:
            rp[rng.integers(0, m + 1)] += int(rng.integers(-3, 4))
        if k == 2 and ci.size:
            ci[rng.integers(0, ci.size)] = int(rng.integers(-3, n + 3))
        if k == 3:
            rp[0] = int(rng.integers(-2, 3))
        if k == 4 and ci.size:
            ci = ci[:-1]
        nnz = int(rp[m]) if m else 0
        valid = (rp[0] == 0 and bool(np.all(np.diff(rp) >= 0)) and 0 <= nnz <= ci.size
                 and (nnz == 0 or (ci[:nnz].min() >= 0 and ci[:nnz].max() < n)))
        A = S.CsrMatrix(m, n, rp.astype(np.int32), ci.astype(np.int32), np.zeros(ci.size))
        try:
            S.csr_validate(A)
            got = True
        except (S.SpmvbError, ValueError):
            got = False
        assert got == valid, (m, n, rp.tolist(), ci.tolist())


def test_validation_rejects_nnz_mismatch():
    A = S.CsrMatrix(2, 2, np.array([0, 1, 2], np.int32), np.array([0, 1], np.int32), np.ones(2))
    lib = S.load()
    rp = np.array([0, 1, 3], np.int32)
    st = lib.spmvb_csr_validate(2, 2, 2, rp.ctypes.data, A.colind.ctypes.data, None)
    assert st == 2 and b"nnz" in lib.spmvb_last_error()


@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_validation_accepts_golden(name):
    g = load_golden(name)
    A = S.CsrMatrix(int(g["m"]), int(g["n"]), g["rowptr"], g["colind"], g["values"])
    assert S.csr_validate(A) == (int(np.diff(g["rowptr"]).max()) if A.m else 0)


# ---- statistics / selection -----------------------------------------------------------
FIELDS = oracle.STAT_FIELDS


def _check_stats(A):
    mine = S.row_stats(A, histogram=True)
    ref = oracle.row_stats(A.m, A.n, A.rowptr, A.colind if A.nnz else None)
    for f in FIELDS:
        assert mine[f] == ref[f], f
    np.testing.assert_array_equal(mine["row_nnz_histogram"], ref["row_nnz_histogram"])
    return mine


@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_row_stats_bitwise_golden(name):
    g = load_golden(name)
    A = S.CsrMatrix(int(g["m"]), int(g["n"]), g["rowptr"], g["colind"], g["values"])
    mine = _check_stats(A)
    np.testing.assert_array_equal(np.array([mine[f] for f in FIELDS]), g["stats"])
    ch = S.choose_spmv_reference(mine)
    assert [ch["kernel"], ch["lanes"], ch["block_r"], ch["block_c"]] == g["choice"].tolist()


@pytest.mark.parametrize("which,rows", [(1, 0), (2, 50000), (3, 0), (4, 40000)])
def test_row_stats_bitwise_workloads(which, rows):
    A = S.generate(which, seed=3, scale_rows=rows)
    st = _check_stats(A)
    if which == 4:  # every stored 4x4 block is dense
        assert st["dense_share_of_stored_4x4"] == 1.0


def test_choose_reference_rules_match_oracle_grid():
    rng = np.random.default_rng(0)
    for _ in range(2000):
        st = dict(nnz=int(rng.choice([1000, 49999, 50000, 10 ** 6])), mean_row_nnz=float(rng.uniform(0, 80)),
                  cv_row_nnz=float(rng.uniform(0, 3)), max_over_mean=float(rng.uniform(1, 100)),
                  ell_padding_overhead=float(rng.uniform(1, 3)), frac_dense_blocks_4x4=float(rng.uniform(0, 1)))
        a = S.choose_spmv_reference(st)
        b = oracle.choose_spmv(st)
        assert [a[k] for k in ("kernel", "lanes", "block_r", "block_c", "rule")] == \
               [b[k] for k in ("kernel", "lanes", "block_r", "block_c", "rule")]
        assert a["reason"]


def test_choose_b200_rules():
    assert S.choose_spmv(dict(nnz=10 ** 7, mean_row_nnz=5, cv_row_nnz=30, max_over_mean=9000))["name"] == "hyb"
    assert S.choose_spmv(dict(nnz=10 ** 7, mean_row_nnz=32, cv_row_nnz=0,
                              dense_share_of_stored_4x4=1.0))["name"] == "bcsr"
    assert S.choose_spmv(dict(nnz=10 ** 7, mean_row_nnz=16, cv_row_nnz=0, ell_padding_overhead=1.0))["name"] == "ell"
    assert S.choose_spmv(dict(nnz=10 ** 7, mean_row_nnz=9, cv_row_nnz=0.01, ell_padding_overhead=1.1))["name"] == "ell"
    assert S.choose_spmv(dict(nnz=10 ** 7, mean_row_nnz=9, cv_row_nnz=0.9, ell_padding_overhead=4))["name"] == "csr_merge"
    c = S.choose_spmv(dict(nnz=10 ** 7, mean_row_nnz=200, cv_row_nnz=0.1, ell_padding_overhead=3))
    assert c["name"] == "csr_vector" and c["lanes"] == 32


# ---- partitioning / sharding ---------------------------------------------------------------
def _partition_rule(rowptr, parts):
    """bounds[g] = lower_bound(rowptr, ceil(g*nnz/parts))."""
    m = rowptr.size - 1
    nnz = int(rowptr[-1])
    b = [0] + [int(np.searchsorted(rowptr, -(-g * nnz // parts), side="left")) for g in range(1, parts)] + [m]
    return np.maximum.accumulate(np.minimum(np.array(b), m)).astype(np.int32)


@pytest.mark.parametrize("which,rows", [(2, 30000), (3, 0), (1, 0)])
@pytest.mark.parametrize("parts", [1, 2, 3, 4, 8])
def test_partition_rule_and_balance(which, rows, parts):
    A = S.generate(which, seed=5, scale_rows=rows)
    b = S.partition_rows(A.rowptr, parts)
    np.testing.assert_array_equal(b, _partition_rule(A.rowptr, parts))
    assert b[0] == 0 and b[-1] == A.m and np.all(np.diff(b) >= 0)
    share = np.diff(A.rowptr[b])
    maxrow = int(np.diff(A.rowptr).max())
    assert share.max() <= -(-A.nnz // parts) + maxrow


def test_partition_edge_cases():
    rp = np.array([0, 0, 0], np.int32)  # all-empty rows
    assert S.partition_rows(rp, 4).tolist() == [0, 0, 0, 0, 2]
    rp = np.array([0, 100], np.int32)  # one heavy row, more parts than rows
    assert S.partition_rows(rp, 3).tolist() == [0, 1, 1, 1]


@pytest.mark.parametrize("parts", [1, 2, 4, 8])
def test_shard_renumbering_round_trip(parts):
    A = S.generate(3, seed=9, scale_rows=20000)
    b = S.partition_rows(A.rowptr, parts)
    for r in range(parts):
        mr, rp, ci = S.shard_csr(A, b, r)
        assert mr == int(np.diff(b).max())
        p0, p1 = A.rowptr[b[r]], A.rowptr[b[r + 1]]
        np.testing.assert_array_equal(rp, A.rowptr[b[r]:b[r + 1] + 1] - p0)
        owner, local = ci // mr, ci % mr
        np.testing.assert_array_equal(b[owner] + local, A.colind[p0:p1])
        assert np.all(local < (b[owner + 1] - b[owner]))


# ---- generators ---------------------------------------------------------------------
def test_partition_and_shard_on_random_rowptrs():
    """partition_rows follows its rule (bounds[g] = lower_bound(rowptr,
    ceil(g*nnz/parts))) on random and skewed rowptrs with empty rows and more
    parts than rows, and every shard's renumbered columns map back to the
    owner's slot layout."""
    rng = np.random.default_rng(3)
    for t in range(3000):
        m, parts = int(rng.integers(0, 30)), int(rng.integers(1, 12))
        lens = rng.integers(0, 5, m) * (rng.random(m) < 0.7)
        if m and rng.random() < 0.2:
            lens[rng.integers(0, m)] = 100
        rp = np.zeros(m + 1, np.int32)
        rp[1:] = np.cumsum(lens)
        nnz = int(rp[-1])
        b = S.partition_rows(rp, parts)
        exp = [0] + [int(np.searchsorted(rp, -(-g * nnz // parts), side="left")) for g in range(1, parts)] + [m]
        assert b.tolist() == [min(max(v, 0), m) for v in exp]
        if m and t % 10 == 0:
            ci = rng.integers(0, m, nnz).astype(np.int32)
            A = S.CsrMatrix(m, m, rp, ci, np.ones(nnz))
            owner = np.searchsorted(b, np.arange(m), side="right") - 1
            for r in range(parts):
                mr, lrp, lci = S.shard_csr(A, b, r)
                slot = owner * mr + (np.arange(m) - b[owner])
                s0, s1 = rp[b[r]], rp[b[r + 1]]
                np.testing.assert_array_equal(lrp, rp[b[r]:b[r + 1] + 1] - s0)
                np.testing.assert_array_equal(lci, slot[ci[s0:s1]])


def test_generators_shapes_and_structure():
    A1 = S.generate(1)
    assert (A1.m, A1.n, A1.nnz) == (100000, 100000, 899980)
    lens = np.diff(A1.rowptr)
    assert lens.min() == 5 and lens.max() == 9
    diag = A1.values[A1.colind == np.repeat(np.arange(A1.m), lens)]
    assert diag.size == A1.m and diag.min() > 9.0 and diag.max() < 11.0
    A2 = S.generate(2, scale_rows=40000)
    assert A2.nnz == 16 * 40000 and np.all(np.diff(A2.rowptr) == 16)
    c = A2.colind.reshape(-1, 16)
    assert np.all(np.diff(c, axis=1) > 0) and c.min() >= 0 and c.max() < A2.n
    assert np.abs(A2.values).max() < 1.0
    A4 = S.generate(4, scale_rows=40000)
    assert A4.nnz == 32 * 40000 and np.all(np.diff(A4.rowptr) == 32)
    c4 = A4.colind.reshape(-1, 8, 4)
    assert np.all(c4 % 4 == np.arange(4)) and np.all(np.diff(c4[:, :, 0], axis=1) > 0)
    # the 4 rows of a block row share the block columns
    assert np.all(c4.reshape(-1, 4, 8, 4)[:, :, :, 0] == c4.reshape(-1, 4, 8, 4)[:, :1, :, 0])


def test_powerlaw_generator_distribution():
    A3 = S.generate(3)
    lens = np.diff(A3.rowptr)
    assert A3.m == 1_000_000 and lens.min() >= 1 and lens.max() <= 50000
    # Zipf(2.1): P(len=1) = 1/zeta(2.1) ~ 0.641; mean of the clipped law ~ 5
    assert abs((lens == 1).mean() - 0.641) < 0.005
    assert 4.0 < lens.mean() < 6.5
    for i in np.flatnonzero(lens > 1000)[:5]:
        c = A3.colind[A3.rowptr[i]:A3.rowptr[i + 1]]
        assert np.all(np.diff(c) > 0)


def test_generators_are_deterministic():
    a = S.generate(3, seed=11, scale_rows=5000)
    b = S.generate(3, seed=11, scale_rows=5000)
    c = S.generate(3, seed=12, scale_rows=5000)
    for f in ("rowptr", "colind", "values"):
        np.testing.assert_array_equal(getattr(a, f), getattr(b, f))
    assert a.nnz != c.nnz or not np.array_equal(a.colind, c.colind)
    x = S.generate_vector(4, 1000)
    np.testing.assert_array_equal(x, S.generate_vector(4, 1000))
    assert np.abs(x).max() < 1.0 and abs(x.mean()) < 0.1


def test_generator_rejects_bad_arguments():
    with pytest.raises(S.SpmvbError):
        S.generate(9)
    with pytest.raises(S.SpmvbError):
        S.generate(2, scale_rows=8)
