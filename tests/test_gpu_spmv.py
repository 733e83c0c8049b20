"""SpMV parity on the GPU: every kernel, every (T, Acc) pair, against the
oracle on the reference's golden matrices, its test-suite edge cases, and
the seeded benchmark workloads (scaled and full size)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import spmvbench_b200 as S
from conftest import GOLDEN_NAMES, load_golden, mixed_x
from gpu_util import (DTYPE_PAIRS, NP, assert_bitwise, assert_rows_within_bound, oracle_y, run_spmv)

pytestmark = pytest.mark.gpu

# (kernel, lanes, block, how it must match csr_omp): "exact" = bit for bit,
# "bcsr" = bit for bit against spmv_bcsr_cpu and bounded against csr_omp,
# "hyb" = bit for bit on rows up to max(K, 256) entries, bounded on the rows
# cut into segments.
VARIANTS = [(S.CSR_SCALAR, 1, 4, "exact")] + \
           [(S.CSR_VECTOR, L, 4, "bound") for L in (2, 4, 8, 16, 32)] + \
           [(S.CSR_WARP, 1, 4, "bound"), (S.CSR_MERGE, 1, 4, "bound"), (S.ELL, 1, 4, "exact"),
            (S.HYB, 1, 4, "hyb"), (S.BCSR, 1, 2, "bcsr"), (S.BCSR, 1, 4, "bcsr")]


def golden_csr(name):
    g = load_golden(name)
    return g, S.CsrMatrix(int(g["m"]), int(g["n"]), g["rowptr"], g["colind"], g["values"])


def check_variant(ctx, A, x, dtype, acc, kernel, lanes, block, how, label, M=None):
    M = M or S.DeviceMatrix(ctx, A, dtype)
    got = run_spmv(M, x, kernel, lanes, block, acc)
    ref = oracle_y(A, x, dtype, acc)
    tag = f"{label} {S.kernel_name(kernel)} lanes={lanes} block={block} dtype={dtype}/{acc}"
    if how == "exact":
        assert_bitwise(ref, got, tag)
    elif how == "bcsr":
        vals = np.ascontiguousarray(A.values, NP[dtype])
        brp, bci, bva = oracle.csr_to_bcsr(A.m, A.n, block, A.rowptr, A.colind, vals)
        yb = oracle.spmv_bcsr(A.m, A.n, block, block, brp, bci, bva, np.ascontiguousarray(x, NP[dtype]), NP[acc])
        assert_bitwise(yb, got, tag + " vs spmv_bcsr_cpu")
        # csr_to_bcsr assigns entries into blocks, so a repeated (row, column)
        # keeps only its last value (src/formats.cpp:86): BCSR equals CSR
        # only on matrices without repeats.
        keys = A.colind.astype(np.int64) + np.repeat(np.arange(A.m), np.diff(A.rowptr)) * A.n
        if np.unique(keys).size == keys.size:
            assert_rows_within_bound(A, x, ref, got, dtype, acc, tag)
    elif how == "hyb":
        # rows in the ELL part (len <= K) and rows packed whole into a chunk
        # (len <= 256) are summed left to right from zero: bit for bit
        K = M.info()["hyb_width"]
        short = np.diff(A.rowptr) <= max(K, 256)
        assert_bitwise(ref[short], got[short], tag + " (whole rows)")
        assert_rows_within_bound(A, x, ref, got, dtype, acc, tag)
    else:
        assert_rows_within_bound(A, x, ref, got, dtype, acc, tag)
    return M


@pytest.mark.parametrize("name", GOLDEN_NAMES)
@pytest.mark.parametrize("dtype,acc", DTYPE_PAIRS)
def test_golden_all_kernels(ctx, name, dtype, acc):
    g, A = golden_csr(name)
    M = S.DeviceMatrix(ctx, A, dtype)
    for x in (g["x"], mixed_x(A.n)):
        for kernel, lanes, block, how in VARIANTS:
            check_variant(ctx, A, x, dtype, acc, kernel, lanes, block, how, name, M)
    if dtype == S.F64 and acc == S.F64:
        # csr_omp's own output on the fixture x is reproduced bit for bit
        assert_bitwise(g["y_dd"], run_spmv(M, g["x"], S.CSR_SCALAR), name)
        assert_bitwise(g["y_ell_dd"], run_spmv(M, g["x"], S.ELL), name)
        assert_bitwise(g["y_bcsr4_dd"], run_spmv(M, g["x"], S.BCSR, block=4), name)
        assert_bitwise(g["y_bcsr2_dd"], run_spmv(M, g["x"], S.BCSR, block=2), name)
    if dtype == S.F32 and acc == S.F32:
        assert_bitwise(g["y_ff"], run_spmv(M, g["x"], S.CSR_SCALAR), name)
    if dtype == S.F32 and acc == S.F64:
        assert_bitwise(g["y_fd"], run_spmv(M, g["x"], S.CSR_SCALAR, acc=S.F64), name)


WORKLOADS_SCALED = [(1, 0), (2, 200000), (3, 200000), (4, 100000)]


@pytest.mark.parametrize("which,rows", WORKLOADS_SCALED)
@pytest.mark.parametrize("dtype,acc", DTYPE_PAIRS)
def test_workloads_all_kernels(ctx, which, rows, dtype, acc):
    A = S.generate(which, seed=31, scale_rows=rows)
    x = S.generate_vector(32, A.n)
    M = S.DeviceMatrix(ctx, A, dtype)
    for kernel, lanes, block, how in VARIANTS:
        if kernel == S.ELL and which == 3:
            continue  # covered by test_ell_refuses_infeasible_padding
        check_variant(ctx, A, x, dtype, acc, kernel, lanes, block, how, f"w{which}", M)


def test_full_size_uniform_fp64(ctx):
    A = S.generate(2, seed=41)
    x = S.generate_vector(42, A.n)
    M = S.DeviceMatrix(ctx, A, S.F64)
    ref = oracle_y(A, x, S.F64, S.F64)
    assert_bitwise(ref, run_spmv(M, x, S.CSR_SCALAR), "C2 scalar")
    assert_bitwise(ref, run_spmv(M, x, S.ELL), "C2 ell")
    for k, lanes in ((S.CSR_MERGE, 1), (S.CSR_VECTOR, 8), (S.CSR_VECTOR, 16), (S.CSR_WARP, 1), (S.HYB, 1)):
        assert_rows_within_bound(A, x, ref, run_spmv(M, x, k, lanes), S.F64, S.F64, S.kernel_name(k))


@pytest.mark.parametrize("acc", [S.F32, S.F64])
def test_full_size_uniform_fp32(ctx, acc):
    """The uniform 1M x 1M, 16 nnz/row matrix stored in fp32: the thread-per-row
    kernels keep csr_omp's order in the accumulator type, so they match its
    fp32 (or fp32-in, fp64-accumulate) output bit for bit."""
    A = S.generate(2, seed=47)
    x = S.generate_vector(48, A.n)
    M = S.DeviceMatrix(ctx, A, S.F32)
    ref = oracle_y(A, x, S.F32, acc)
    assert_bitwise(ref, run_spmv(M, x, S.CSR_SCALAR, acc=acc), f"C2 fp32/{acc} scalar")
    assert_bitwise(ref, run_spmv(M, x, S.ELL, acc=acc), f"C2 fp32/{acc} ell")
    for k, lanes in ((S.CSR_MERGE, 1), (S.CSR_VECTOR, 16), (S.CSR_WARP, 1), (S.HYB, 1)):
        assert_rows_within_bound(A, x, ref, run_spmv(M, x, k, lanes, acc=acc), S.F32, acc,
                                 f"C2 fp32/{acc} {S.kernel_name(k)}")


def test_full_size_powerlaw_fp64(ctx):
    A = S.generate(3, seed=43)
    x = S.generate_vector(44, A.n)
    M = S.DeviceMatrix(ctx, A, S.F64)
    ref = oracle_y(A, x, S.F64, S.F64)
    assert_bitwise(ref, run_spmv(M, x, S.CSR_SCALAR), "C3 scalar")
    for k, lanes in ((S.CSR_MERGE, 1), (S.HYB, 1), (S.CSR_WARP, 1), (S.CSR_VECTOR, 4)):
        assert_rows_within_bound(A, x, ref, run_spmv(M, x, k, lanes), S.F64, S.F64, S.kernel_name(k))


def test_full_size_blocks_fp64(ctx):
    A = S.generate(4, seed=45)
    x = S.generate_vector(46, A.n)
    M = S.DeviceMatrix(ctx, A, S.F64)
    check_variant(ctx, A, x, S.F64, S.F64, S.BCSR, 1, 4, "bcsr", "C4", M)
    assert_bitwise(oracle_y(A, x, S.F64, S.F64), run_spmv(M, x, S.CSR_SCALAR), "C4 scalar")
    assert M.info()["bcsr4_block_nnz"] == 125000 * 8


def test_ell_refuses_infeasible_padding(ctx):
    # 1M rows x a 50,000-entry row = 5e10 padded slots (~600 GB): the
    # reference's eager ELL cannot run this matrix; here it is a clear error.
    A = S.generate(3, seed=47)
    M = S.DeviceMatrix(ctx, A, S.F64)
    with pytest.raises(S.SpmvbError) as e:
        M.prepare(S.ELL)
    assert e.value.status == 3 and "hybrid" in str(e.value)


def test_ell_with_more_slots_than_int32(ctx):
    """Padded ELL of 200,000 rows x an 11,000-entry row: 2.2e9 slots (26 GB),
    past 2^31, so every slot index (builder, kernel) must be 64-bit. The
    thread-per-row sum over each row's real entries equals csr_omp bit for
    bit, the longest row included."""
    import torch
    free, _ = torch.cuda.mem_get_info()
    if free < 40e9:
        pytest.skip("needs 40 GB of free device memory")
    rng = np.random.default_rng(71)
    m = n = 200_000
    lens = np.full(m, 4, np.int64)
    lens[m - 7] = 11_000
    rowptr = np.zeros(m + 1, np.int64)
    np.cumsum(lens, out=rowptr[1:])
    short = np.sort(rng.integers(0, n, (m, 4), dtype=np.int32), axis=1)
    long_row = np.sort(rng.choice(n, 11_000, replace=False)).astype(np.int32)
    colind = np.concatenate([short[:m - 7].ravel(), long_row, short[m - 6:].ravel()])
    assert colind.size == rowptr[-1]
    values = rng.standard_normal(rowptr[-1])
    A = S.CsrMatrix(m, n, rowptr.astype(np.int32), colind, values)
    x = S.generate_vector(72, n)
    M = S.DeviceMatrix(ctx, A, S.F64)
    M.prepare(S.ELL)
    assert M.info()["ell_padded_nnz"] == m * 11_000 > 2**31
    assert_bitwise(oracle_y(A, x, S.F64, S.F64), run_spmv(M, x, S.ELL), "ELL past 2^31 slots")
    M.close()


@pytest.mark.parametrize("which,rows", [(2, 50000), (3, 100000), (4, 20000), (1, 0)])
def test_device_formats_match_reference_layout(ctx, which, rows):
    A = S.generate(which, seed=51, scale_rows=rows)
    M = S.DeviceMatrix(ctx, A, S.F64)
    if which != 3:
        w, ecol, ev, rl = M.export_ell()
        ow, ocol, ov, orl = oracle.csr_to_ell(A.m, A.rowptr, A.colind, A.values)
        assert w == ow
        assert_bitwise(ocol, ecol, "ell colind")
        assert_bitwise(ov, ev, "ell values")
        assert_bitwise(orl, rl, "row_lengths")
    for b in (2, 4):
        rp, ci, va = M.export_bcsr(b)
        orp, oci, ova = oracle.csr_to_bcsr(A.m, A.n, b, A.rowptr, A.colind, A.values)
        assert_bitwise(orp, rp, f"bcsr{b} rowptr")
        assert_bitwise(oci, ci, f"bcsr{b} colind")
        assert_bitwise(ova, va, f"bcsr{b} values")


@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_golden_formats_match_reference(ctx, name):
    g, A = golden_csr(name)
    M = S.DeviceMatrix(ctx, A, S.F64)
    w, ecol, ev, rl = M.export_ell()
    assert w == int(g["ell_width"])
    assert_bitwise(g["ell_colind"], ecol, "ell colind")
    assert_bitwise(g["ell_values"], ev, "ell values")
    assert_bitwise(g["ell_row_lengths"], rl, "row_lengths")
    for b in (2, 4):
        rp, ci, va = M.export_bcsr(b)
        assert_bitwise(g[f"bcsr{b}_rowptr"], rp, "bcsr rowptr")
        assert_bitwise(g[f"bcsr{b}_colind"], ci, "bcsr colind")
        assert_bitwise(g[f"bcsr{b}_values"], va, "bcsr values")


def test_merge_is_deterministic(ctx):
    A = S.generate(3, seed=53, scale_rows=300000)
    x = S.generate_vector(54, A.n)
    M = S.DeviceMatrix(ctx, A, S.F64)
    a = run_spmv(M, x, S.CSR_MERGE)
    for _ in range(3):
        assert_bitwise(a, run_spmv(M, x, S.CSR_MERGE), "merge rerun")


def test_empty_shapes(ctx):
    for m, n in ((0, 5), (5, 0), (1, 1)):
        A = S.CsrMatrix(m, n, np.zeros(m + 1, np.int32), np.zeros(0, np.int32), np.zeros(0))
        M = S.DeviceMatrix(ctx, A, S.F64)
        for kernel, lanes, block, _ in VARIANTS:
            got = run_spmv(M, np.zeros(n), kernel, lanes, block)
            assert got.shape == (m,) and np.all(got == 0.0)


def test_host_buffer_entry_point_matches_device(ctx):
    A = S.generate(2, seed=55, scale_rows=100000)
    x = S.generate_vector(56, A.n)
    M = S.DeviceMatrix(ctx, A, S.F64)
    for kernel in (S.CSR_SCALAR, S.CSR_MERGE, S.ELL):
        assert_bitwise(run_spmv(M, x, kernel), M.spmv_host(x, kernel=kernel), "host entry")


@pytest.mark.parametrize("dtype,acc", DTYPE_PAIRS)
def test_host_entry_pinned_y_every_kernel(ctx, dtype, acc):
    """A pinned (mapped) y is written by the kernel itself, every kernel but
    the merge path; a pageable y goes through the device staging and a copy.
    Both must equal the device-buffer call bit for bit, on a skewed matrix
    (long rows cut into HYB segments) as well as a uniform one."""
    import torch
    for w, seed in ((2, 57), (3, 58)):
        A = S.generate(w, seed=seed, scale_rows=60000)
        x = S.generate_vector(seed + 1, A.n)
        M = S.DeviceMatrix(ctx, A, dtype)
        xp = torch.from_numpy(x.astype(NP[dtype])).pin_memory()
        for kernel, lanes, block, _ in VARIANTS:
            dev = run_spmv(M, x, kernel, lanes, block, acc)
            yp = torch.full((A.m,), float("nan"), dtype=torch.float64 if acc == S.F64 else torch.float32).pin_memory()
            M.spmv_host(xp.numpy(), kernel=kernel, lanes=lanes, block=block, acc=acc, out=yp.numpy())
            tag = f"w{w} {S.kernel_name(kernel)} lanes={lanes} block={block} {dtype}/{acc}"
            assert_bitwise(dev, yp.numpy(), tag + " pinned y")
            y = M.spmv_host(x.astype(NP[dtype]), kernel=kernel, lanes=lanes, block=block, acc=acc)
            assert_bitwise(dev, y, tag + " pageable y")


@pytest.mark.parametrize("K", [-1, 1, 3, 8, 64, 257])
def test_hyb_widths_are_exact_bounded_and_deterministic(ctx, K):
    """Every width of the hybrid format (-1 = width 0: every row chunked):
    rows up to max(K, 256) bit-identical to csr_omp, rows cut into segments
    within the gamma_n bound, and the same bits on every rerun (the cut rows'
    counters reset themselves)."""
    A = S.generate(3, seed=57, scale_rows=150000)
    x = S.generate_vector(58, A.n)
    M = S.DeviceMatrix(ctx, A, S.F64)
    M.prepare(S.HYB, K)
    info = M.info()
    K = max(K, 0)
    assert info["hyb_width"] == K
    lens = np.diff(A.rowptr)
    assert info["hyb_long_rows"] == int((lens > K).sum())
    assert info["hyb_tail_nnz"] == int(lens[lens > K].sum())
    assert info["hyb_ell_nnz"] == int(lens[lens <= K].sum())
    check_variant(ctx, A, x, S.F64, S.F64, S.HYB, 1, 4, "hyb", f"hyb K={K}", M)
    a = run_spmv(M, x, S.HYB)
    for _ in range(2):
        assert_bitwise(a, run_spmv(M, x, S.HYB), "hyb rerun")


@pytest.mark.parametrize("dtype,acc", DTYPE_PAIRS)
def test_hyb_width_zero_writes_empty_rows(ctx, dtype, acc):
    """Width 0 lists the empty rows and writes their zeros in the same
    launch; every other row goes through the chunks."""
    B = S.generate(3, seed=59, scale_rows=60000)
    lens = np.diff(B.rowptr)
    lens[::7] = 0  # every 7th row emptied
    rowptr = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    keep = np.repeat(np.arange(B.m) % 7 != 0, np.diff(B.rowptr))
    A = S.CsrMatrix(B.m, B.n, rowptr, B.colind[keep], B.values[keep])
    x = S.generate_vector(60, A.n)
    M = S.DeviceMatrix(ctx, A, dtype)
    M.prepare(S.HYB, -1)
    assert M.info()["hyb_width"] == 0 and M.info()["hyb_long_rows"] == int((lens > 0).sum())
    y = run_spmv(M, x, S.HYB, acc=acc)
    assert np.all(y[::7] == 0.0)
    assert_rows_within_bound(A, x, oracle_y(A, x, dtype, acc), y, dtype, acc, "hyb K=0")


@pytest.mark.parametrize("dtype,acc", DTYPE_PAIRS)
def test_bcsr_long_block_rows_and_empty_chunks(ctx, dtype, acc):
    """BCSR on the shapes the streamed kernel's chunk plan has to handle: a
    block row longer than one chunk (the plain kernel takes that matrix),
    and long runs of empty block rows (chunks whose copy has no bytes);
    both bit for bit against spmv_bcsr_cpu."""
    rng = np.random.default_rng(61)
    m = n = 4000
    lens = np.zeros(m, np.int64)
    lens[1000:1100] = rng.integers(1, 30, 100)   # rows 0..999 and 1100.. mostly empty
    lens[3000:3050] = rng.integers(1, 30, 50)
    cols = [np.sort(rng.choice(n, int(k), replace=False)) for k in lens]
    dense = np.sort(rng.choice(n, 3000, replace=False))  # one long row: > 64 4x4 blocks
    for label, heavy in (("empty runs", False), ("long block row", True)):
        rl = lens.copy()
        cl = list(cols)
        if heavy:
            rl[2000] = dense.size
            cl[2000] = dense
        rowptr = np.concatenate([[0], np.cumsum(rl)]).astype(np.int32)
        colind = np.concatenate(cl).astype(np.int32)
        A = S.CsrMatrix(m, n, rowptr, colind, rng.uniform(-1, 1, colind.size))
        x = mixed_x(n)
        M = S.DeviceMatrix(ctx, A, dtype)
        for block in (2, 4):
            check_variant(ctx, A, x, dtype, acc, S.BCSR, 1, block, "bcsr", label, M)


def _adversarial_csr(rng):
    """Small CSR with empty rows, repeated and unsorted columns, dense rows and
    ragged 2x2 / 4x4 tails (the shapes of tests/test_random_parity.py)."""
    m = int(rng.integers(1, 60))
    n = int(rng.integers(1, 70))
    kind = rng.integers(0, 4)
    if kind == 0:
        lens = rng.integers(0, min(n, 6) + 1, m)
    elif kind == 1:
        lens = np.where(rng.random(m) < 0.1, rng.integers(0, 3 * n + 1, m), rng.integers(0, 3, m))
    elif kind == 2:
        lens = np.full(m, n)
    else:
        lens = np.where(rng.random(m) < 0.6, 0, rng.integers(1, n + 1, m))
    rowptr = np.zeros(m + 1, np.int32)
    rowptr[1:] = np.cumsum(lens)
    nnz = int(rowptr[-1])
    colind = rng.integers(0, n, nnz).astype(np.int32)
    return S.CsrMatrix(m, n, rowptr, colind, rng.uniform(-1, 1, nnz))


def _distinct_columns(A):
    """A with each row's repeated columns dropped (first kept), order kept."""
    rows_c, rows_v = [], []
    for i in range(A.m):
        c = A.colind[A.rowptr[i]:A.rowptr[i + 1]]
        _, first = np.unique(c, return_index=True)
        keep = np.sort(first)
        rows_c.append(c[keep])
        rows_v.append(A.values[A.rowptr[i]:A.rowptr[i + 1]][keep])
    rp = np.zeros(A.m + 1, np.int32)
    rp[1:] = np.cumsum([r.size for r in rows_c])
    ci = np.concatenate(rows_c).astype(np.int32) if A.m else np.zeros(0, np.int32)
    va = np.concatenate(rows_v) if A.m else np.zeros(0)
    return S.CsrMatrix(A.m, A.n, rp, ci, va)


def test_device_bcsr_and_row_stats_on_adversarial_matrices(ctx):
    """The on-device BCSR conversion (one stable radix sort of block keys) and
    the device block census of row statistics on 120 adversarial matrices:
    BCSR 2x2 / 4x4 equal the oracle's csr_to_bcsr (the reference's layout,
    last duplicate wins) bit for bit, and every statistic equals the host
    computation bit for bit."""
    rng = np.random.default_rng(77)
    for t in range(120):
        A = _adversarial_csr(rng)
        M = S.DeviceMatrix(ctx, A, S.F64 if t % 2 == 0 else S.F32)
        vals = A.values if t % 2 == 0 else A.values.astype(np.float32)
        for b in (2, 4):
            rp, ci, va = M.export_bcsr(b)
            orp, oci, ova = oracle.csr_to_bcsr(A.m, A.n, b, A.rowptr, A.colind, vals)
            assert_bitwise(orp, rp, f"case {t} bcsr{b} rowptr")
            assert_bitwise(oci, ci, f"case {t} bcsr{b} colind")
            assert_bitwise(ova, va, f"case {t} bcsr{b} values")
        host, dev = S.row_stats(A, histogram=True), M.row_stats(histogram=True)
        for f in host:
            if f == "row_nnz_histogram":
                assert_bitwise(host[f], dev[f], f"case {t} histogram")
            else:
                assert host[f] == dev[f], (t, f, host[f], dev[f])
        M.close()


@pytest.mark.parametrize("which", [1, 2, 3, 4])
def test_device_row_stats_equal_host_on_workloads(ctx, which):
    """Full-size benchmark matrices: the device block census gives the host's
    statistics bit for bit (and the reference's, through the host pins)."""
    A = S.generate(which, seed=2024)
    M = S.DeviceMatrix(ctx, A, S.F64)
    host, dev = S.row_stats(A), M.row_stats()
    assert host == dev
    M.close()


@pytest.mark.parametrize("which,rows", [(2, 200000), (1, 0), (2, 100004), (2, 100002), (4, 40000)])
@pytest.mark.parametrize("stages", ["2", "3", "4"])
def test_ell_tma_stream_is_bit_identical(ctx, monkeypatch, which, rows, stages):
    """The ELL kernel whose matrix stream goes through the TMA engine
    (SPMVB_ELL_STREAM=tma, per-warp ring of STAGES slots): bit-identical to
    csr_omp in every (storage, accumulator) pair, on widths 9 and 16, a row
    count that is not a multiple of 32 (100,004: the last chunk's copy
    reaches past m), and where ell_rows runs instead (m = 100,002 not a
    multiple of 4; width 32)."""
    monkeypatch.setenv("SPMVB_ELL_STREAM", "tma")
    monkeypatch.setenv("SPMVB_ELL_TMA_STAGES", stages)
    A = S.generate(which, seed=57, scale_rows=rows)
    x = mixed_x(A.n, seed=58)
    for dt, acc in DTYPE_PAIRS:
        M = S.DeviceMatrix(ctx, A, dt)
        assert_bitwise(oracle_y(A, x, dt, acc), run_spmv(M, x, S.ELL, acc=acc), f"ell tma {dt}/{acc}")
        M.close()
    ctx.check()  # no bounded wait gave up


@pytest.mark.parametrize("which,rows", [(4, 40000), (4, 40004), (1, 0), (1, 1001), (2, 30000)])
def test_bcsr_tensor_core_experiment_within_gamma(ctx, monkeypatch, which, rows):
    """BCSR 4x4 on the fp64 tensor cores (SPMVB_BCSR_MMA=1, mma.sync m8n8k4,
    two block rows per warp): within the gamma_n bound of csr_omp, including
    an odd number of block rows (the last warp has no second block row), a
    last block row cut by m, and a last block column cut by n."""
    monkeypatch.setenv("SPMVB_BCSR_MMA", "1")
    A = S.generate(which, seed=59, scale_rows=rows)
    x = mixed_x(A.n, seed=60)
    M = S.DeviceMatrix(ctx, A, S.F64)
    got = run_spmv(M, x, S.BCSR, block=4)
    assert_rows_within_bound(A, x, oracle_y(A, x, S.F64, S.F64), got, S.F64, S.F64, "bcsr dmma")
    M.close()
    rng = np.random.default_rng(61)
    for t in range(20):
        C = _distinct_columns(_adversarial_csr(rng))  # repeated entries: BCSR keeps the last one
        xc = rng.uniform(-1, 1, C.n)
        MC = S.DeviceMatrix(ctx, C, S.F64)
        assert_rows_within_bound(C, xc, oracle_y(C, xc, S.F64, S.F64), run_spmv(MC, xc, S.BCSR, block=4),
                                 S.F64, S.F64, f"bcsr dmma adversarial {t}")
        MC.close()
