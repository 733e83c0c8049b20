"""Command-line driver, the B200 counterpart of SpMVBench's `bench`
(bench/bench_main.cpp:957-984):

    python -m spmvbench_b200.driver --stats    [--workload W ...]
    python -m spmvbench_b200.driver --auto     [--workload W ...] [--dtype f64|f32]
    python -m spmvbench_b200.driver --bench    [--workload W ...] [--dtype ...] [--iters N]
    python -m spmvbench_b200.driver --validate [--workload W ...]
    python -m spmvbench_b200.driver --spmm     [--dtype ...] [--k K] [--iters N]
    python -m spmvbench_b200.driver --profile KERNEL --workload W [--steps N] [--warmup N]

Matrices: the seeded benchmark workloads (--workload: 1 banded, 2 uniform,
3 power-law, 4 4x4 blocks, 5 the SpMM matrix; see spmvbench_b200.WORKLOADS),
or files (--matrix a.mtx b.csrbin ...), or every .mtx file of $SPMVBENCH_DATA
(default data/) with --all, as the reference's bench takes them.

--stats    row statistics (compute_row_stats fields, bench_main.cpp:102-139)
--auto     choose_spmv's pick against every kernel measured on the device; a
           hit is a pick within 1.1x of the fastest (the reference counts exact
           hits only, bench_main.cpp:229-253); writes results/heuristic.csv
           with the reference's columns (bench_main.cpp:408-417)
--bench    every kernel: warm median/min/mean/max per launch over 20 replays
           of a CUDA graph of 10 launches (one event pair each), cold median
           per launch after a 256 MB flush, GFLOP/s, compulsory (bw_lo) and
           no-reuse (bw_hi) GB/s, the fraction of the measured HBM peak, the
           random-gather ceiling and the transfer time of x in and y out;
           the reference's vendor baseline row (cusparse_spmv, through
           torch's sparse CSR SpMV; --no-baseline skips it) and every
           kernel's speedup over it; writes results/bench.csv with the
           reference's columns first (bench_main.cpp:873-886) and
           results/gpu_info.txt
--validate every kernel in the reference's modes fp32/fp32, fp32/fp64 and
           fp64/fp64 against SciPy's float64 y = A x (an independent CPU
           product, as the reference validates against SciPy): the
           reference's error statistics, a per-row gamma_n criterion, bit
           equality for the kernels that keep csr_omp's order (fp64); writes
           results/accuracy.csv with the reference's columns
--spmm     SpMM Y = A X on the k=64 workload (A = the uniform 1M x 16 matrix,
           X 1,000,000 x k) for tiles 16/32/64, plain and bucketed, the
           timings of spmm_csr_tiled (spmm_cuda.cu:215-270: median over
           `iters` launches after warm-up); GFLOP/s (2*nnz*k), compulsory GB/s
           (A + X + Y once) and no-reuse GB/s (A + one X row per entry + Y,
           the traffic when X does not fit in L2), beside the reference's
           cusparse_spmm baseline (torch's sparse CSR x dense product) and
           each tile's speedup over it; writes results/spmm.csv
--profile  warmup + steps launches of one kernel on one workload (for ncu);
           KERNEL `spmm` runs spmvb_spmm (tile 64) with k = --k
"""
from __future__ import annotations

import argparse
import csv
import json
import os
import statistics
import sys

import numpy as np

from . import (BCSR, CSR_MERGE, CSR_SCALAR, CSR_VECTOR, CSR_WARP, ELL, F32, F64, HYB, WORKLOADS,
               Context, DeviceMatrix, choose_spmv, generate, generate_vector, kernel_name, query_gpu,
               read_csr_cache, read_matrix_market, row_stats)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# (label, kernel id, lanes, block) - the variants the reference's bench times
# (bench_main.cpp:651-658), plus every lane count, 2x2 blocks and HYB.
VARIANTS = [("csr_scalar", CSR_SCALAR, 1, 4)] + \
           [(f"csr_vector_l{L}", CSR_VECTOR, L, 4) for L in (2, 4, 8, 16, 32)] + \
           [("csr_warp", CSR_WARP, 1, 4), ("csr_merge", CSR_MERGE, 1, 4), ("ell", ELL, 1, 4),
            ("hyb", HYB, 1, 4), ("bcsr_2x2", BCSR, 1, 2), ("bcsr_4x4", BCSR, 1, 4)]
EXACT = {CSR_SCALAR, ELL}  # kernels that keep csr_omp's summation order


def _peak_gbs():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _models(kernel, block, M, A, es):
    """(compulsory, no-reuse) bytes per launch for the format `kernel` reads:
    the reference's ByteModel lo / hi (bench_main.cpp:443-457; ELL counts
    only the real entries and BCSR its block storage, :661-678). lo reads x
    once; hi fetches an x value (or an x slice per block row) per stored entry."""
    m, n, nnz = A.m, A.n, A.nnz
    if kernel in (ELL, HYB):
        base = nnz * (es + 4) + m * 4 + m * es
        return base + n * es, base + nnz * es
    if kernel == BCSR:
        info = M.info()
        bn = info["bcsr2_block_nnz" if block <= 2 else "bcsr4_block_nnz"]
        b = 2 if block <= 2 else 4
        base = bn * (b * b * es + 4) + ((m + b - 1) // b + 1) * 4 + m * es
        return base + n * es, base + bn * b * b * es
    base = nnz * (es + 4) + (m + 1) * 4 + m * es
    return base + n * es, base + nnz * es


# results/bench.csv: the reference's columns in its order (bench_main.cpp:873-886),
# then the columns this driver adds.
BENCH_COLUMNS = ["device", "matrix", "precision", "kernel", "is_baseline", "iters", "median_ms", "min_ms",
                 "mean_ms", "max_ms", "gflops", "bw_lo_gbs", "bw_hi_gbs", "bw_pct_peak", "transfer_ms",
                 "speedup", "baseline",
                 "gpus", "peak_gbs", "roofline_frac", "cold_ms", "gather_frac", "lanes", "block"]
# results/heuristic.csv: the reference's columns (bench_main.cpp:408-417), then the rule text.
HEURISTIC_COLUMNS = ["matrix", "device", "chosen", "oracle_best", "chosen_ms", "best_ms", "hit", "slowdown",
                     "reason"]


def bench_row(matrix, precision, label, lanes, block, t, flops, lo, hi, peak, transfer_ms, gather=None,
              nnz=None):
    """One results/bench.csv row. `t` holds the timing summary of _time
    (median/min/mean/max ms per launch, iters, cold ms). bw_pct_peak follows
    the reference (no-reuse traffic over the peak, in percent); roofline_frac
    is the compulsory traffic over the peak. is_baseline is 0 and speedup /
    baseline are empty here; _measure_all fills speedup and baseline when the
    cuSPARSE baseline row runs, and marks that row is_baseline = 1."""
    med = t["median_ms"]
    gbs = (lambda b: b / (med * 1e-3) / 1e9) if med > 0 else (lambda b: 0.0)
    row = {"device": "cuda", "matrix": matrix, "precision": precision, "kernel": label, "is_baseline": 0,
           "iters": t["iters"], "median_ms": med, "min_ms": t["min_ms"], "mean_ms": t["mean_ms"],
           "max_ms": t["max_ms"], "gflops": flops / (med * 1e-3) / 1e9 if med > 0 else 0.0,
           "bw_lo_gbs": gbs(lo), "bw_hi_gbs": gbs(hi), "bw_pct_peak": 100.0 * gbs(hi) / peak if peak else 0.0,
           "transfer_ms": transfer_ms, "speedup": "", "baseline": "",
           "gpus": 1, "peak_gbs": peak, "roofline_frac": gbs(lo) / peak if peak else 0.0,
           "cold_ms": t["cold_ms"],
           "gather_frac": (nnz / (med * 1e-3) / gather) if (gather and nnz and med > 0) else "",
           "lanes": lanes, "block": block}
    assert list(row) == BENCH_COLUMNS
    return row


_FLUSH = None
GRAPH_LAUNCHES = 10   # launches captured per graph
GRAPH_REPLAYS = 20    # timed replays (median reported)


def _time(M, x, y, kernel, lanes, block, iters, warmup):
    """Timing summary of one launch: median / min / mean / max ms over the
    warm replays (and their count, `iters`), and the cold median `cold_ms`.

    Warm: GRAPH_LAUNCHES launches captured once as a CUDA graph, each of
    GRAPH_REPLAYS replays timed by one event pair (so no host launch gap is
    counted), median and min over the replays. Cold: one launch right after a
    write of a 256 MB buffer (twice the L2), median over `iters`; the flush
    keeps the GPU busy, so the launch starts without a host gap."""
    import torch
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for _ in range(warmup):
            M.spmv(x, y, kernel=kernel, lanes=lanes, block=block, stream=s)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s, capture_error_mode="relaxed"):
            for _ in range(GRAPH_LAUNCHES):
                M.spmv(x, y, kernel=kernel, lanes=lanes, block=block, stream=s)
        g.replay()
        s.synchronize()
        warm = []
        for _ in range(GRAPH_REPLAYS):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(s)
            g.replay()
            b.record(s)
            b.synchronize()
            warm.append(a.elapsed_time(b) / GRAPH_LAUNCHES)
        del g
        cold = []
        for _ in range(iters):
            _FLUSH.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(s)
            M.spmv(x, y, kernel=kernel, lanes=lanes, block=block, stream=s)
            b.record(s)
            b.synchronize()
            cold.append(a.elapsed_time(b))
    return {"median_ms": statistics.median(warm), "min_ms": min(warm), "mean_ms": statistics.fmean(warm),
            "max_ms": max(warm), "iters": len(warm), "cold_ms": statistics.median(cold)}


def _data_dir():
    """$SPMVBENCH_DATA, else data/ (bench_main.cpp:77-82)."""
    return os.environ.get("SPMVBENCH_DATA") or "data"


def _sources(args):
    """The matrices a command runs on, as (name, key) pairs: the files named
    by --matrix (Matrix Market, or a binary CSR cache ending in .csrbin),
    every .mtx file of the data directory with --all (sorted, as the
    reference's list_matrices, bench_main.cpp:84-96), else the seeded
    workloads of --workload. Names are file stems, as in the reference."""
    if getattr(args, "matrix", None):
        return [(os.path.splitext(os.path.basename(p))[0], p) for p in args.matrix]
    if getattr(args, "all", False):
        d = _data_dir()
        files = sorted(os.path.join(d, f) for f in os.listdir(d) if f.endswith(".mtx")) if os.path.isdir(d) else []
        if not files:
            raise SystemExit(f"no .mtx files found in {d}")
        return [(os.path.splitext(os.path.basename(p))[0], p) for p in files]
    return [(WORKLOADS[w], w) for w in args.workload]


def _load(key, seed=2024):
    """CSR of a source key: a seeded workload id, a .csrbin cache or a .mtx file."""
    if isinstance(key, int):
        return generate(key, seed=seed)
    if key.endswith(".csrbin"):
        return read_csr_cache(key)
    return read_matrix_market(key)


def _time_eager(launch, iters, warmup):
    """Timing summary of an eager launch (used for the vendor baseline, whose
    calls allocate and are not captured in a graph): warm = GRAPH_REPLAYS
    rounds of GRAPH_LAUNCHES back-to-back calls, one event pair per round
    (host launch gaps included); cold = one call after the L2 flush."""
    import torch
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        launch()
    torch.cuda.synchronize()
    warm, cold = [], []
    for _ in range(GRAPH_REPLAYS):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(GRAPH_LAUNCHES):
            launch()
        b.record()
        b.synchronize()
        warm.append(a.elapsed_time(b) / GRAPH_LAUNCHES)
    for _ in range(iters):
        _FLUSH.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        launch()
        b.record()
        b.synchronize()
        cold.append(a.elapsed_time(b))
    return {"median_ms": statistics.median(warm), "min_ms": min(warm), "mean_ms": statistics.fmean(warm),
            "max_ms": max(warm), "iters": len(warm), "cold_ms": statistics.median(cold)}


def _torch_csr(A, dtype):
    """A as a torch sparse CSR tensor on the GPU (for the cuSPARSE baselines)."""
    import warnings

    import torch
    npd = np.float64 if dtype == F64 else np.float32
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", UserWarning)  # torch's beta-state notice for sparse CSR
        return torch.sparse_csr_tensor(torch.from_numpy(np.ascontiguousarray(A.rowptr, np.int32)).cuda(),
                                       torch.from_numpy(np.ascontiguousarray(A.colind, np.int32)).cuda(),
                                       torch.from_numpy(np.ascontiguousarray(A.values, npd)).cuda(),
                                       size=(A.m, A.n), check_invariants=False)


def _cusparse_row(name, precision, A, M, x, y, dtype, iters, warmup, peak, transfer):
    """The reference bench's vendor baseline row (cusparse_spmv,
    bench_main.cpp:643-650): cuSPARSE CSR SpMV through torch's sparse CSR
    matrix-vector product, timed beside the library's kernels. A comparison
    only; nothing of the library calls it. None if it cannot run here."""
    import torch
    if A.nnz == 0 or A.m == 0:
        return None
    try:
        Ac = _torch_csr(A, dtype)
        yc = torch.mv(Ac, x)
        M.spmv(x, y, kernel=CSR_SCALAR)
        torch.cuda.synchronize()
        scale = float(y.abs().max()) or 1.0
        diff = float((yc - y).abs().max()) / scale
        t = _time_eager(lambda: torch.mv(Ac, x), iters, warmup)
    except Exception as e:  # noqa: BLE001 - the baseline is optional
        print(f"  cusparse_spmv: unavailable ({e})")
        return None
    es = 8 if dtype == F64 else 4
    lo, hi = _models(CSR_SCALAR, 4, M, A, es)
    row = bench_row(name, precision, "cusparse_spmv", 1, 1, t, 2.0 * A.nnz, lo, hi, peak, transfer)
    row.update(is_baseline=1, baseline="cusparse_spmv")
    print(f"  cusparse_spmv: max |y - y_csr_scalar| / max|y| = {diff:.2e}")
    return row


def _setup(key, dtype, seed=2024):
    import torch
    A = _load(key, seed)
    xh = generate_vector(999, A.n)
    npd = np.float64 if dtype == F64 else np.float32
    ctx = Context(0)
    M = DeviceMatrix(ctx, A, dtype)
    x = torch.from_numpy(xh.astype(npd)).cuda()
    y = torch.empty(A.m, dtype=torch.float64 if dtype == F64 else torch.float32, device="cuda")
    return ctx, A, M, x, y, xh


def _usable(M, kernel, block):
    try:
        M.prepare(kernel, block if kernel == BCSR else 0)
        return True
    except Exception as e:  # noqa: BLE001 - an unsupported format is reported, not fatal
        print(f"  {kernel_name(kernel)}: {e}")
        return False


def cmd_stats(args):
    for name, key in _sources(args):
        A = _load(key, args.seed)
        s = row_stats(A)
        print(f"=== {name} ===")
        print("  " + ", ".join(f"{k}={v:.6g}" if isinstance(v, float) else f"{k}={v}" for k, v in s.items()))
    return 0


def _transfer_ms(x, y, xh, reps=10):
    """Median of `reps` rounds of one upload of x and one download of y from
    and to pageable host memory: the reference's transfer_ms
    (SpmvRunner::measure_transfer_ms, spmv_cuda.cu:340-372), kernel excluded."""
    import torch
    hx = torch.from_numpy(np.ascontiguousarray(xh)).to(x.dtype)
    for _ in range(2):
        x.copy_(hx)
        y.cpu()
    ts = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        x.copy_(hx)
        y.cpu()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def _measure_all(name, key, dtype, iters, warmup, seed=2024, baseline=False):
    """Every usable kernel on one matrix: a list of (kernel id, bench row);
    with `baseline`, the cuSPARSE row first (kernel id None)."""
    ctx, A, M, x, y, xh = _setup(key, dtype, seed)
    es = 8 if dtype == F64 else 4
    peak, _ = _peak_gbs()
    precision = "fp64" if dtype == F64 else "fp32"
    gather = ctx.gather_rate(max(A.n, 1), max(A.nnz, 1 << 24))  # the probe needs enough gathers to time
    transfer = _transfer_ms(x, y, xh)
    out = []
    for label, k, lanes, block in VARIANTS:
        if k == BCSR and key == 3:
            continue  # 1M block rows x 50,000-entry rows: blocks would not be the format
        if not _usable(M, k, block):
            continue
        t = _time(M, x, y, k, lanes, block, iters, warmup)
        lo, hi = _models(k, block, M, A, es)
        out.append((k, bench_row(name, precision, label, lanes, block, t, 2.0 * A.nnz, lo, hi, peak,
                                 transfer, gather, A.nnz)))
    if baseline:
        cs = _cusparse_row(name, precision, A, M, x, y, dtype, iters, warmup, peak, transfer)
        if cs is not None:
            for _, r in out:  # speedup over the vendor baseline, as the reference reports it
                r.update(baseline="cusparse_spmv", speedup=cs["median_ms"] / r["median_ms"])
            out.insert(0, (None, cs))
    return A, out, gather


def _write_gpu_info(peak, src):
    """results/gpu_info.txt in the reference's key=value form (bench_main.cpp:888-899)."""
    g = query_gpu(0)
    os.makedirs("results", exist_ok=True)
    with open(os.path.join("results", "gpu_info.txt"), "w") as f:
        f.write(f"name={g['name']}\ncompute_capability={g['major']}.{g['minor']}\nassumed_peak_gbs={peak}\n"
                f"peak_source={'measured copy bandwidth (MEASURED_PEAKS.json)' if src == 'measured' else src}\n"
                f"theoretical_peak_gbs={g['peak_gbs']:.1f}\n"
                "bandwidth_model=no-reuse (x fetched per nonzero) for bw_hi_gbs and bw_pct_peak; "
                "compulsory (x once) for bw_lo_gbs and roofline_frac\n"
                f"sm_count={g['sm_count']}\nl2_bytes={g['l2_bytes']}\nmkl_available=0\n")


def cmd_auto(args):
    dtype = F64 if args.dtype == "f64" else F32
    out = []
    for name, key in _sources(args):
        A, rows, _ = _measure_all(name, key, dtype, args.iters, args.warmup, args.seed)
        st = row_stats(A)
        c = choose_spmv(st)
        best = min((r for _, r in rows), key=lambda r: r["median_ms"])
        pick = [r for k, r in rows if k == c["kernel"] and (c["kernel"] != CSR_VECTOR or r["lanes"] == c["lanes"])
                and (c["kernel"] != BCSR or r["block"] == c["block_r"])]
        chosen_ms = pick[0]["median_ms"] if pick else float("nan")
        slow = chosen_ms / best["median_ms"]
        row = dict(matrix=name, device="cuda", chosen=c["name"], oracle_best=best["kernel"],
                   chosen_ms=chosen_ms, best_ms=best["median_ms"], hit=int(slow <= 1.1), slowdown=slow,
                   reason=c["reason"])
        assert list(row) == HEURISTIC_COLUMNS
        out.append(row)
        print(f"{name:24s} chosen={c['name']:12s} best={best['kernel']:14s} "
              f"chosen_ms={chosen_ms:.4f} best_ms={best['median_ms']:.4f} slowdown={slow:.3f}")
    hits = sum(r["hit"] for r in out)
    print(f"heuristic-vs-oracle: {hits}/{len(out)} picks within 1.1x of the fastest; "
          f"worst slowdown {max(r['slowdown'] for r in out):.3f}x")
    _write_csv("heuristic.csv", out)
    return 0


def cmd_bench(args):
    dtype = F64 if args.dtype == "f64" else F32
    peak, src = _peak_gbs()
    out = []
    for name, key in _sources(args):
        A, rows, gather = _measure_all(name, key, dtype, args.iters, args.warmup, args.seed,
                                       baseline=not args.no_baseline)
        print(f"=== {name} ({args.dtype}) m={A.m} nnz={A.nnz}; HBM peak {peak:.0f} GB/s ({src}), "
              f"gather ceiling {gather / 1e9:.1f} G/s ===")
        for _, r in rows:
            gf = f"{100 * r['gather_frac']:5.1f}% gather" if r["gather_frac"] != "" else " " * 12
            sp = f"  {r['speedup']:5.2f}x cuSPARSE" if r["speedup"] != "" else ""
            print(f"  {r['kernel']:16s} {r['median_ms'] * 1e3:9.2f} us  {r['gflops']:8.1f} GFLOP/s "
                  f"{r['bw_lo_gbs']:8.1f} GB/s  {100 * r['roofline_frac']:5.1f}% HBM  "
                  f"{gf}  cold {r['cold_ms'] * 1e3:8.2f} us{sp}")
            out.append(r)
    _write_csv("bench.csv", out)
    _write_gpu_info(peak, src)
    return 0


# results/accuracy.csv: the reference's columns (src/validate.cpp:210), then
# the row criterion this driver applies.
ACCURACY_COLUMNS = ["matrix", "kernel", "mode", "max_rel_err", "l2_rel_err", "max_abs_err",
                    "rows_checked", "rows_failed", "criterion"]
VALIDATE_MODES = [("fp32/fp32", F32, F32), ("fp32/fp64", F32, F64), ("fp64/fp64", F64, F64)]


def err_stats(yhat, ref):
    """The reference's ErrStats (src/validate.cpp:99-117): max over rows of
    |d| / max(|ref|, 1e-30), sqrt(sum d^2 / sum ref^2), max |d|."""
    yhat = np.asarray(yhat, np.float64)
    ref = np.asarray(ref, np.float64)
    d = np.abs(yhat - ref)
    den = float(np.dot(ref, ref))
    num = float(np.dot(d, d))
    return {"max_rel_err": float(np.max(d / np.maximum(np.abs(ref), 1e-30))) if ref.size else 0.0,
            "l2_rel_err": (num / den) ** 0.5 if den > 0 else num ** 0.5,
            "max_abs_err": float(d.max()) if d.size else 0.0}


def row_bound_failures(rowptr, colind, vals, x, ref, got, u, tol):
    """Rows of `got` outside max(tol*|ref|, 2*gamma_n(u)*sum_j |a_ij x_j|),
    n = the row's length, gamma_n = n*u / (1 - n*u): the reference GPU test's
    criterion (tests/test_cuda_correctness.cpp:53-56,88). `ref` is the exact
    (float64) product of the same stored values and x; returns the failing
    row indices."""
    m = rowptr.size - 1
    if m == 0:
        return np.zeros(0, np.int64)
    lens = np.diff(rowptr).astype(np.int64)
    rows = np.repeat(np.arange(m), lens)
    abs_sum = np.bincount(rows, weights=np.abs(np.asarray(vals, np.float64) * np.asarray(x, np.float64)[colind]),
                          minlength=m)
    nu = lens * u
    allowed = np.maximum(tol * np.abs(ref), 2.0 * (nu / (1.0 - nu)) * abs_sum)
    diff = np.abs(np.asarray(got, np.float64) - ref)
    bad = ~(diff <= allowed)  # NaN fails
    return np.flatnonzero(bad)


def scipy_product(A, vals, x):
    """y = A x by SciPy in float64 on the given stored values: an independent
    CPU product (SciPy's CSR matvec, as the reference's tools/reference.py
    uses it), not this library and not the oracle."""
    import scipy.sparse as sp
    M = sp.csr_matrix((np.asarray(vals, np.float64), A.colind, A.rowptr), shape=(A.m, A.n))
    return M @ np.asarray(x, np.float64)


def cmd_validate(args):
    """Every GPU kernel, in the reference's three precision modes, against
    SciPy's float64 y = A x (src/validate.cpp:190-250 validates the CPU
    kernels against SciPy the same way). Each result gets the reference's
    error statistics against SciPy on the original fp64 data, and must pass
    the per-row gamma_n criterion against SciPy's product of the values and x
    as the kernel stored them (fp32 storage rounds them first); kernels that
    keep csr_omp's order must also equal that product bit for bit in fp64.
    Writes results/accuracy.csv; exit status 1 on any failure."""
    import torch
    bad = 0
    out = []
    gate_ok = gate_total = 0
    for name, key in _sources(args):
        A = _load(key, args.seed)
        xh = generate_vector(999, A.n)
        y64 = scipy_product(A, A.values, xh)
        ctx = Context(0)
        for mode, dt, acc in VALIDATE_MODES:
            npd = np.float64 if dt == F64 else np.float32
            vals = np.ascontiguousarray(A.values, npd)
            xs = np.ascontiguousarray(xh, npd)
            exact = scipy_product(A, vals, xs)  # the stored operands, multiplied exactly as csr_omp orders them
            u = 2.0 ** -53 if acc == F64 else 2.0 ** -24
            tol = 1e-12 if acc == F64 else 1e-5
            M = DeviceMatrix(ctx, A, dt)
            x = torch.from_numpy(xs).cuda()
            y = torch.empty(max(A.m, 1), dtype=torch.float64 if acc == F64 else torch.float32, device="cuda")
            for label, k, lanes, block in VARIANTS:
                if key == 3 and k == BCSR:
                    continue  # 1M block rows of 50,000-entry rows: not a block format
                if not _usable(M, k, block):
                    continue
                y.fill_(float("nan"))
                M.spmv(x, y, kernel=k, lanes=lanes, block=block, acc=acc)
                torch.cuda.synchronize()
                got = y.cpu().numpy()[:A.m]
                fails = row_bound_failures(A.rowptr, A.colind, vals, xs, exact, got, u, tol)
                ok = fails.size == 0
                crit = f"gamma_n(2^{-53 if acc == F64 else -24}) or tol {tol:g}"
                if dt == F64 and acc == F64 and k in EXACT:
                    ok = ok and np.array_equal(got, exact)
                    crit = "bit-identical to SciPy (csr_omp order)"
                st = err_stats(got, y64)
                out.append({"matrix": name, "kernel": label, "mode": mode, **st, "rows_checked": A.m,
                            "rows_failed": int(fails.size), "criterion": crit})
                bad += not ok
                print(f"  {name:24s} {mode:9s} {label:16s} max_rel={st['max_rel_err']:.3e} "
                      f"l2_rel={st['l2_rel_err']:.3e} {'ok' if ok else 'FAIL (rows ' + str(fails[:3].tolist()) + ')'}")
                if mode == "fp64/fp64" and label == "csr_scalar":
                    gate_total += 1
                    gate_ok += st["max_rel_err"] < 1e-12
            M.close()
        ctx.close()
    assert not out or list(out[0]) == ACCURACY_COLUMNS
    _write_csv("accuracy.csv", out)
    print(f"[validate] fp64 GPU CSR within 1e-12 relative vs SciPy: {gate_ok}/{gate_total}")
    print("validate:", "ok" if bad == 0 else f"{bad} failures")
    return 1 if bad else 0


def _spmm_setup(key, dtype, k, seed=2024):
    import torch
    A = _load(key, seed)
    npd = np.float64 if dtype == F64 else np.float32
    ctx = Context(0)
    M = DeviceMatrix(ctx, A, dtype)
    X = torch.from_numpy(generate_vector(998, A.n * k).astype(npd).reshape(A.n, k)).cuda()
    Y = torch.empty(A.m, k, dtype=torch.float64 if dtype == F64 else torch.float32, device="cuda")
    return ctx, A, M, X, Y


def cmd_spmm(args):
    import torch
    dtype = F64 if args.dtype == "f64" else F32
    es = 8 if dtype == F64 else 4
    peak, src = _peak_gbs()
    k = args.k
    name, key = _sources(args)[0] if (args.matrix or args.all) else (WORKLOADS[5], 5)
    _, A, M, X, Y = _spmm_setup(key, dtype, k, args.seed)
    a_bytes = A.nnz * (es + 4) + (A.m + 1) * 4
    comp = a_bytes + A.n * k * es + A.m * k * es
    noreuse = a_bytes + A.nnz * k * es + A.m * k * es
    print(f"=== SpMM {name} ({args.dtype}) m={A.m} nnz={A.nnz} k={k}; HBM peak {peak:.0f} GB/s ({src}); "
          f"X {A.n * k * es / 1e6:.0f} MB ===")
    out = []
    base_ms = None
    if not args.no_baseline and A.nnz > 0:
        # The reference's SpMM baseline (cusparse_spmm, bench_main.cpp:700-722):
        # cuSPARSE CSR x dense through torch's sparse CSR product; comparison only.
        try:
            Ac = _torch_csr(A, dtype)
            for _ in range(args.warmup):
                Yc = torch.sparse.mm(Ac, X)
            ts = []
            for _ in range(args.iters):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                Yc = torch.sparse.mm(Ac, X)
                b.record()
                b.synchronize()
                ts.append(a.elapsed_time(b))
            base_ms = statistics.median(ts)
            M.spmm(X, Y, k, tile=64)
            torch.cuda.synchronize()
            diff = float((Yc - Y).abs().max()) / (float(Y.abs().max()) or 1.0)
            del Yc, Ac
            r = dict(matrix=name, precision=args.dtype, k=k, tile="cusparse_spmm", bucketed=0, median_ms=base_ms,
                     min_ms=min(ts), gflops=2 * A.nnz * k / (base_ms * 1e-3) / 1e9,
                     compulsory_gbs=comp / (base_ms * 1e-3) / 1e9, no_reuse_gbs=noreuse / (base_ms * 1e-3) / 1e9)
            r["frac_hbm_no_reuse"] = r["no_reuse_gbs"] / peak
            r["speedup"] = ""
            out.append(r)
            print(f"  cusparse_spmm     {base_ms:8.3f} ms  {r['gflops']:8.1f} GFLOP/s  "
                  f"(max |Y - Y_tile64| / max|Y| = {diff:.2e})")
        except Exception as e:  # noqa: BLE001 - the baseline is optional
            print(f"  cusparse_spmm: unavailable ({e})")
            base_ms = None
    for bucketed in (False, True):
        for tile in (16, 32, 64):
            for _ in range(args.warmup):
                M.spmm(X, Y, k, tile=tile, bucketed=bucketed)
            ts = []
            for _ in range(args.iters):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                M.spmm(X, Y, k, tile=tile, bucketed=bucketed)
                b.record()
                b.synchronize()
                ts.append(a.elapsed_time(b))
            med = statistics.median(ts)
            r = dict(matrix=name, precision=args.dtype, k=k, tile=tile, bucketed=int(bucketed),
                     median_ms=med, min_ms=min(ts), gflops=2 * A.nnz * k / (med * 1e-3) / 1e9,
                     compulsory_gbs=comp / (med * 1e-3) / 1e9, no_reuse_gbs=noreuse / (med * 1e-3) / 1e9)
            r["frac_hbm_no_reuse"] = r["no_reuse_gbs"] / peak
            r["speedup"] = base_ms / med if base_ms else ""
            sp = f"  {r['speedup']:5.2f}x cuSPARSE" if base_ms else ""
            print(f"  tile {tile:2d} {'bucketed' if bucketed else 'plain   '} {med:8.3f} ms  {r['gflops']:8.1f} GFLOP/s "
                  f"compulsory {r['compulsory_gbs']:7.1f} GB/s  no-reuse {r['no_reuse_gbs']:7.1f} GB/s "
                  f"({100 * r['frac_hbm_no_reuse']:5.1f}% HBM){sp}")
            out.append(r)
    _write_csv("spmm.csv", out)
    return 0


def cmd_profile(args):
    import torch
    dtype = F64 if args.dtype == "f64" else F32
    name, key = _sources(args)[0]
    if args.profile == "spmm":
        _, A, M, X, Y = _spmm_setup(key, dtype, args.k, args.seed)
        for _ in range(args.warmup):
            M.spmm(X, Y, args.k, tile=64)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            M.spmm(X, Y, args.k, tile=64)
        b.record()
        b.synchronize()
        print(f"spmm k={args.k} on {name}: "
              f"{a.elapsed_time(b) / max(1, args.steps) * 1e3:.2f} us per launch "
              f"({args.steps} launches after {args.warmup} warm-up)")
        return 0
    ctx, A, M, x, y, _ = _setup(key, dtype, args.seed)
    label = {v[0]: v for v in VARIANTS}
    if args.profile not in label:
        raise SystemExit(f"--profile expects one of {sorted(label)}")
    _, k, lanes, block = label[args.profile]
    M.prepare(k, block if k == BCSR else 0)
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        M.spmv(x, y, kernel=k, lanes=lanes, block=block)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        M.spmv(x, y, kernel=k, lanes=lanes, block=block)
    b.record()
    b.synchronize()
    print(f"{args.profile} on {name}: {a.elapsed_time(b) / max(1, args.steps) * 1e3:.2f} us "
          f"per launch ({args.steps} launches after {args.warmup} warm-up)")
    return 0


def _write_csv(name, rows):
    if not rows:
        return
    os.makedirs("results", exist_ok=True)
    keys = list(rows[0].keys())
    with open(os.path.join("results", name), "w", newline="") as f:
        wr = csv.DictWriter(f, fieldnames=keys)
        wr.writeheader()
        wr.writerows(rows)
    print(f"wrote results/{name}")


def _workload_id(text: str) -> int:
    """A seeded workload by id (1..5) or by name (spmvbench_b200.WORKLOADS)."""
    names = {v: k for k, v in WORKLOADS.items()}
    if text in names:
        return names[text]
    try:
        w = int(text)
    except ValueError:
        w = 0
    if w not in WORKLOADS:
        raise argparse.ArgumentTypeError(f"unknown workload {text!r}: one of 1-5 or {', '.join(names)}")
    return w


def main(argv=None):
    p = argparse.ArgumentParser(prog="python -m spmvbench_b200.driver")
    g = p.add_mutually_exclusive_group(required=True)
    g.add_argument("--stats", action="store_true")
    g.add_argument("--auto", action="store_true")
    g.add_argument("--bench", action="store_true")
    g.add_argument("--validate", action="store_true")
    g.add_argument("--spmm", action="store_true")
    g.add_argument("--profile", metavar="KERNEL")
    p.add_argument("--workload", type=_workload_id, nargs="+", default=[1, 2, 3, 4],
                   help="workload ids (1-5) or names (" + ", ".join(WORKLOADS.values()) + ")")
    p.add_argument("--matrix", nargs="+", metavar="FILE",
                   help="Matrix Market (.mtx) or CSR-cache (.csrbin) files instead of the seeded workloads")
    p.add_argument("--all", action="store_true", help="every .mtx file in $SPMVBENCH_DATA (default data/)")
    p.add_argument("--seed", type=int, default=2024, help="seed of the generated workloads")
    p.add_argument("--no-baseline", action="store_true",
                   help="--bench without the cuSPARSE comparison row (torch's sparse CSR SpMV)")
    p.add_argument("--dtype", choices=["f64", "f32"], default="f64")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--steps", type=int, default=1)
    p.add_argument("--k", type=int, default=64)
    a = p.parse_args(argv)
    if a.stats:
        return cmd_stats(a)
    if a.auto:
        return cmd_auto(a)
    if a.bench:
        return cmd_bench(a)
    if a.validate:
        return cmd_validate(a)
    if a.spmm:
        return cmd_spmm(a)
    return cmd_profile(a)


if __name__ == "__main__":
    sys.exit(main())
