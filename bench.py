#!/usr/bin/env python3
"""Benchmark of the SpMV hot path on B200: one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload: fp64 SpMV y = A x on the uniform-random matrix
(1,000,000 x 1,000,000, exactly 16 distinct sorted uniform columns per row,
values and x U(-1,1), seeded). A step is one product y = A x over the whole
matrix, inputs resident in HBM. At N GPUs the matrix's rows are split into N
nnz-balanced contiguous blocks (spmvb_partition_rows) and each rank computes
its block's rows with the full x resident: strong scaling, no collective on
the data path. `value` = 2*nnz / (the slowest rank's time per step). The
kernel is the one the B200 heuristic picks for the matrix. Each rank cycles
through C copies of its row block so that the matrix bytes touched between
two uses of a copy exceed the L2 (C * block bytes >= 1.5 * L2); the K timed
steps are captured once as a CUDA graph and replayed between two events.

Extra objects on the same line:
  roofline      HBM roofline of the SpMV kernel on one GPU (algorithmic bytes
                of the rank's block per launch / CUDA-event launch time, over
                MEASURED_PEAKS.json hbm_gbs)
  gather_roofline  the same launches against the device's random-gather
                ceiling (one 8-byte x gather per entry; the ceiling is
                measured live by spmvb_probe_gather_rate)
  cpu_baseline  the reference's own csr_omp (oracle/_ref, compiled from the
                reference sources; the C restatement if that is absent) on
                the same matrix, all host threads, rank 0 at N=1: the
                reference arm's command run in a separate process (50 steps)
  e2e           the same product through the host-buffer API: every rank
                copies its rows' slice of x in from pinned host memory, the
                slices are all-gathered over NVLink, and each rank's rows of y
                are written to pinned host memory, every step, inside the
                timed region (spmvb_dist_pipeline_submit, 3 calls in flight)
  spmm_k64      fp64 SpMM Y = A X, X 1,000,000 x 64, A's rows sharded as above
                and X replicated
  iterated      x <- A x over the row blocks, x slices exchanged each step by
                ncclAllGather and, separately, by the peer exchange (the SpMV
                stores its slice into every rank's x); `parity`: after 20
                steps of each exchange every rank's x equals a one-rank run of
                the same steps bit for bit (the ELL kernel sums in csr_omp
                order); a mismatch makes the run exit non-zero
  replicas      (N > 1) every rank runs its own full-size matrix: weak scaling
  workloads     (N = 1) every benchmark matrix: each kernel timed, the
                choose_spmv pick against the fastest, GFLOP/s and HBM
                fraction of the pick, the reference's own GPU kernels
                (oracle/_ref/libspmvref_cuda.so, its SpmvRunner protocol) on
                the same matrices where it can hold them, and SpMM k = 64 in
                fp64 and fp32 against the reference's spmm_csr_tiled
  clocks        nvidia-smi samples taken while the timed loop and a short
                untimed run of the same kernel just before it execute

--impl reference times the reference's CPU implementation (csr_omp) of the
same workload on the host cores (rank 0 only), with the reference's own
protocol (warm-up runs, then the median of timed runs), and prints the same
metric. It builds the matrix with the oracle's statement of the generator, so
it loads nothing of this library.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import os
import re
import statistics
import subprocess
import sys
import threading
import time

import numpy as np  # noqa: E402

# Every CPU this process may use, read before any OpenMP runtime starts: a
# runtime started with OMP_PROC_BIND set binds the calling thread to one CPU.
HOST_CPUS = sorted(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else None

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOAD = "uniform_1m_16_fp64"
METRIC = "fp64 SpMV GFLOP/s (uniform 1M x 1M, 16 nnz/row)"
SEED = 2024
X_SEED = 999
M_ROWS, NNZ = 1_000_000, 16_000_000
PARITY_STEPS = 20


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-workloads", action="store_true", help="skip the per-workload objects (N = 1)")
    p.add_argument("--soak-s", type=float, default=1.5, help="untimed run before the timed loop (clock sampling)")
    return p.parse_args()


def bench_config(world: int, kernel: str) -> dict:
    """The `config` object; identical in both arms but for `kernel`."""
    return {"workload": WORKLOAD, "m": M_ROWS, "n": M_ROWS, "nnz": NNZ,
            "partition": "whole matrix" if world == 1 else
            f"{world} nnz-balanced row blocks (spmvb_partition_rows), x replicated",
            "l2": "each rank cycles copies of its row block so >= 1.5x L2 of matrix bytes pass between two uses "
                  "of a copy (1 copy of 212 MB at N=1); x stays L2-resident",
            "kernel": kernel}


def host_threads() -> int:
    return len(HOST_CPUS) if HOST_CPUS else (os.cpu_count() or 1)


def prepare_cpu_run():
    """Before the oracle's OpenMP runtime first loads (a process without
    torch, whose own runtime would be picked up instead): all host CPUs in
    this thread's mask and the threads bound to neighbouring cores
    (OMP_PROC_BIND=close, read when the runtime starts)."""
    if HOST_CPUS:
        os.sched_setaffinity(0, HOST_CPUS)
    os.environ["OMP_PROC_BIND"] = "close"


def cpu_baseline_in_clean_process(steps: int) -> dict:
    """The reference arm's own command (`--impl reference`) in a separate
    process: the reference's csr_omp with the system OpenMP runtime, away
    from torch (which loads its own libgomp.so.1, already started unbound),
    so the CPU baseline and the reference arm are the same measurement."""
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "OMP_PROC_BIND")}
    out = subprocess.run([sys.executable, os.path.abspath(__file__), "--impl", "reference", "--steps", str(steps),
                          "--warmup", "3"], capture_output=True, text=True, timeout=600, env=env)
    line = next((ln for ln in out.stdout.splitlines() if ln.startswith("{")), None)
    if out.returncode != 0 or line is None:
        return {"unavailable": (out.stderr or out.stdout)[-300:]}
    d = json.loads(line)
    cpu = dict(d["cpu_baseline"])
    cpu["process"] = "separate process without torch: the same command as the reference arm"
    return cpu


def spmv_bytes(m, n, nnz, vbytes=8, ibytes=4, ybytes=8):
    """Compulsory traffic of CSR SpMV: values + colind + rowptr + x + y once
    (the reference's bw_lo model, bench/bench_main.cpp:449-457)."""
    return nnz * (vbytes + ibytes) + (m + 1) * ibytes + n * vbytes + m * ybytes


def kernel_bytes(S, kernel, M, m, n, nnz, es=8, block=4):
    """Compulsory bytes of the format `kernel` reads: ELL/HYB read row_lengths
    (m ints) instead of rowptr (bench/bench_main.cpp:661-667); BCSR its
    blocks (bench/bench_main.cpp:668-678)."""
    if kernel in (S.ELL, S.HYB):
        return nnz * (es + 4) + m * 4 + n * es + m * es
    if kernel == S.BCSR:
        b = 2 if block <= 2 else 4
        bn = M.info()["bcsr2_block_nnz" if b == 2 else "bcsr4_block_nnz"]
        return bn * (b * b * es + 4) + ((m + b - 1) // b + 1) * 4 + n * es + m * es
    return spmv_bytes(m, n, nnz, es, 4, es)


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic(kernel_name: str):
    """DRAM bytes per launch of `kernel_name` on the full headline matrix from
    the committed ncu summary (profiles/*.md line `dram_bytes_per_launch: N`)."""
    pdir = os.path.join(ROOT, "profiles")
    if not os.path.isdir(pdir):
        return None
    for fn in sorted(os.listdir(pdir)):
        if fn.startswith(kernel_name) and WORKLOAD in fn and fn.endswith(".md"):
            m = re.search(r"dram_bytes_per_launch:\s*([0-9]+)", open(os.path.join(pdir, fn)).read())
            if m:
                return int(m.group(1))
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples every 200 ms (read only)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", ",".join(str(g) for g in self.gpus), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [c.strip() for c in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        loaded = [s for s in sm if mx and s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------
def csr_omp_runner(m, n, rowptr, colind, values, x, threads):
    """A callable running csr_omp once: the reference's own code when
    oracle/_ref was built, else the C restatement; and its kind."""
    import oracle
    if oracle.ref_available():
        R = oracle.RefCsr(m, n, rowptr, colind, values)
        y = np.empty(m)
        return (lambda: R.spmv(x, np.float64, threads, out=y)), "reference"  # noqa: E731
    return (lambda: oracle.spmv_csr(m, rowptr, colind, values, x, np.float64, threads)), "port"  # noqa: E731


# Timed SpMVs per reference step: the host's memory bandwidth is shared with
# other tenants, so one step samples several runs.
RUNS_PER_STEP = 8


def time_csr_omp(run, warmup, runs=None, budget_s=None, min_runs=10, warm_s=1.0):
    """The reference bench's CPU protocol (bench/bench_main.cpp:474-487): warm-up
    runs (at least `warmup`, and for at least `warm_s` seconds), then timed runs
    (steady clock, each run timed alone), median. Either exactly `runs` timed
    runs, or runs until `budget_s` (at least `min_runs`, at most 500).
    Returns (median ms, mean ms, runs, min ms)."""
    w_end = time.perf_counter() + warm_s
    done = 0
    while done < warmup or time.perf_counter() < w_end:
        run()
        done += 1
    times = []
    t_end = time.perf_counter() + (budget_s or 0.0)
    while (len(times) < runs) if runs else (len(times) < min_runs or (time.perf_counter() < t_end and len(times) < 500)):
        t0 = time.perf_counter()
        run()
        times.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(times), statistics.fmean(times), len(times), min(times)


def host_state() -> dict:
    """What can make the same CPU run differ between two moments on one host:
    transparent huge pages (mode, and how much of this process they back),
    load average, and the cores' current clock (median over /proc/cpuinfo)."""
    st = {}
    try:
        st["thp"] = open("/sys/kernel/mm/transparent_hugepage/enabled").read().strip()
    except OSError:
        pass
    try:
        for ln in open("/proc/self/smaps_rollup"):
            if ln.startswith("AnonHugePages:"):
                st["anon_huge_kb"] = int(ln.split()[1])
    except OSError:
        pass
    try:
        st["loadavg"] = open("/proc/loadavg").read().split()[:3]
        mhz = [float(ln.split(":")[1]) for ln in open("/proc/cpuinfo") if ln.startswith("cpu MHz")]
        st["cpu_mhz_median"] = statistics.median(mhz) if mhz else None
    except (OSError, ValueError):
        pass
    return st


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    prepare_cpu_run()
    import oracle
    m, n, rp, ci, va = oracle.generate(2, SEED)
    x = oracle.generate_vector(X_SEED, n)
    threads = host_threads()
    run, kind = csr_omp_runner(m, n, rp, ci, va, x, threads)
    warm = max(3, args.warmup)
    ms, mean_ms, runs, min_ms = time_csr_omp(run, warm, runs=args.steps * RUNS_PER_STEP)
    gflops = 2.0 * (int(rp[m])) / (ms * 1e-3) / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": gflops, "unit": "GFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": warm, "ms_per_step": ms, "ms_per_step_mean": mean_ms,
        "ms_per_spmv_min": min_ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": bench_config(args.gpus, "csr_omp (spmv_csr_cpu, OpenMP static)"),
        "cpu_baseline": {"value": gflops, "unit": "GFLOP/s", "cores": threads, "kind": kind,
                         "omp_proc_bind": os.environ.get("OMP_PROC_BIND"), "host": host_state(),
                         "sample": f"full {WORKLOAD} SpMVs: {warm}+ warm-up runs over at least 1 s, then "
                                   f"{args.steps} steps of {RUNS_PER_STEP} runs, each run timed alone, median of the "
                                   f"{runs} runs (the reference bench's CPU protocol: warm-up, median of timed runs)",
                         "min_gflops": 2.0 * (int(rp[m])) / (min_ms * 1e-3) / 1e9},
        "e2e": {"value": gflops, "unit": "GFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------
def gpu_local_cpus(torch, device: int):
    """CPUs on the GPU's own NUMA node (from its PCI address in sysfs), or None."""
    try:
        p = torch.cuda.get_device_properties(device)
        addr = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        text = open(f"/sys/bus/pci/devices/{addr}/local_cpulist").read().strip()
        cpus = set()
        for part in text.split(","):
            a, _, b = part.partition("-")
            cpus.update(range(int(a), int(b or a) + 1))
        return sorted(cpus & os.sched_getaffinity(0)) or None
    except (AttributeError, OSError, ValueError):
        return None


def row_block(S, A, r0, r1):
    """Rows [r0, r1) of A as a CSR with global column indices."""
    p0, p1 = int(A.rowptr[r0]), int(A.rowptr[r1])
    return S.CsrMatrix(r1 - r0, A.n, (A.rowptr[r0:r1 + 1] - p0).astype(np.int32), A.colind[p0:p1],
                       A.values[p0:p1])


def graph_time_ms(torch, stream, launch, count, replays=1):
    """Per-launch ms of `count` launches of launch(i, stream) captured as one
    CUDA graph: median over `replays` replays, each between two events on
    `stream` (the stream the graph runs on)."""
    graph, cap = torch.cuda.CUDAGraph(), torch.cuda.Stream()
    cap.wait_stream(stream)
    with torch.cuda.graph(graph, stream=cap, capture_error_mode="relaxed"):
        for i in range(count):
            launch(i, cap)
    stream.wait_stream(cap)
    times = []
    for _ in range(replays):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        with torch.cuda.stream(stream):
            graph.replay()
        e1.record(stream)
        e1.synchronize()
        times.append(e0.elapsed_time(e1) / count)
    del graph
    return statistics.median(times)


def event_time_ms(torch, stream, launch, iters, warmup, flush=None):
    """The reference's SpmvRunner::run protocol (src/cuda/spmv_cuda.cu:466-486):
    one event pair around each launch, median; with `flush`, a write of a
    buffer larger than L2 before each launch (outside its event pair)."""
    for i in range(warmup):
        launch(i, stream)
    times = []
    for i in range(iters):
        if flush is not None:
            with torch.cuda.stream(stream):
                flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        launch(i, stream)
        e1.record(stream)
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    return statistics.median(times)


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ---- per-workload sweep (N = 1) ------------------------------------------------
SWEEP = [("banded_100k_hb4_fp64", 1, "f64"), ("uniform_1m_16_fp64", 2, "f64"), ("uniform_1m_16_fp32", 2, "f32"),
         ("powerlaw_1m_zipf2.1_fp64", 3, "f64"), ("bcsr4x4_500k_8blk_fp64", 4, "f64")]
REF_KERNEL_IDS = {"csr_scalar": 0, "csr_vector": 1, "csr_warp": 2, "csr_merge": 3, "ell": 4, "bcsr_4x4": 5}


def workload_sweep(torch, S, ctx, stream, A2, peak, flush, log):
    """Every benchmark matrix: every kernel timed warm (graph of 10 launches,
    median of 10 replays), the choose_spmv pick against the fastest, the pick
    cold (after an L2 flush), and the reference's own kernels beside it."""
    import oracle
    out = {}
    have_ref = oracle.ref_cuda_available()
    for name, which, dt in SWEEP:
        t0 = time.perf_counter()
        A = A2 if which == 2 else S.generate(which, seed=SEED)
        xh = S.generate_vector(X_SEED, A.n)
        dtype = S.F64 if dt == "f64" else S.F32
        es = 8 if dtype == S.F64 else 4
        npd = np.float64 if dtype == S.F64 else np.float32
        stats = S.row_stats(A)
        choice = S.choose_spmv(stats)
        vec_lanes = choice["lanes"] if choice["kernel"] == S.CSR_VECTOR else \
            min(32, max(2, 1 << max(0, math.ceil(math.log2(max(1.0, stats["mean_row_nnz"]))))))
        cands = [("csr_scalar", S.CSR_SCALAR, 1, 4), (f"csr_vector_l{vec_lanes}", S.CSR_VECTOR, vec_lanes, 4),
                 ("csr_warp", S.CSR_WARP, 1, 4), ("csr_merge", S.CSR_MERGE, 1, 4), ("ell", S.ELL, 1, 4),
                 ("hyb", S.HYB, 1, 4), ("bcsr_4x4", S.BCSR, 1, 4)]
        if choice["kernel"] == S.BCSR and choice["block_r"] <= 2:
            cands.append(("bcsr_2x2", S.BCSR, 1, 2))
        M = S.DeviceMatrix(ctx, A, dtype)
        x = torch.from_numpy(xh.astype(npd)).cuda()
        y = torch.empty(A.m, dtype=torch.float64 if dtype == S.F64 else torch.float32, device="cuda")
        times, skipped = {}, {}
        for label, k, lanes, block in cands:
            try:
                M.prepare(k, block if k == S.BCSR else 0)
            except S.SpmvbError as e:
                skipped[label] = str(e)
                continue

            def launch(i, s, k=k, lanes=lanes, block=block):
                M.spmv(x, y, kernel=k, lanes=lanes, block=block, stream=s)
            for i in range(3):
                launch(i, stream)
            times[label] = graph_time_ms(torch, stream, launch, 10, replays=10)
        pick_label = next(lb for lb, k, lanes, block in cands
                          if k == choice["kernel"] and (k != S.CSR_VECTOR or lanes == choice["lanes"])
                          and (k != S.BCSR or block == (2 if choice["block_r"] <= 2 else 4)))
        if pick_label not in times:
            raise RuntimeError(f"{name}: choose_spmv picked {pick_label}, which cannot run here: "
                               f"{skipped.get(pick_label)}")
        pk = next(c for c in cands if c[0] == pick_label)
        fastest = min(times, key=times.get)
        t_pick = times[pick_label]
        pick_bytes = kernel_bytes(S, pk[1], M, A.m, A.n, A.nnz, es, pk[3])

        def launch_pick(i, s):
            M.spmv(x, y, kernel=pk[1], lanes=pk[2], block=pk[3], stream=s)
        cold = event_time_ms(torch, stream, launch_pick, 10, 3, flush=flush)
        # The reference's SpmvRunner::run protocol, run in C++ by the library.
        ours_ref_protocol = M.spmv_time(x, y, kernel=pk[1], lanes=pk[2], block=pk[3], iters=20, warmup=5,
                                        stream=stream)["median_ms"]
        entry = {
            "m": A.m, "n": A.n, "nnz": A.nnz, "dtype": dt, "pick": pick_label, "rule": choice["reason"],
            "us": {k: round(v * 1e3, 2) for k, v in times.items()}, "unavailable": skipped or None,
            "fastest": fastest, "pick_over_fastest": t_pick / times[fastest],
            "gflops": 2.0 * A.nnz / (t_pick * 1e-3) / 1e9, "bytes_per_launch": pick_bytes,
            "hbm_frac": pick_bytes / (t_pick * 1e-3) / 1e9 / peak,
            "cold_us": cold * 1e3, "cold_gflops": 2.0 * A.nnz / (cold * 1e-3) / 1e9,
            "timed_as": "warm: graph of 10 launches, median of 10 replays; cold: one launch after a 256 MB "
                        "flush, median of 10",
        }
        if have_ref and dt == "f64" and which in (1, 2, 4):
            # The reference's SpmvRunner (eager ELL + BCSR uploads) on the same
            # matrix and x; its run(): per-launch event pairs, median. Not on
            # the power-law matrix, whose padded ELL (~600 GB) it cannot hold.
            R = oracle.RefCudaRunner(A.m, A.n, A.rowptr, A.colind, A.values, xh)
            ref_t = {}
            for label, kid in REF_KERNEL_IDS.items():
                ref_t[label], _ = R.run(kid, lanes=vec_lanes if kid == 1 else 4, block=4, iters=20, warmup=5)
            R.close()
            best = min(ref_t, key=ref_t.get)
            entry["reference_kernels"] = {
                "us": {k: round(v * 1e3, 2) for k, v in ref_t.items()}, "best": best,
                "ours_pick_same_protocol_us": ours_ref_protocol * 1e3,
                "speedup_vs_best": ref_t[best] / ours_ref_protocol,
                "protocol": "reference SpmvRunner::run: one event pair per launch, median of 20 after 5 warm-up; "
                            "ours by the same C++ loop (spmvb_spmv_time)"}
        M.close()
        del x, y
        out[name] = entry
        log(f"[bench] {name}: pick {pick_label} {t_pick * 1e3:.1f} us ({entry['gflops']:.0f} GFLOP/s, "
            f"{entry['hbm_frac']:.3f} HBM), fastest {fastest} {times[fastest] * 1e3:.1f} us "
            f"[{time.perf_counter() - t0:.1f} s]")
    out["spmm_uniform_1m_16_k64"] = spmm_sweep(torch, S, ctx, stream, A2, peak, log)
    return out


def spmm_sweep(torch, S, ctx, stream, A, peak, log):
    """SpMM Y = A X, k = 64, fp64 and fp32: every tile, plain and bucketed,
    per-launch median; the reference's spmm_csr_tiled_f64 beside the fp64 row."""
    import oracle
    k = 64
    Xh = S.generate_vector(X_SEED + 1, A.n * k).reshape(A.n, k)
    res = {}
    for dt in ("f64", "f32"):
        dtype = S.F64 if dt == "f64" else S.F32
        es = 8 if dt == "f64" else 4
        M = S.DeviceMatrix(ctx, A, dtype)
        X = torch.from_numpy(Xh.astype(np.float64 if dt == "f64" else np.float32)).cuda()
        Y = torch.empty(A.m, k, dtype=X.dtype, device="cuda")
        t = {}
        for tile in (16, 32, 64):
            for buck in (False, True):
                def launch(i, s, tile=tile, buck=buck):
                    M.spmm(X, Y, k, tile=tile, bucketed=buck, stream=s)
                t[f"t{tile}{'_bucketed' if buck else ''}"] = event_time_ms(torch, stream, launch, 7, 2)
        best = min(t, key=t.get)
        comp = A.nnz * (es + 4) + (A.m + 1) * 4 + A.n * k * es + A.m * k * es
        entry = {"dtype": dt, "us": {kk: round(v * 1e3, 1) for kk, v in t.items()}, "best": best,
                 "gflops": 2.0 * A.nnz * k / (t[best] * 1e-3) / 1e9, "compulsory_bytes": comp,
                 "hbm_frac_compulsory": comp / (t[best] * 1e-3) / 1e9 / peak,
                 "timed_as": "one event pair per launch, median of 7 after 2 warm-up"}
        if dt == "f64" and oracle.ref_cuda_available():
            rt = {}
            for tile in (16, 32, 64):
                for bal in (False, True):
                    _, ms = oracle.ref_cuda_spmm(A.m, A.n, A.rowptr, A.colind, A.values, Xh, k, tile=tile,
                                                 balanced=bal, iters=5, warmup=2)
                    rt[f"t{tile}{'_bucketed' if bal else ''}"] = ms
            rb = min(rt, key=rt.get)
            entry["reference_kernels"] = {"us": {kk: round(v * 1e3, 1) for kk, v in rt.items()}, "best": rb,
                                          "speedup_vs_best": rt[rb] / t[best],
                                          "protocol": "reference spmm_csr_tiled_f64: per-launch events, median"}
        res[dt] = entry
        M.close()
        del X, Y
        log(f"[bench] spmm k=64 {dt}: best {best} {t[best] * 1e3:.0f} us ({entry['gflops']:.0f} GFLOP/s)")
    return res


# ------------------------------------------------------------------------------
def main():
    args = parse()
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    import torch
    import torch.distributed as dist

    import spmvbench_b200 as S

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    # With several ranks, each runs on its GPU's NUMA node, so the pinned host
    # buffers of the e2e loop (first touched here) sit next to its PCIe link.
    # One rank keeps every core (the CPU baseline uses them all).
    host_cpus = gpu_local_cpus(torch, local) if world > 1 else None
    if host_cpus:
        os.sched_setaffinity(0, host_cpus)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    def log(msg):
        if rank == 0:
            print(msg, file=sys.stderr, flush=True)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def all_true(ok: bool) -> bool:
        if world == 1:
            return ok
        t = torch.tensor([1 if ok else 0], dtype=torch.int32, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        return bool(t.item())

    ctx = S.Context(local)
    stream = torch.cuda.current_stream()
    gpu = S.query_gpu(local)
    peak, peak_src = measured_peak()

    # ---- the matrix, its row blocks and this rank's block ----
    t_setup = time.perf_counter()
    A = S.generate(2, seed=SEED)
    xh = S.generate_vector(X_SEED, A.n)
    stats = S.row_stats(A)
    choice = S.choose_spmv(stats)
    kernel, lanes, block = choice["kernel"], choice["lanes"], choice["block_r"]
    kname = {S.CSR_SCALAR: "csr_scalar_warp", S.CSR_MERGE: "csr_merge", S.CSR_VECTOR: "csr_vector",
             S.CSR_WARP: "csr_vector", S.ELL: "ell_rows", S.HYB: "hyb_rows", S.BCSR: "bcsr_rows"}[kernel]
    bounds = S.partition_rows(A.rowptr, world)
    r0, r1 = int(bounds[rank]), int(bounds[rank + 1])
    B = row_block(S, A, r0, r1)
    block_bytes = kernel_bytes(S, kernel, None, B.m, B.n, B.nnz) if kernel != S.BCSR else None
    # Copies of the block's matrix arrays (its bytes less x and y, which every
    # copy shares or rewrites) such that 1.5x the L2 of them pass between two
    # uses of a copy.
    matrix_bytes = (block_bytes - 8 * (B.n + B.m)) if block_bytes else 0
    copies = max(1, min(16, math.ceil(1.5 * gpu["l2_bytes"] / max(1, matrix_bytes))))
    mats = []
    for _ in range(copies):
        Mc = S.DeviceMatrix(ctx, B, S.F64)
        Mc.prepare(kernel, block if kernel == S.BCSR else 0)
        mats.append(Mc)
    if block_bytes is None:
        block_bytes = kernel_bytes(S, kernel, mats[0], B.m, B.n, B.nnz, 8, block)
    x = torch.from_numpy(xh).cuda()
    ys = [torch.empty(max(B.m, 1), dtype=torch.float64, device="cuda") for _ in range(copies)]
    log(f"[bench] setup {time.perf_counter() - t_setup:.1f} s: rank 0 rows [{r0}, {r1}), {copies} copies, "
        f"kernel {S.kernel_name(kernel)}")

    def step(i, s):
        c = i % copies
        mats[c].spmv(x, ys[c], kernel=kernel, lanes=lanes, block=block, stream=s)

    for i in range(args.warmup):
        step(i, stream)
    barrier()
    sampler = ClockSampler(list(range(world)) if rank == 0 else [])
    if rank == 0:
        sampler.start()
    t_soak = time.perf_counter() + args.soak_s
    i = 0
    while time.perf_counter() < t_soak:  # untimed, same kernel, keeps clocks at their loaded state
        for _ in range(20):
            step(i, stream)
            i += 1
        torch.cuda.synchronize()
    # The K timed steps are captured once as a CUDA graph and replayed: the
    # same K launches, without host launch gaps between them (launches are
    # counted when captured; the replay runs each once).
    launches0 = S.launch_count()
    graph, cap = torch.cuda.CUDAGraph(), torch.cuda.Stream()
    cap.wait_stream(stream)
    with torch.cuda.graph(graph, stream=cap, capture_error_mode="relaxed"):
        for i in range(args.steps):
            step(i, cap)
    launches = S.launch_count() - launches0
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    with torch.cuda.stream(stream):
        graph.replay()
    ev1.record(stream)
    ev1.synchronize()
    barrier()
    clocks = sampler.stop() if rank == 0 else None
    del graph
    ms_rank = ev0.elapsed_time(ev1) / args.steps
    ms = max_over_ranks(ms_rank)
    if world > 1:
        lt = torch.tensor([launches], dtype=torch.int64, device="cuda")
        dist.all_reduce(lt)
        launches = int(lt.item())
    gflops = 2.0 * A.nnz / (ms * 1e-3) / 1e9
    achieved = block_bytes / (ms_rank * 1e-3) / 1e9
    # The device's random-gather ceiling (one 8-byte gather per entry from
    # the L2-resident x), measured live on this GPU.
    gather_peak = ctx.gather_rate(A.n, A.nnz)
    gathers_achieved = B.nnz / (ms_rank * 1e-3)
    y_dev = ys[0][:B.m].cpu().numpy().copy()
    log(f"[bench] product: {ms * 1e3:.2f} us per step (rank 0 {ms_rank * 1e3:.2f}), {gflops:.0f} GFLOP/s")

    # ---- the row-sharded matrix handle: e2e product and iterated x <- A x ----
    uid = None
    if world > 1:
        obj = [S.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        uid = obj[0]
    D = S.DistMatrix(ctx, world, rank, uid, A, bounds, S.F64)

    # e2e: per step, each rank's slice of x in from pinned host memory, the
    # slices all-gathered over NVLink, the rank's rows of y out to pinned
    # host memory.
    depth = 3
    xs = torch.from_numpy(xh[r0:r1].copy()).pin_memory()
    yps = [torch.empty(max(B.m, 1), dtype=torch.float64).pin_memory() for _ in range(depth)]
    pipe = S.DistPipeline(D, depth=depth)
    for i in range(depth):
        pipe.submit(xs.numpy(), yps[i].numpy(), kernel=kernel, lanes=lanes)
    pipe.wait()
    barrier()
    launches_e2e0 = S.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    pipe.fork(stream)
    h0 = time.perf_counter()
    for i in range(args.steps):
        pipe.submit(xs.numpy(), yps[i % depth].numpy(), kernel=kernel, lanes=lanes)
    host_submit_ms = (time.perf_counter() - h0) * 1e3 / args.steps
    pipe.join(stream)
    e1.record(stream)
    e1.synchronize()
    pipe.wait()
    barrier()
    launches_e2e = S.launch_count() - launches_e2e0
    pipe.close()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    e2e_same = all_true(bool(np.array_equal(yps[(args.steps - 1) % depth].numpy()[:B.m], y_dev)))
    e2e = {"value": 2.0 * A.nnz / (e2e_ms * 1e-3) / 1e9, "unit": "GFLOP/s", "ms_per_step": e2e_ms,
           "h2d_bytes_per_step": int(A.n * 8), "d2h_bytes_per_step": int(A.m * 8),
           "h2d_bytes_per_rank": int(B.m * 8), "d2h_bytes_per_rank": int(B.m * 8),
           "api": "spmvb_dist_pipeline_submit, 3 calls in flight: every step each rank copies its rows' slice "
                  "of x in from pinned host memory, the slices are all-gathered on the devices (ncclAllGather), "
                  "and the kernel writes the rank's rows of y into pinned host memory",
           "kernel_launches": int(launches_e2e), "y_equals_device_product": e2e_same,
           "host_submit_ms_per_step": max_over_ranks(host_submit_ms)}

    # iterated x <- A x: timing of both exchanges, then parity
    it_steps = 10 * args.steps

    def time_iterated():
        D.set_x(xh / 4.0)
        D.iterate(args.warmup, kernel=kernel, lanes=lanes, stream=stream)
        barrier()
        kms, sms = D.iterate_timed(it_steps, kernel=kernel, lanes=lanes, stream=stream)  # eager, per-step marks
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        D.iterate(it_steps, kernel=kernel, lanes=lanes, stream=stream)  # graph replays where available
        b.record(stream)
        b.synchronize()
        barrier()
        return (max_over_ranks(a.elapsed_time(b) / it_steps), max_over_ranks(sms / it_steps),
                max_over_ranks(kms / it_steps))

    def parity_digest():
        D.set_x(xh)
        D.iterate(PARITY_STEPS, kernel=kernel, lanes=lanes, stream=stream)
        return digest(D.get_x())

    def iterated_line(times, exchange):
        t_ms, eager_ms, kms = times
        return {"value": 2.0 * A.nnz / (t_ms * 1e-3) / 1e9, "unit": "GFLOP/s", "ms_per_step": t_ms,
                "eager_ms_per_step": eager_ms, "kernel_ms_per_step": kms, "exchange": exchange}

    by_exchange = {"nccl": iterated_line(time_iterated(), "ncclAllGather" if world > 1 else "device copy")}
    digests = {"nccl": parity_digest()}
    try:
        D.enable_peer(stream=stream)
        by_exchange["peer"] = iterated_line(time_iterated(), "SpMV stores into every rank's x (CUDA IPC), "
                                            "steps replayed as a CUDA graph")
        digests["peer"] = parity_digest()
    except S.SpmvbError as e:
        by_exchange["peer"] = {"unavailable": str(e)}
    D.close()
    # The same steps on one rank holding the whole matrix.
    D1 = S.DistMatrix(ctx, 1, 0, None, A, np.array([0, A.m], np.int32), S.F64)
    D1.set_x(xh)
    D1.iterate(PARITY_STEPS, kernel=kernel, lanes=lanes, stream=stream)
    one = digest(D1.get_x())
    D1.close()
    parity = {ex: all_true(d == one) for ex, d in digests.items()}
    parity["steps"] = PARITY_STEPS
    parity["against"] = "one rank holding the whole matrix, same kernel and steps; sha256 of x on every rank"
    best = min((v for v in by_exchange.values() if "ms_per_step" in v), key=lambda v: v["ms_per_step"])
    iterated = dict(best, bounds=bounds.tolist(), scaling="strong", steps=it_steps, by_exchange=by_exchange,
                    parity=parity)

    # ---- SpMM k = 64: A's rows sharded, X replicated ----
    k = 64
    Xd = torch.from_numpy(S.generate_vector(X_SEED + 1, A.n * k).reshape(A.n, k)).cuda()
    Yd = torch.empty(max(B.m, 1), k, dtype=torch.float64, device="cuda")
    for _ in range(args.warmup):
        mats[0].spmm(Xd, Yd, k, tile=64, stream=stream)
    barrier()
    spmm_steps = max(3, args.steps // 5)
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(spmm_steps):
        mats[0].spmm(Xd, Yd, k, tile=64, stream=stream)
    s1.record(stream)
    s1.synchronize()
    barrier()
    spmm_ms = max_over_ranks(s0.elapsed_time(s1) / spmm_steps)
    spmm_bytes = A.nnz * 12 + (A.m + 1) * 4 + A.n * k * 8 + A.m * k * 8
    spmm = {"value": 2.0 * A.nnz * k / (spmm_ms * 1e-3) / 1e9, "unit": "GFLOP/s", "k": k, "tile": 64,
            "ms_per_step": spmm_ms, "steps": spmm_steps,
            "compulsory_gbs_per_gpu": spmm_bytes / world / (spmm_ms * 1e-3) / 1e9}
    del Xd, Yd
    for Mc in mats:
        Mc.close()

    # ---- replicas: every rank its own full matrix (weak scaling), N > 1 ----
    replicas = None
    if world > 1:
        Ar = S.generate(2, seed=SEED + rank)
        Mr = S.DeviceMatrix(ctx, Ar, S.F64)
        Mr.prepare(kernel, 0)
        yr = torch.empty(Ar.m, dtype=torch.float64, device="cuda")

        def rstep(i, s):
            Mr.spmv(x, yr, kernel=kernel, lanes=lanes, block=block, stream=s)
        for i in range(args.warmup):
            rstep(i, stream)
        barrier()
        rms = max_over_ranks(graph_time_ms(torch, stream, rstep, args.steps))
        replicas = {"value": world * 2.0 * Ar.nnz / (rms * 1e-3) / 1e9, "unit": "GFLOP/s", "ms_per_step": rms,
                    "scaling": "weak", "what": "every rank its own 1M x 1M, 16/row matrix (seed + rank)"}
        Mr.close()
        del yr

    # ---- N = 1: every workload, and the CPU baseline ----
    workloads = None
    cpu = None
    if rank == 0 and world == 1:
        if not args.no_workloads:
            flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
            workloads = workload_sweep(torch, S, ctx, stream, A, peak, flush, log)
            del flush
        if not args.no_cpu_baseline:
            cpu = cpu_baseline_in_clean_process(50)

    if rank == 0:
        full_traffic = profiled_traffic(kname)
        traffic = None if full_traffic is None else int(round(full_traffic * B.nnz / A.nnz))
        line = {
            "metric": METRIC, "value": gflops, "unit": "GFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": bench_config(world, S.kernel_name(kernel)),
            "details": {"lanes": lanes, "rule": choice["reason"], "rank0_rows": [r0, r1], "rank0_nnz": B.nnz,
                        "copies_per_rank": copies, "bytes_per_launch_rank0": block_bytes,
                        "timed_as": "K steps captured as one CUDA graph, replayed once between two events; "
                                    "max over ranks",
                        "host_cpus_per_rank": len(host_cpus) if host_cpus else None},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": peak_src, "per": "GPU (rank 0's row block)",
                         "traffic": traffic, "kernel": kname,
                         "traffic_source": None if traffic is None else
                         "ncu dram bytes per launch on the full matrix, scaled by the block's share of nnz"},
            "gather_roofline": {"achieved": gathers_achieved, "peak": gather_peak, "unit": "gathers/s",
                                "frac": gathers_achieved / gather_peak,
                                "peak_source": "measured live (spmvb_probe_gather_rate)"},
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches), "clocks": clocks,
            "spmm_k64": spmm, "iterated": iterated, "replicas": replicas, "workloads": workloads,
        }
        print(json.dumps(line), flush=True)
    ok = e2e_same and all(v for kk, v in parity.items() if kk in ("nccl", "peer"))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if not ok:
        print("bench: multi-rank results differ from the one-rank run (see iterated.parity / e2e)",
              file=sys.stderr)
        return 3
    return 0


if __name__ == "__main__":
    sys.exit(main())
