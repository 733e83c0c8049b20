"""Behaviour of the C ABI on the GPU: argument checks reject bad buffers
before any kernel can touch them, the reference's clamping of lanes / block
/ tile is kept, launches are counted, and the single-rank distributed path
iterates exactly like the oracle."""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import oracle
import spmvbench_b200 as S
from gpu_util import assert_bitwise, assert_rows_within_bound, oracle_y, run_spmv

pytestmark = pytest.mark.gpu


def small(ctx, dtype=S.F64):
    A = S.generate(2, seed=71, scale_rows=1000)
    return A, S.DeviceMatrix(ctx, A, dtype)


def test_host_pointer_rejected(ctx):
    A, M = small(ctx)
    x_host = torch.zeros(A.n, dtype=torch.float64)  # CPU memory
    y = torch.zeros(A.m, dtype=torch.float64, device="cuda")
    with pytest.raises(S.SpmvbError) as e:
        M.spmv(x_host, y)
    assert e.value.status == 1 and "host memory" in str(e.value)


def test_undersized_buffer_rejected(ctx):
    A, M = small(ctx)
    big = torch.zeros(1 << 23, dtype=torch.float64, device="cuda")  # 64 MiB allocation
    x = torch.zeros(A.n, dtype=torch.float64, device="cuda")
    tail = big[(1 << 23) - 10:]  # 10 entries before the end of the allocation
    with pytest.raises(S.SpmvbError) as e:
        M.spmv(x, tail)
    assert e.value.status == 1 and "bytes" in str(e.value)


def test_bad_arguments(ctx):
    A, M = small(ctx)
    x = torch.zeros(A.n, dtype=torch.float64, device="cuda")
    y = torch.zeros(A.m, dtype=torch.float64, device="cuda")
    with pytest.raises(S.SpmvbError) as e:
        M.spmv(x, y, kernel=17)
    assert e.value.status == 1
    with pytest.raises(S.SpmvbError) as e:
        M.spmv(x, y.float(), acc=S.F32)  # fp64 storage, fp32 accumulation
    assert e.value.status == 3


def test_reference_clamping_of_lanes_block_tile(ctx):
    A, M = small(ctx)
    x = S.generate_vector(72, A.n)
    # lanes outside {2,4,8,16} -> 32 (src/cuda/spmv_cuda.cu:415-419)
    assert_bitwise(run_spmv(M, x, S.CSR_VECTOR, lanes=32), run_spmv(M, x, S.CSR_VECTOR, lanes=7), "lanes")
    # block <= 2 -> 2x2, else 4x4 (src/cuda/spmv_cuda.cu:449-457)
    assert_bitwise(run_spmv(M, x, S.BCSR, block=2), run_spmv(M, x, S.BCSR, block=1), "block")
    assert_bitwise(run_spmv(M, x, S.BCSR, block=4), run_spmv(M, x, S.BCSR, block=9), "block")
    k = 8
    B = torch.from_numpy(S.generate_vector(73, A.n * k).reshape(A.n, k)).cuda()
    Y1 = torch.empty(A.m, k, dtype=torch.float64, device="cuda")
    Y2 = torch.empty_like(Y1)
    M.spmm(B, Y1, k, tile=32)
    M.spmm(B, Y2, k, tile=48)  # anything else -> 32 (src/cuda/spmm_cuda.cu:155-168)
    torch.cuda.synchronize()
    assert torch.equal(Y1, Y2)


def test_launch_count_and_info(ctx):
    A, M = small(ctx)
    x = S.generate_vector(74, A.n)
    run_spmv(M, x, S.CSR_SCALAR)  # first call also builds the row partition
    before = S.launch_count()
    run_spmv(M, x, S.CSR_SCALAR)
    assert S.launch_count() == before + 1
    M.prepare(S.BCSR, 4)
    info = M.info()
    _, bci, _ = oracle.csr_to_bcsr(A.m, A.n, 4, A.rowptr, A.colind, A.values)
    assert info["bcsr4_block_nnz"] == bci.size and info["bcsr2_block_nnz"] == -1
    assert info["ell_padded_nnz"] == A.m * 16 and info["ell_touched_nnz"] == A.nnz
    assert info["device_bytes"] > A.nnz * 12
    g = S.query_gpu(0)
    assert g["major"] >= 10 and g["sm_count"] > 0


def test_single_rank_iteration_matches_oracle(ctx):
    A = S.generate(2, seed=75, scale_rows=50000)
    x0 = S.generate_vector(76, A.n)
    bounds = S.partition_rows(A.rowptr, 1)
    D = S.DistMatrix(ctx, 1, 0, None, A, bounds, S.F64)
    D.set_x(x0)
    D.iterate(3, kernel=S.CSR_SCALAR)
    got = D.get_x()
    x = x0
    for _ in range(3):
        x = oracle_y(A, x, S.F64, S.F64)
    assert_bitwise(x, got, "iterated")
    kms, sms = D.iterate_timed(2, kernel=S.CSR_SCALAR)
    assert 0 < kms <= sms
    D.close()


@pytest.mark.parametrize("exchange", ["nccl", "peer"])
def test_power_iteration_single_rank(ctx, exchange):
    """Power iteration x <- A x / ||A x|| on the sharded handle (one rank, both
    exchanges): the eigenvalue estimate and x follow a CPU power iteration
    built on the oracle's csr_omp within 1e-12, and a rerun is bit-identical."""
    A = S.generate(2, seed=86, scale_rows=40000)
    x0 = S.generate_vector(87, A.n)
    D = S.DistMatrix(ctx, 1, 0, None, A, S.partition_rows(A.rowptr, 1), S.F64)
    if exchange == "peer":
        D.enable_peer()
    runs = []
    for _ in range(2):
        D.set_x(x0)
        lam = D.power_iterate(12, kernel=S.ELL)
        runs.append((lam, D.get_x()))
    assert runs[0][0] == runs[1][0]
    assert_bitwise(runs[0][1], runs[1][1], "power iteration rerun")
    x = x0.copy()
    for _ in range(12):
        y = oracle_y(A, x, S.F64, S.F64)
        ref_lam = float(np.sqrt(np.dot(y, y)))
        x = y / ref_lam
    assert abs(runs[0][0] - ref_lam) <= 1e-12 * ref_lam
    np.testing.assert_allclose(runs[0][1], x, rtol=1e-11, atol=1e-14)
    D.close()


@pytest.mark.parametrize("depth,kernel", [(1, "ELL"), (3, "ELL"), (3, "CSR_MERGE")])
def test_dist_pipeline_single_rank_matches_oracle(ctx, depth, kernel):
    """The row-sharded host-buffer product with one rank: 6 calls with
    different x (pinned) in flight, each y equal to csr_omp (bit for bit
    for ELL, through staged y for the merge path within gamma_n)."""
    k = getattr(S, kernel)
    A = S.generate(2, seed=84, scale_rows=70000)
    D = S.DistMatrix(ctx, 1, 0, None, A, S.partition_rows(A.rowptr, 1), S.F64)
    P = S.DistPipeline(D, depth=depth)
    xs = [torch.from_numpy(S.generate_vector(85 + i, A.n)).pin_memory() for i in range(6)]
    ys = [torch.full((A.m,), float("nan"), dtype=torch.float64).pin_memory() for _ in range(6)]
    for i in range(6):
        P.submit(xs[i].numpy(), ys[i].numpy(), kernel=k)
    P.wait()
    for i in range(6):
        ref = oracle_y(A, xs[i].numpy(), S.F64, S.F64)
        if k == S.CSR_MERGE:
            assert_rows_within_bound(A, xs[i].numpy(), ref, ys[i].numpy(), S.F64, S.F64, f"call {i}")
        else:
            assert_bitwise(ref, ys[i].numpy(), f"call {i}")
    with pytest.raises(ValueError):
        P.submit(xs[0].numpy()[:10], ys[0].numpy(), kernel=k)
    P.close()
    D.close()


def test_dist_pipeline_outlived_by_nothing(ctx):
    """Destroying the dist handle before its host-buffer pipeline lets the
    pipeline's calls in flight finish, after which the pipeline's calls fail
    with an error (not a crash) and its destroy still succeeds."""
    A = S.generate(2, seed=89, scale_rows=30000)
    D = S.DistMatrix(ctx, 1, 0, None, A, S.partition_rows(A.rowptr, 1), S.F64)
    P = S.DistPipeline(D, depth=2)
    x = torch.from_numpy(S.generate_vector(90, A.n)).pin_memory()
    y = torch.full((A.m,), float("nan"), dtype=torch.float64).pin_memory()
    P.submit(x.numpy(), y.numpy(), kernel=S.ELL)
    D.close()
    assert_bitwise(oracle_y(A, x.numpy(), S.F64, S.F64), y.numpy(), "call finished before the handle went")
    with pytest.raises(S.SpmvbError):
        P.submit(x.numpy(), y.numpy(), kernel=S.ELL)
    with pytest.raises(S.SpmvbError):
        P.wait()
    P.close()


@pytest.mark.parametrize("depth", [1, 3])
def test_pipeline_streams_host_buffers(ctx, depth):
    """Streamed host-buffer SpMV: 7 calls with different x and separate y
    buffers (pinned), several in flight, each equal to csr_omp bit for bit;
    fork/join order them against a caller's stream."""
    A = S.generate(2, seed=82, scale_rows=80000)
    M = S.DeviceMatrix(ctx, A, S.F64)
    P = S.Pipeline(M, depth=depth)
    xs = [torch.from_numpy(S.generate_vector(83 + i, A.n)).pin_memory() for i in range(7)]
    ys = [torch.full((A.m,), float("nan"), dtype=torch.float64).pin_memory() for _ in range(7)]
    s = torch.cuda.Stream()
    P.fork(s)
    for i in range(7):
        P.submit(xs[i].numpy(), ys[i].numpy(), kernel=S.ELL if i % 2 else S.CSR_SCALAR)
    P.join(s)
    s.synchronize()
    P.wait()
    for i in range(7):
        assert_bitwise(oracle_y(A, xs[i].numpy(), S.F64, S.F64), ys[i].numpy(), f"pipeline call {i}")
    P.close()


def test_pipeline_every_kernel_pinned_and_pageable_y(ctx):
    """Pipeline calls on every kernel, y alternating between pinned buffers
    (written by the kernel directly, except the merge path) and pageable
    ones (staged and copied), against the device-buffer call bit for bit."""
    A = S.generate(3, seed=86, scale_rows=50000)
    M = S.DeviceMatrix(ctx, A, S.F64)
    x = torch.from_numpy(S.generate_vector(87, A.n)).pin_memory()
    xd = x.cuda()
    calls = [(S.CSR_SCALAR, 1, 4), (S.CSR_VECTOR, 8, 4), (S.CSR_WARP, 1, 4), (S.CSR_MERGE, 1, 4),
             (S.HYB, 1, 4), (S.BCSR, 1, 2), (S.BCSR, 1, 4), (S.CSR_MERGE, 1, 4)]
    P = S.Pipeline(M, depth=3)
    outs = []
    for i, (k, lanes, block) in enumerate(calls):
        y = (torch.full((A.m,), float("nan"), dtype=torch.float64).pin_memory().numpy() if i % 2 == 0
             else np.full(A.m, np.nan))
        P.submit(x.numpy(), y, kernel=k, lanes=lanes, block=block)
        outs.append(y)
    P.wait()
    for (k, lanes, block), y in zip(calls, outs):
        yd = torch.empty(A.m, dtype=torch.float64, device="cuda")
        M.spmv(xd, yd, kernel=k, lanes=lanes, block=block)
        torch.cuda.synchronize()
        assert_bitwise(yd.cpu().numpy(), y, f"pipeline {S.kernel_name(k)} lanes={lanes} block={block}")
    P.close()


@pytest.mark.parametrize("kernel", ["ELL", "CSR_MERGE", "CSR_SCALAR"])
def test_single_rank_peer_exchange(ctx, kernel):
    """Peer exchange with one rank: the SpMV writes the next x itself (fused
    for ELL, SpMV + copy kernel otherwise); set_x between iterations restarts
    from a new x. Thread-per-row kernels stay bit-identical to csr_omp."""
    k = getattr(S, kernel)
    A = S.generate(2, seed=78, scale_rows=60000)
    D = S.DistMatrix(ctx, 1, 0, None, A, S.partition_rows(A.rowptr, 1), S.F64)
    D.enable_peer()
    assert D.exchange == "peer"
    for seed, iters in ((79, 3), (80, 2)):
        x0 = S.generate_vector(seed, A.n)
        D.set_x(x0)
        D.iterate(iters, kernel=k)
        got = D.get_x()
        x = x0
        for _ in range(iters):
            x = oracle_y(A, x, S.F64, S.F64)
        if k == S.CSR_MERGE:
            np.testing.assert_allclose(got, x, rtol=1e-9, atol=1e-12)
        else:
            assert_bitwise(x, got, f"peer {kernel}")
    kms, sms = D.iterate_timed(2, kernel=k)
    assert 0 < kms <= sms
    if k == S.ELL:
        # 5 steps: one eager step, then two replays of the captured 2-step
        # graph; every replayed kernel is counted.
        before = S.launch_count()
        D.iterate(5, kernel=k)
        assert S.launch_count() - before == 5
    x0 = S.generate_vector(81, A.n)
    D.set_x(x0)
    D.iterate(7, kernel=k)
    x = x0
    for _ in range(7):
        x = oracle_y(A, x, S.F64, S.F64)
    if k == S.CSR_MERGE:
        np.testing.assert_allclose(D.get_x(), x, rtol=1e-9, atol=1e-12)
    else:
        assert_bitwise(x, D.get_x(), f"peer {kernel} graph")
    ctx.check()
    D.close()


def test_bounded_wait_reports_timeout(ctx):
    """Failure detection on the GPU: a wait that nothing will satisfy gives up
    after its limit, the kernel records it, and the host gets
    SPMVB_ERR_TIMEOUT; the context stays usable afterwards."""
    lib = S.load()
    assert lib.spmvb_selftest_wait_timeout(ctx.handle) == 7
    assert b"bounded wait" in lib.spmvb_last_error()
    ctx.check()  # the error word was cleared
    A, M = small(ctx)
    x = S.generate_vector(77, A.n)
    assert_bitwise(oracle_y(A, x, S.F64, S.F64), run_spmv(M, x, S.CSR_SCALAR), "after timeout")
    ctx.check()


_NEVER_JOINS = r"""
import os, sys
sys.path.insert(0, os.environ["SPMVB_ROOT"])
import spmvbench_b200 as S
ctx = S.Context(0)
A = S.generate(2, seed=1, scale_rows=1000)
b = S.partition_rows(A.rowptr, 2)
try:
    S.DistMatrix(ctx, 2, 0, S.nccl_unique_id(), A, b, S.F64)   # rank 1 never starts
    print("NO-ERROR")
except S.SpmvbError as e:
    print("STATUS", e.status)
"""


def test_rank_that_never_joins_times_out(tmp_path):
    """Failure detection on the host: communicator set-up is non-blocking and
    bounded, so a missing peer gives SPMVB_ERR_TIMEOUT, not a hang. Only the
    bootstrap waits; no collective is ever launched on the GPU."""
    env = dict(os.environ, SPMVB_NCCL_INIT_TIMEOUT_S="5", NCCL_NVLS_ENABLE="0",
               SPMVB_ROOT=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    out = subprocess.run([sys.executable, "-c", _NEVER_JOINS], env=env, capture_output=True, text=True,
                         timeout=120)
    assert "STATUS 7" in out.stdout, out.stdout + out.stderr


def test_spmv_time_is_the_reference_protocol(ctx):
    """spmvb_spmv_time: SpmvRunner::run's measurement in C++ (warm-up, one
    event pair per launch, median/mean/min/max); y is the kernel's result."""
    A = S.generate(2, seed=88, scale_rows=50000)
    xh = S.generate_vector(89, A.n)
    M = S.DeviceMatrix(ctx, A, S.F64)
    x = torch.from_numpy(xh).cuda()
    y = torch.full((A.m,), float("nan"), dtype=torch.float64, device="cuda")
    t = M.spmv_time(x, y, kernel=S.ELL, iters=9, warmup=2)
    assert 0 < t["min_ms"] <= t["median_ms"] <= t["max_ms"] and t["min_ms"] <= t["mean_ms"] <= t["max_ms"]
    torch.cuda.synchronize()
    assert_bitwise(oracle_y(A, xh, S.F64, S.F64), y.cpu().numpy(), "timed launches")
    with pytest.raises(S.SpmvbError):
        M.spmv_time(x, y, kernel=S.ELL, iters=0)
    M.close()
