"""Row-sharded iterated SpMV across 2 ranks on the CPU (gloo).

Each rank takes its nnz-balanced row block and the renumbered columns from
the library's own shard planner (spmvb_shard_csr), computes its y slice with
the oracle (standing in for the GPU kernel), and the padded slices are
all-gathered into x exactly as spmvb_dist_iterate does with ncclAllGather.
Row sharding keeps each row's summation order, so after several steps every
rank must hold the single-process result bit for bit.

The second test makes one rank leave before the exchange: the survivor must
get an error from the collective within the process-group timeout instead of
hanging."""
from __future__ import annotations

import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _iterate_worker(rank, world, port, which, rows, iters, outdir):
    import torch

    import oracle
    import spmvbench_b200 as S
    _init(rank, world, port, 60)
    try:
        A = S.generate(which, seed=21, scale_rows=rows)
        x = S.generate_vector(22, A.n)
        bounds = S.partition_rows(A.rowptr, world)
        mr, rp, ci = S.shard_csr(A, bounds, rank)
        vals = A.values[A.rowptr[bounds[rank]]:A.rowptr[bounds[rank + 1]]]
        ml = int(bounds[rank + 1] - bounds[rank])
        x_pad = np.zeros(world * mr)
        for r in range(world):
            x_pad[r * mr:r * mr + bounds[r + 1] - bounds[r]] = x[bounds[r]:bounds[r + 1]]
        for _ in range(iters):
            y = np.zeros(mr)
            y[:ml] = oracle.spmv_csr(ml, rp, ci, vals, x_pad)
            parts = [torch.zeros(mr, dtype=torch.float64) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(y))
            x_pad = torch.cat(parts).numpy()
        out = np.concatenate([x_pad[r * mr:r * mr + bounds[r + 1] - bounds[r]] for r in range(world)])
        np.save(os.path.join(outdir, f"rank{rank}.npy"), out)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("which,rows", [(2, 6000), (3, 8000), (1, 5000)])
def test_row_sharded_iteration_matches_single_process(which, rows):
    import oracle
    import spmvbench_b200 as S
    world, iters = 2, 3
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_iterate_worker, args=(world, _free_port(), which, rows, iters, d), nprocs=world,
                           start_method="spawn")
        A = S.generate(which, seed=21, scale_rows=rows)
        x = S.generate_vector(22, A.n)
        for _ in range(iters):
            x = oracle.spmv_csr(A.m, A.rowptr, A.colind, A.values, x)
        for r in range(world):
            np.testing.assert_array_equal(np.load(os.path.join(d, f"rank{r}.npy")), x)


def _leaver_worker(rank, world, port, outdir):
    import torch
    _init(rank, world, port, 10)
    if rank == 1:
        # Leaves between steps, with nothing in flight.
        os._exit(0)
    status = "no error"
    try:
        parts = [torch.zeros(4) for _ in range(world)]
        dist.all_gather(parts, torch.ones(4))
    except Exception as e:  # noqa: BLE001 - any collective error is the signal
        status = "error: " + type(e).__name__
    with open(os.path.join(outdir, "rank0.txt"), "w") as f:
        f.write(status)
    os._exit(0)


def test_departed_rank_is_detected_not_hung():
    world = 2
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.start_processes(_leaver_worker, args=(world, _free_port(), d), nprocs=world,
                                 start_method="spawn", join=False)
        for p in ctx.processes:
            p.join(60)
            assert not p.is_alive(), "a rank hung"
        assert open(os.path.join(d, "rank0.txt")).read().startswith("error")
