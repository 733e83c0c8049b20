"""One rank of the multi-GPU parity test (launched by tests/test_gpu_dist.py
under torch.distributed.run): iterated y = A x, x <- y, row-sharded over the
ranks, x slices exchanged by ncclAllGather and by the peer-memory exchange,
checked bit for bit against the single-process oracle iteration (row
sharding keeps every row's order; merge-path rows within 1e-9)."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import oracle  # noqa: E402
import spmvbench_b200 as S  # noqa: E402

rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
torch.cuda.set_device(local)
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
ctx = S.Context(local)

if len(sys.argv) > 1 and sys.argv[1] == "peer-timeout":
    # Rank 1 skips a step (it leaves between steps, nothing in flight): rank
    # 0's end-of-step barrier waits for a phase nobody publishes, gives up
    # after SPMVB_PEER_TIMEOUT_MS, and the host gets SPMVB_ERR_TIMEOUT.
    A = S.generate(2, seed=93, scale_rows=20000)
    bounds = S.partition_rows(A.rowptr, world)
    obj = [S.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    D = S.DistMatrix(ctx, world, rank, obj[0], A, bounds, S.F64)
    D.enable_peer()
    D.set_x(S.generate_vector(94, A.n))
    status = 0
    if rank == 0:
        D.iterate(1, kernel=S.ELL)
        try:
            D.get_x()
        except S.SpmvbError as e:
            status = e.status
        ctx.check()   # the error word was read and cleared; the context is usable
        print(f"rank 0 status {status}", flush=True)
    dist.barrier()
    D.close()
    # Rank 1's close still stores its last phase into rank 0's memory (rank
    # 0, whose handle gave up, leaves its buffers allocated): rank 0 stays
    # alive until rank 1's close has returned.
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if rank != 0 or status == 7 else 1)

bad = 0
for which, rows, kernel in ((2, 200000, S.ELL), (3, 300000, S.CSR_MERGE), (1, 0, S.CSR_SCALAR)):
    A = S.generate(which, seed=91, scale_rows=rows)
    x0 = S.generate_vector(92, A.n) / 4.0
    bounds = S.partition_rows(A.rowptr, world)
    x = x0
    for _ in range(3):
        x = oracle.spmv_csr(A.m, A.rowptr, A.colind, A.values, x, np.float64)
    for exchange in ("nccl", "peer"):
        obj = [S.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        D = S.DistMatrix(ctx, world, rank, obj[0], A, bounds, S.F64)
        if exchange == "peer":
            D.enable_peer()
            assert D.exchange == "peer"
            D.set_x(x0 * 3.0)   # overwritten below: set_x restarts cleanly after any step count
            D.iterate(4, kernel=kernel)   # one eager step, one replay of the 2-step graph, one eager
            D.set_x(x0)
            D.iterate(3, kernel=kernel)   # one eager step, one graph replay
        else:
            D.set_x(x0)
            D.iterate(2, kernel=kernel)
            D.iterate(1, kernel=kernel)
        got = D.get_x()
        D.close()
        if kernel == S.CSR_MERGE:
            ok = np.allclose(got, x, rtol=1e-9, atol=1e-12)
        else:
            ok = np.array_equal(got, x)
        print(f"rank {rank} workload {which} kernel {S.kernel_name(kernel)} exchange {exchange}: "
              f"{'ok' if ok else 'MISMATCH'}", flush=True)
        bad += not ok
# Power iteration over the row blocks: the norm is taken over the whole
# vector in a rank-independent order, so every rank's x and eigenvalue
# estimate equal a one-rank run bit for bit (ELL keeps csr_omp's order).
A = S.generate(2, seed=97, scale_rows=120000)
x0 = S.generate_vector(98, A.n)
D1 = S.DistMatrix(ctx, 1, 0, None, A, S.partition_rows(A.rowptr, 1), S.F64)
D1.set_x(x0)
lam1 = D1.power_iterate(8, kernel=S.ELL)
x1 = D1.get_x()
D1.close()
bounds = S.partition_rows(A.rowptr, world)
for exchange in ("nccl", "peer"):
    obj = [S.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    D = S.DistMatrix(ctx, world, rank, obj[0], A, bounds, S.F64)
    if exchange == "peer":
        D.enable_peer()
    D.set_x(x0)
    lam = D.power_iterate(8, kernel=S.ELL)
    ok = lam == lam1 and np.array_equal(D.get_x(), x1)
    D.close()
    print(f"rank {rank} power iteration exchange {exchange}: {'ok' if ok else 'MISMATCH'}", flush=True)
    bad += not ok

# Host-buffer product over the row blocks (spmvb_dist_pipeline): each rank
# submits its rows' slice of x and must get its rows of csr_omp's y.
for which, rows, kernel in ((2, 200000, S.ELL), (3, 300000, S.CSR_MERGE)):
    A = S.generate(which, seed=95, scale_rows=rows)
    bounds = S.partition_rows(A.rowptr, world)
    r0, r1 = int(bounds[rank]), int(bounds[rank + 1])
    obj = [S.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    D = S.DistMatrix(ctx, world, rank, obj[0], A, bounds, S.F64)
    P = S.DistPipeline(D, depth=3)
    xs = [S.generate_vector(96 + i, A.n) for i in range(5)]
    ys = [torch.empty(max(r1 - r0, 1), dtype=torch.float64).pin_memory() for _ in range(5)]
    xl = [torch.from_numpy(x[r0:r1].copy()).pin_memory() for x in xs]
    for i in range(5):
        P.submit(xl[i].numpy(), ys[i].numpy(), kernel=kernel)
    P.wait()
    ok = True
    for i in range(5):
        ref = oracle.spmv_csr(A.m, A.rowptr, A.colind, A.values, xs[i], np.float64)[r0:r1]
        got = ys[i].numpy()[:r1 - r0]
        ok &= np.allclose(got, ref, rtol=1e-9, atol=1e-12) if kernel == S.CSR_MERGE else np.array_equal(got, ref)
    P.close()
    D.close()
    print(f"rank {rank} workload {which} kernel {S.kernel_name(kernel)} exchange pipeline: "
          f"{'ok' if ok else 'MISMATCH'}", flush=True)
    bad += not ok
dist.barrier()
dist.destroy_process_group()
sys.exit(1 if bad else 0)
