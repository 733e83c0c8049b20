"""One rank of the multi-GPU parity test (launched by tests/test_gpu_dist.py
under torch.distributed.run): iterated y = A x, x <- y, row-sharded over the
ranks with ncclAllGather of the padded slices, checked bit for bit against
the single-process oracle iteration (row sharding keeps every row's order)."""
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
bad = 0
for which, rows, kernel in ((2, 200000, S.ELL), (3, 300000, S.CSR_MERGE), (1, 0, S.CSR_SCALAR)):
    A = S.generate(which, seed=91, scale_rows=rows)
    x0 = S.generate_vector(92, A.n) / 4.0
    bounds = S.partition_rows(A.rowptr, world)
    obj = [S.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    D = S.DistMatrix(ctx, world, rank, obj[0], A, bounds, S.F64)
    D.set_x(x0)
    D.iterate(3, kernel=kernel)
    got = D.get_x()
    D.close()
    x = x0
    for _ in range(3):
        x = oracle.spmv_csr(A.m, A.rowptr, A.colind, A.values, x, np.float64)
    if kernel == S.CSR_MERGE:
        r, _ = oracle.gamma_ratio(A.rowptr, A.colind, A.values, x0, x, x, np.float64)
        ok = np.allclose(got, x, rtol=1e-9, atol=0)
    else:
        ok = np.array_equal(got, x)
    print(f"rank {rank} workload {which} kernel {S.kernel_name(kernel)}: {'ok' if ok else 'MISMATCH'}", flush=True)
    bad += not ok
dist.barrier()
dist.destroy_process_group()
sys.exit(1 if bad else 0)
