"""ctypes binding of libspmvb.so, the C ABI declared in include/spmvb.h.

The library is built in-tree (spmvbench_b200/lib/libspmvb.so, see
spmvbench_b200/csrc/Makefile). Importing this module never falls back to
anything else: if the library is missing the import fails with the build
command to run.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libspmvb.so")

OK = 0
STATUS = {
    0: "ok", 1: "invalid argument", 2: "invalid matrix", 3: "unsupported",
    4: "out of memory", 5: "CUDA error", 6: "NCCL error", 7: "timeout", 8: "no device", 9: "i/o error",
}

F32, F64 = 0, 1

# Kernel ids (values 0..5 follow the reference's KernelId).
CSR_SCALAR, CSR_VECTOR, CSR_WARP, CSR_MERGE, ELL, BCSR, HYB = range(7)
KERNEL_NAMES = ["csr_scalar", "csr_vector", "csr_warp", "csr_merge", "ell", "bcsr", "hyb"]
PREPARE_SPMM_BUCKETS = -1


class SpmvbError(RuntimeError):
    """A libspmvb call returned a non-zero status."""

    def __init__(self, status: int, func: str, message: str):
        self.status = status
        super().__init__(f"{func}: {STATUS.get(status, status)}: {message}")


class GpuInfo(C.Structure):
    _fields_ = [("name", C.c_char * 256), ("major", C.c_int), ("minor", C.c_int),
                ("sm_count", C.c_int), ("l2_bytes", C.c_int), ("max_smem_per_block", C.c_int),
                ("global_mem_bytes", C.c_int64), ("peak_gbs", C.c_double), ("peak_known", C.c_int)]


class MatrixInfo(C.Structure):
    _fields_ = [("m", C.c_int32), ("n", C.c_int32), ("nnz", C.c_int64), ("dtype", C.c_int),
                ("max_row_nnz", C.c_int32), ("ell_padded_nnz", C.c_int64),
                ("ell_touched_nnz", C.c_int64), ("bcsr2_block_nnz", C.c_int64),
                ("bcsr4_block_nnz", C.c_int64), ("hyb_width", C.c_int32),
                ("hyb_ell_nnz", C.c_int64), ("hyb_tail_nnz", C.c_int64),
                ("hyb_long_rows", C.c_int32), ("device_bytes", C.c_int64)]


class RowStats(C.Structure):
    _fields_ = [("nnz", C.c_int64), ("rows", C.c_int32), ("cols", C.c_int32),
                ("mean_row_nnz", C.c_double), ("median_row_nnz", C.c_double),
                ("min_row_nnz", C.c_int32), ("max_row_nnz", C.c_int32),
                ("stddev_row_nnz", C.c_double), ("cv_row_nnz", C.c_double),
                ("max_over_mean", C.c_double), ("ell_padding_overhead", C.c_double),
                ("frac_dense_blocks_4x4", C.c_double), ("density", C.c_double),
                ("dense_share_of_stored_4x4", C.c_double)]


class Choice(C.Structure):
    _fields_ = [("kernel", C.c_int32), ("lanes", C.c_int32), ("block_r", C.c_int32),
                ("block_c", C.c_int32), ("rule", C.c_int32), ("reason", C.c_char * 256)]


P = C.c_void_p
I32P = C.POINTER(C.c_int32)
I64P = C.POINTER(C.c_int64)

# name: (restype, argtypes)
SIGNATURES = {
    "spmvb_version": (C.c_char_p, []),
    "spmvb_last_error": (C.c_char_p, []),
    "spmvb_status_string": (C.c_char_p, [C.c_int]),
    "spmvb_launch_count": (C.c_uint64, []),
    "spmvb_gpu_available": (C.c_int, []),
    "spmvb_query_gpu": (C.c_int, [C.c_int, C.POINTER(GpuInfo)]),
    "spmvb_context_create": (C.c_int, [C.c_int, C.POINTER(P)]),
    "spmvb_context_destroy": (C.c_int, [P]),
    "spmvb_context_check": (C.c_int, [P]),
    "spmvb_selftest_wait_timeout": (C.c_int, [P]),
    "spmvb_matrix_create_csr": (C.c_int, [P, C.c_int, C.c_int32, C.c_int32, C.c_int64,
                                          P, P, P, C.POINTER(P)]),
    "spmvb_matrix_destroy": (C.c_int, [P]),
    "spmvb_csr_validate": (C.c_int, [C.c_int32, C.c_int32, C.c_int64, P, P, I32P]),
    "spmvb_shard_csr": (C.c_int, [C.c_int32, P, P, C.c_int, C.c_int, P, I32P, I64P, P, P]),
    "spmvb_matrix_prepare": (C.c_int, [P, C.c_int, C.c_int]),
    "spmvb_matrix_get_info": (C.c_int, [P, C.POINTER(MatrixInfo)]),
    "spmvb_matrix_export_ell": (C.c_int, [P, P, P, P]),
    "spmvb_matrix_export_bcsr": (C.c_int, [P, C.c_int, P, P, P]),
    "spmvb_spmv": (C.c_int, [P, C.c_int, C.c_int, C.c_int, P, P, C.c_int, P]),
    "spmvb_spmv_host": (C.c_int, [P, C.c_int, C.c_int, C.c_int, P, P, C.c_int, P]),
    "spmvb_spmv_time": (C.c_int, [P, C.c_int, C.c_int, C.c_int, P, P, C.c_int, C.c_int, C.c_int, P, P]),
    "spmvb_spmv_merge_noalloc": (C.c_int, [C.c_int, C.c_int32, C.c_int32, C.c_int64, P, P, P, P, P,
                                           C.c_int, P]),
    "spmvb_spmm": (C.c_int, [P, C.c_int, C.c_int, C.c_int, P, P, C.c_int, P]),
    "spmvb_matrix_set_spmm_bands": (C.c_int, [P, C.c_int]),
    "spmvb_spmm_host": (C.c_int, [P, C.c_int, C.c_int, C.c_int, P, P, C.c_int, P]),
    "spmvb_probe_gather_rate": (C.c_int, [P, C.c_int64, C.c_int64, C.POINTER(C.c_double)]),
    "spmvb_compute_row_stats": (C.c_int, [P, P, C.c_int32, C.c_int32, C.c_int64,
                                          C.POINTER(RowStats), P, C.c_int64]),
    "spmvb_matrix_row_stats": (C.c_int, [P, C.POINTER(RowStats), P, C.c_int64]),
    "spmvb_choose_spmv": (C.c_int, [C.POINTER(RowStats), C.POINTER(Choice)]),
    "spmvb_choose_spmv_reference": (C.c_int, [C.POINTER(RowStats), C.POINTER(Choice)]),
    "spmvb_kernel_name": (C.c_char_p, [C.c_int]),
    "spmvb_generate": (C.c_int, [C.c_int, C.c_uint64, C.c_int32, I32P, I32P, I64P, P, P, P]),
    "spmvb_generate_vector": (C.c_int, [C.c_uint64, C.c_int64, P]),
    "spmvb_partition_rows": (C.c_int, [P, C.c_int32, C.c_int32, P]),
    "spmvb_nccl_unique_id": (C.c_int, [P, C.c_size_t]),
    "spmvb_dist_create": (C.c_int, [P, C.c_int, C.c_int, P, C.c_int, C.c_int32, C.c_int64,
                                    P, P, P, P, C.POINTER(P)]),
    "spmvb_dist_destroy": (C.c_int, [P]),
    "spmvb_dist_set_x": (C.c_int, [P, P, P]),
    "spmvb_dist_iterate": (C.c_int, [P, C.c_int, C.c_int, C.c_int, P]),
    "spmvb_dist_iterate_timed": (C.c_int, [P, C.c_int, C.c_int, C.c_int, P,
                                           C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    "spmvb_dist_get_x": (C.c_int, [P, P, P]),
    "spmvb_dist_power_iterate": (C.c_int, [P, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_double), P]),
    "spmvb_dist_enable_peer": (C.c_int, [P, P]),
    "spmvb_dist_exchange": (C.c_int, [P]),
    "spmvb_dist_get_info": (C.c_int, [P, I32P, I32P, I32P, I64P]),
    "spmvb_dist_pipeline_create": (C.c_int, [P, C.c_int, C.POINTER(P)]),
    "spmvb_dist_pipeline_fork": (C.c_int, [P, P]),
    "spmvb_dist_pipeline_submit": (C.c_int, [P, C.c_int, C.c_int, P, P]),
    "spmvb_dist_pipeline_join": (C.c_int, [P, P]),
    "spmvb_dist_pipeline_wait": (C.c_int, [P]),
    "spmvb_dist_pipeline_destroy": (C.c_int, [P]),
    "spmvb_pipeline_create": (C.c_int, [P, C.c_int, C.POINTER(P)]),
    "spmvb_pipeline_fork": (C.c_int, [P, P]),
    "spmvb_pipeline_submit": (C.c_int, [P, C.c_int, C.c_int, C.c_int, P, P, C.c_int]),
    "spmvb_pipeline_join": (C.c_int, [P, P]),
    "spmvb_pipeline_wait": (C.c_int, [P]),
    "spmvb_pipeline_destroy": (C.c_int, [P]),
    "spmvb_read_matrix_market": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(P)]),
    "spmvb_csr_cache_write": (C.c_int, [C.c_char_p, C.c_int32, C.c_int32, C.c_int64, P, P, P]),
    "spmvb_csr_cache_read": (C.c_int, [C.c_char_p, C.POINTER(P)]),
    "spmvb_host_csr_get": (C.c_int, [P, I32P, I32P, I64P, C.POINTER(P), C.POINTER(P), C.POINTER(P)]),
    "spmvb_host_csr_free": (None, [P]),
}

_lib = None


def load() -> C.CDLL:
    """Load libspmvb.so once; raise ImportError with the build command if absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `make -C {os.path.join(_HERE, 'csrc')}` "
            "(or __graft_entry__.build()); there is no CPU fallback")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, func: str) -> None:
    if status != OK:
        msg = load().spmvb_last_error()
        raise SpmvbError(status, func, msg.decode() if msg else "")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)
