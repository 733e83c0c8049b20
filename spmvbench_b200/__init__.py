"""spmvbench_b200 - B200 (sm_100a) SpMV / SpMM kernels behind the C ABI of
include/spmvb.h, with a thin Python mirror used by the tests and bench.py.

The Python layer only moves arguments: every computation runs in
lib/libspmvb.so (hand-written CUDA kernels plus the C++ host runtime).
Device buffers are torch tensors (torch is used for device memory and
streams only). Host-side matrices are numpy CSR triples, mirroring the
reference's CsrMatrix<T> (include/spmvbench/csr.hpp:16-35).
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import (BCSR, CSR_MERGE, CSR_SCALAR, CSR_VECTOR, CSR_WARP, ELL, F32, F64, HYB,
                   KERNEL_NAMES, SpmvbError, call, load)

__all__ = [
    "CsrMatrix", "Context", "DeviceMatrix", "DistMatrix", "DistPipeline", "SpmvbError", "generate",
    "read_matrix_market", "write_csr_cache", "read_csr_cache", "Pipeline",
    "generate_vector", "row_stats", "choose_spmv", "choose_spmv_reference", "partition_rows",
    "launch_count", "gpu_available", "csr_validate", "shard_csr", "query_gpu", "kernel_name", "nccl_unique_id",
    "CSR_SCALAR", "CSR_VECTOR", "CSR_WARP", "CSR_MERGE", "ELL", "BCSR", "HYB", "F32", "F64",
    "KERNEL_NAMES", "WORKLOADS",
]

# Benchmark workloads produced by generate(): id -> name.
WORKLOADS = {1: "banded_100k_hb4", 2: "uniform_1m_16", 3: "powerlaw_1m_zipf2.1",
             4: "bcsr4x4_500k_8blk", 5: "spmm_uniform_1m_16_k64"}


def _np_dtype(d: int):
    return np.float64 if d == F64 else np.float32


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p) if a is not None and a.size else None


def _host_in(a, dtype, count: int, what: str) -> np.ndarray:
    """A host input the C ABI reads `count` entries of, as a contiguous array
    of `dtype`; shorter arrays are refused (the C side cannot see lengths)."""
    arr = np.ascontiguousarray(a, dtype)
    if arr.size < count:
        raise ValueError(f"{what} holds {arr.size} entries; {count} are needed")
    return arr


def _host_out(a, dtype, count: int, what: str) -> np.ndarray:
    """A caller-supplied host output the C ABI writes `count` entries of: it
    must already have the element type, be contiguous and be long enough,
    since a converted copy would not be the caller's array."""
    if not isinstance(a, np.ndarray) or a.dtype != dtype or not a.flags.c_contiguous or not a.flags.writeable:
        raise ValueError(f"{what} must be a writeable C-contiguous {np.dtype(dtype).name} array")
    if a.size < count:
        raise ValueError(f"{what} holds {a.size} entries; {count} are needed")
    return a


def _int32(a, what: str) -> np.ndarray:
    """`a` as a contiguous int32 array; integer values outside int32 are an
    error instead of wrapping."""
    arr = np.asarray(a)
    if arr.dtype != np.int32 and arr.dtype.kind in "iu" and arr.size and \
            (int(arr.min()) < -2**31 or int(arr.max()) > 2**31 - 1):
        raise ValueError(f"{what} has values outside the int32 index range")
    return np.ascontiguousarray(arr, np.int32)


def _csr_buffers(A: "CsrMatrix", value_dtype=None):
    """Contiguous int32 rowptr and colind of A (and its values as
    `value_dtype`), with their lengths checked against m and rowptr[m]: the C
    ABI takes plain pointers and reads m + 1 and nnz entries through them, so a
    short array here would be read past its end."""
    rp = _int32(A.rowptr, "rowptr")
    if rp.ndim != 1 or rp.size < A.m + 1:
        raise ValueError(f"rowptr holds {rp.size} entries; m + 1 = {A.m + 1} are needed")
    nnz = int(rp[A.m]) if A.m else 0
    ci = _int32(A.colind, "colind")
    if ci.size < nnz:
        raise ValueError(f"colind holds {ci.size} entries; rowptr[m] = {nnz} are needed")
    if value_dtype is None:
        return rp, ci
    va = np.ascontiguousarray(A.values, value_dtype)
    if va.size < nnz:
        raise ValueError(f"values holds {va.size} entries; rowptr[m] = {nnz} are needed")
    return rp, ci, va


@dataclass
class CsrMatrix:
    """Host CSR with int32 indices (reference CsrMatrix<T>)."""
    m: int
    n: int
    rowptr: np.ndarray
    colind: np.ndarray
    values: np.ndarray

    @property
    def nnz(self) -> int:
        return int(self.rowptr[self.m]) if self.m else 0

    def astype(self, dtype) -> "CsrMatrix":
        return CsrMatrix(self.m, self.n, self.rowptr, self.colind,
                         np.ascontiguousarray(self.values, dtype=dtype))

    def row_lengths(self) -> np.ndarray:
        return np.diff(self.rowptr)


def generate(which: int, seed: int = 2024, scale_rows: int = 0) -> CsrMatrix:
    """Seeded benchmark matrix `which` (1..5, see WORKLOADS), fp64 values."""
    lib = load()
    m, n, nnz = C.c_int32(), C.c_int32(), C.c_int64()
    _lib.check(lib.spmvb_generate(which, seed, scale_rows, C.byref(m), C.byref(n), C.byref(nnz),
                                  None, None, None), "spmvb_generate")
    rowptr = np.zeros(m.value + 1, np.int32)
    colind = np.zeros(max(nnz.value, 1), np.int32)
    values = np.zeros(max(nnz.value, 1), np.float64)
    _lib.check(lib.spmvb_generate(which, seed, scale_rows, C.byref(m), C.byref(n), C.byref(nnz),
                                  _ptr(rowptr), colind.ctypes.data_as(C.c_void_p),
                                  values.ctypes.data_as(C.c_void_p)), "spmvb_generate")
    return CsrMatrix(m.value, n.value, rowptr, colind[:nnz.value], values[:nnz.value])


def _take_host_csr(h) -> CsrMatrix:
    """Copies a spmvb_host_csr handle into a CsrMatrix and frees it."""
    lib = load()
    try:
        m, n, nnz = C.c_int32(), C.c_int32(), C.c_int64()
        rp, ci, va = C.c_void_p(), C.c_void_p(), C.c_void_p()
        call("spmvb_host_csr_get", h, C.byref(m), C.byref(n), C.byref(nnz), C.byref(rp), C.byref(ci), C.byref(va))

        def arr(ptr, count, ctype, dtype):
            if count == 0:
                return np.zeros(0, dtype)
            return np.ctypeslib.as_array(C.cast(ptr, C.POINTER(ctype)), shape=(count,)).copy()

        return CsrMatrix(m.value, n.value, arr(rp, m.value + 1, C.c_int32, np.int32),
                         arr(ci, nnz.value, C.c_int32, np.int32), arr(va, nnz.value, C.c_double, np.float64))
    finally:
        lib.spmvb_host_csr_free(h)


def read_matrix_market(path: str, threads: int = 0) -> CsrMatrix:
    """The reference's read_matrix_market (same CSR, same errors), parsed by
    `threads` threads (0 = all). fp64 values; .astype(np.float32) gives the
    reference's read_matrix_market<float>."""
    h = C.c_void_p()
    call("spmvb_read_matrix_market", os.fsencode(path), threads, C.byref(h))
    return _take_host_csr(h)


def write_csr_cache(path: str, A: CsrMatrix) -> None:
    """Binary CSR cache of A (validated), read back by read_csr_cache."""
    rp, ci, va = _csr_buffers(A, np.float64)
    call("spmvb_csr_cache_write", os.fsencode(path), A.m, A.n, A.nnz, _ptr(rp), _ptr(ci), _ptr(va))


def read_csr_cache(path: str) -> CsrMatrix:
    h = C.c_void_p()
    call("spmvb_csr_cache_read", os.fsencode(path), C.byref(h))
    return _take_host_csr(h)


def generate_vector(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float64)
    call("spmvb_generate_vector", seed, n, _ptr(out))
    return out


def launch_count() -> int:
    return int(load().spmvb_launch_count())


def gpu_available() -> bool:
    return bool(load().spmvb_gpu_available())


def query_gpu(device: int = 0) -> dict:
    g = _lib.GpuInfo()
    call("spmvb_query_gpu", device, C.byref(g))
    return {"name": g.name.decode(), "major": g.major, "minor": g.minor, "sm_count": g.sm_count,
            "l2_bytes": g.l2_bytes, "global_mem_bytes": g.global_mem_bytes,
            "peak_gbs": g.peak_gbs, "peak_known": bool(g.peak_known)}


def kernel_name(k: int) -> str:
    return load().spmvb_kernel_name(k).decode()


def row_stats(A: CsrMatrix, histogram: bool = False) -> dict:
    s = _lib.RowStats()
    rp, ci = _csr_buffers(A)
    hist = None
    if histogram:
        mx = int(np.max(np.diff(rp))) if A.m else 0
        hist = np.zeros(mx + 1, np.int64)
    call("spmvb_compute_row_stats", _ptr(rp), _ptr(ci), A.m, A.n, A.nnz, C.byref(s),
         _ptr(hist), 0 if hist is None else hist.size)
    d = {f: getattr(s, f) for f, _ in _lib.RowStats._fields_}
    if histogram:
        d["row_nnz_histogram"] = hist
    return d


def _stats_struct(d: dict) -> _lib.RowStats:
    s = _lib.RowStats()
    for f, _ in _lib.RowStats._fields_:
        setattr(s, f, d.get(f, 0))
    return s


def _choice(fn: str, stats: dict) -> dict:
    c = _lib.Choice()
    call(fn, C.byref(_stats_struct(stats)), C.byref(c))
    return {"kernel": c.kernel, "lanes": c.lanes, "block_r": c.block_r, "block_c": c.block_c,
            "rule": c.rule, "reason": c.reason.decode(), "name": kernel_name(c.kernel)}


def choose_spmv(stats: dict) -> dict:
    """B200 kernel choice from row statistics."""
    return _choice("spmvb_choose_spmv", stats)


def choose_spmv_reference(stats: dict) -> dict:
    """The reference's rule set (src/select.cpp:93-165), unchanged."""
    return _choice("spmvb_choose_spmv_reference", stats)


def partition_rows(rowptr: np.ndarray, parts: int) -> np.ndarray:
    rp = np.ascontiguousarray(rowptr, np.int32)
    out = np.zeros(parts + 1, np.int32)
    call("spmvb_partition_rows", _ptr(rp), rp.size - 1, parts, _ptr(out))
    return out


def csr_validate(A: CsrMatrix) -> int:
    """Host validation of a CSR (raises SpmvbError); returns the longest row."""
    rp, ci = _csr_buffers(A)
    mx = C.c_int32()
    call("spmvb_csr_validate", A.m, A.n, A.nnz, _ptr(rp), _ptr(ci), C.byref(mx))
    return mx.value


def shard_csr(A: CsrMatrix, bounds: np.ndarray, rank: int):
    """Rank `rank`'s rows of a square CSR with columns renumbered into the
    padded gather layout. Returns (max_rows, local rowptr, local colind)."""
    rp, ci = _csr_buffers(A)
    b = np.ascontiguousarray(bounds, np.int32)
    nranks = b.size - 1
    mr, ln = C.c_int32(), C.c_int64()
    call("spmvb_shard_csr", A.m, _ptr(rp), _ptr(ci), nranks, rank, _ptr(b), C.byref(mr), C.byref(ln), None, None)
    orp = np.zeros(int(b[rank + 1] - b[rank]) + 1, np.int32)
    oci = np.zeros(max(ln.value, 1), np.int32)
    call("spmvb_shard_csr", A.m, _ptr(rp), _ptr(ci), nranks, rank, _ptr(b), C.byref(mr), C.byref(ln),
         _ptr(orp), oci.ctypes.data_as(C.c_void_p))
    return mr.value, orp, oci[:ln.value]


def nccl_unique_id() -> bytes:
    buf = (C.c_char * 128)()
    call("spmvb_nccl_unique_id", buf, 128)
    return bytes(buf)


def _stream_ptr(stream):
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return C.c_void_p(stream.cuda_stream)


class Context:
    """One device (spmvb_context)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        call("spmvb_context_create", device, C.byref(h))
        self.handle = h
        self.device = device

    def gather_rate(self, n: int = 1_000_000, gathers: int = 16_000_000) -> float:
        """Measured random 8-byte gathers per second from an L2-resident
        vector of n doubles (the ceiling of locality-free SpMV)."""
        r = C.c_double()
        call("spmvb_probe_gather_rate", self.handle, n, gathers, C.byref(r))
        return r.value

    def check(self) -> None:
        """Synchronize and raise if a kernel gave up a bounded wait."""
        call("spmvb_context_check", self.handle)

    def close(self):
        if self.handle:
            load().spmvb_context_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DeviceMatrix:
    """A matrix uploaded to one device (spmvb_matrix). `dtype` is the storage
    type; kernels accept acc = dtype, or F64 accumulation of F32 storage."""

    def __init__(self, ctx: Context, A: CsrMatrix, dtype: int = F64):
        self.ctx = ctx
        self.m, self.n, self.nnz = A.m, A.n, A.nnz
        self.dtype = dtype
        rp, ci, va = _csr_buffers(A, _np_dtype(dtype))
        h = C.c_void_p()
        call("spmvb_matrix_create_csr", ctx.handle, dtype, A.m, A.n, A.nnz, _ptr(rp), _ptr(ci),
             _ptr(va), C.byref(h))
        self.handle = h

    def close(self):
        if getattr(self, "handle", None):
            load().spmvb_matrix_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def prepare(self, kernel: int, param: int = 0) -> None:
        call("spmvb_matrix_prepare", self.handle, kernel, param)

    def row_stats(self, histogram: bool = False) -> dict:
        """row_stats() of the uploaded matrix, with the block census on the
        device (spmvb_matrix_row_stats); bit-identical to row_stats(A)."""
        s = _lib.RowStats()
        hist = np.zeros(self.info()["max_row_nnz"] + 1, np.int64) if histogram else None
        call("spmvb_matrix_row_stats", self.handle, C.byref(s), _ptr(hist), 0 if hist is None else hist.size)
        d = {f: getattr(s, f) for f, _ in _lib.RowStats._fields_}
        if histogram:
            d["row_nnz_histogram"] = hist
        return d

    def info(self) -> dict:
        i = _lib.MatrixInfo()
        call("spmvb_matrix_get_info", self.handle, C.byref(i))
        return {f: getattr(i, f) for f, _ in _lib.MatrixInfo._fields_}

    # -- device-buffer entry points (torch tensors) --
    def spmv(self, x, y, kernel: int = CSR_SCALAR, lanes: int = 4, block: int = 4,
             acc: int | None = None, stream=None) -> None:
        acc = self.dtype if acc is None else acc
        call("spmvb_spmv", self.handle, kernel, lanes, block, C.c_void_p(x.data_ptr()),
             C.c_void_p(y.data_ptr()), acc, _stream_ptr(stream))

    def set_spmm_bands(self, bands: int) -> None:
        """Column bands of the plain tile-64 SpMM sweep (0 = automatic,
        1 = one row-order pass); bit-identical results either way."""
        call("spmvb_matrix_set_spmm_bands", self.handle, bands)

    def spmv_time(self, x, y, kernel: int = CSR_SCALAR, lanes: int = 4, block: int = 4, iters: int = 20,
                  warmup: int = 5, acc: int | None = None, stream=None) -> dict:
        """SpmvRunner::run's measurement in C++ (spmvb_spmv_time): median /
        mean / min / max ms of `iters` launches, one event pair each."""
        acc = self.dtype if acc is None else acc
        out = np.zeros(4)
        call("spmvb_spmv_time", self.handle, kernel, lanes, block, C.c_void_p(x.data_ptr()),
             C.c_void_p(y.data_ptr()), acc, iters, warmup, _stream_ptr(stream), _ptr(out))
        return dict(zip(("median_ms", "mean_ms", "min_ms", "max_ms"), out.tolist()))

    def spmm(self, X, Y, k: int, tile: int = 32, bucketed: bool = False,
             acc: int | None = None, stream=None) -> None:
        acc = self.dtype if acc is None else acc
        call("spmvb_spmm", self.handle, tile, int(bucketed), k, C.c_void_p(X.data_ptr()),
             C.c_void_p(Y.data_ptr()), acc, _stream_ptr(stream))

    # -- host-buffer entry points (numpy arrays; copies inside, synchronous) --
    def spmv_host(self, x: np.ndarray, kernel: int = CSR_SCALAR, lanes: int = 4, block: int = 4,
                  acc: int | None = None, out: np.ndarray | None = None, stream=None) -> np.ndarray:
        acc = self.dtype if acc is None else acc
        x = _host_in(x, _np_dtype(self.dtype), self.n, "x")
        y = _host_out(out, _np_dtype(acc), self.m, "out") if out is not None else np.empty(self.m, _np_dtype(acc))
        s = C.c_void_p(0) if stream is None else _stream_ptr(stream)
        call("spmvb_spmv_host", self.handle, kernel, lanes, block, _ptr(x), _ptr(y), acc, s)
        return y

    def spmm_host(self, X: np.ndarray, k: int, tile: int = 32, bucketed: bool = False,
                  acc: int | None = None, stream=None) -> np.ndarray:
        acc = self.dtype if acc is None else acc
        X = _host_in(X, _np_dtype(self.dtype), self.n * k, "X")
        Y = np.empty((self.m, k), _np_dtype(acc))
        s = C.c_void_p(0) if stream is None else _stream_ptr(stream)
        call("spmvb_spmm_host", self.handle, tile, int(bucketed), k, _ptr(X), _ptr(Y), acc, s)
        return Y

    def export_ell(self):
        width = self.info()["max_row_nnz"]
        col = np.zeros(self.m * width, np.int32)
        val = np.zeros(self.m * width, _np_dtype(self.dtype))
        rl = np.zeros(self.m, np.int32)
        call("spmvb_matrix_export_ell", self.handle, _ptr(col), _ptr(val), _ptr(rl))
        return width, col, val, rl

    def export_bcsr(self, block: int):
        self.prepare(BCSR, block)
        bnnz = self.info()["bcsr2_block_nnz" if block == 2 else "bcsr4_block_nnz"]
        mb = (self.m + block - 1) // block
        rp = np.zeros(mb + 1, np.int32)
        ci = np.zeros(max(bnnz, 1), np.int32)
        va = np.zeros(max(bnnz, 1) * block * block, _np_dtype(self.dtype))
        call("spmvb_matrix_export_bcsr", self.handle, block, _ptr(rp), _ptr(ci), _ptr(va))
        return rp, ci[:bnnz], va[:bnnz * block * block]


class Pipeline:
    """Streamed y = A x over host buffers: up to `depth` calls in flight on
    their own streams (pinned host buffers let copies in, kernels and copies
    out of different calls overlap). Keep x unchanged and y unread until
    wait() (or join())."""

    def __init__(self, M: "DeviceMatrix", depth: int = 3):
        h = C.c_void_p()
        call("spmvb_pipeline_create", M.handle, depth, C.byref(h))
        self.handle = h
        self.M = M
        self._keep = []

    def fork(self, stream):
        call("spmvb_pipeline_fork", self.handle, _stream_ptr(stream))

    def submit(self, x: np.ndarray, y: np.ndarray, kernel: int = CSR_SCALAR, lanes: int = 4, block: int = 4,
               acc: int | None = None):
        acc = self.M.dtype if acc is None else acc
        # Both arrays are used in place (x read, y written after return), so
        # they must already have the right type, layout and length.
        if not isinstance(x, np.ndarray) or x.dtype != _np_dtype(self.M.dtype) or not x.flags.c_contiguous \
                or x.size < self.M.n:
            raise ValueError(f"x must be a C-contiguous {np.dtype(_np_dtype(self.M.dtype)).name} array of "
                             f"at least {self.M.n} entries")
        _host_out(y, _np_dtype(acc), self.M.m, "y")
        self._keep.append((x, y))  # alive until wait()
        call("spmvb_pipeline_submit", self.handle, kernel, lanes, block, _ptr(x), _ptr(y), acc)

    def join(self, stream):
        call("spmvb_pipeline_join", self.handle, _stream_ptr(stream))

    def wait(self):
        call("spmvb_pipeline_wait", self.handle)
        self._keep.clear()

    def close(self):
        if getattr(self, "handle", None):
            load().spmvb_pipeline_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()


class DistMatrix:
    """One rank's shard of a row-partitioned square matrix for iterated
    y = A x, x <- y, with the x slices exchanged by ncclAllGather or, after
    enable_peer(), stored by the SpMV into every rank's x over peer memory."""

    def __init__(self, ctx: Context, nranks: int, rank: int, uid: bytes | None, A: CsrMatrix,
                 bounds: np.ndarray, dtype: int = F64):
        rp, ci, va = _csr_buffers(A, _np_dtype(dtype))
        b = np.ascontiguousarray(bounds, np.int32)
        ub = C.create_string_buffer(uid, 128) if uid is not None else None
        h = C.c_void_p()
        call("spmvb_dist_create", ctx.handle, nranks, rank, ub, dtype, A.m, A.nnz, _ptr(rp),
             _ptr(ci), _ptr(va), _ptr(b), C.byref(h))
        self.handle = h
        self.m = A.m
        self.dtype = dtype

    def close(self):
        if getattr(self, "handle", None):
            load().spmvb_dist_destroy(self.handle)
            self.handle = None

    def set_x(self, x: np.ndarray, stream=None):
        x = _host_in(x, _np_dtype(self.dtype), self.m, "x")
        call("spmvb_dist_set_x", self.handle, _ptr(x), _stream_ptr(stream))

    def iterate(self, iters: int, kernel: int = CSR_SCALAR, lanes: int = 4, stream=None):
        call("spmvb_dist_iterate", self.handle, kernel, lanes, iters, _stream_ptr(stream))

    def iterate_timed(self, iters: int, kernel: int = CSR_SCALAR, lanes: int = 4, stream=None):
        k = C.c_double()
        s = C.c_double()
        call("spmvb_dist_iterate_timed", self.handle, kernel, lanes, iters, _stream_ptr(stream),
             C.byref(k), C.byref(s))
        return k.value, s.value

    def power_iterate(self, iters: int, kernel: int = CSR_SCALAR, lanes: int = 4, stream=None) -> float:
        """`iters` steps of x <- A x / ||A x||_2 (collective); returns the last
        norm, the dominant eigenvalue's magnitude once converged."""
        lam = C.c_double()
        call("spmvb_dist_power_iterate", self.handle, kernel, lanes, iters, C.byref(lam), _stream_ptr(stream))
        return lam.value

    def enable_peer(self, stream=None):
        """Collective: switch the x exchange from ncclAllGather to direct
        stores into every rank's x over peer memory (raises SpmvbError with
        status UNSUPPORTED on every rank when some rank cannot map it)."""
        call("spmvb_dist_enable_peer", self.handle, _stream_ptr(stream))

    @property
    def exchange(self) -> str:
        return "peer" if load().spmvb_dist_exchange(self.handle) == 1 else "nccl"

    def get_x(self, stream=None) -> np.ndarray:
        out = np.empty(self.m, _np_dtype(self.dtype))
        call("spmvb_dist_get_x", self.handle, _ptr(out), _stream_ptr(stream))
        return out

    def row_range(self) -> tuple[int, int]:
        i = self.info()
        return i["row_begin"], i["row_end"]

    def info(self) -> dict:
        a, b, c = C.c_int32(), C.c_int32(), C.c_int32()
        d = C.c_int64()
        call("spmvb_dist_get_info", self.handle, C.byref(a), C.byref(b), C.byref(c), C.byref(d))
        return {"row_begin": a.value, "row_end": b.value, "max_rows": c.value, "local_nnz": d.value}


class DistPipeline:
    """Row-sharded y = A x over host buffers (spmvb_dist_pipeline): each rank
    submits its own rows' slice of x and receives its rows of y; the slices
    are all-gathered on the devices over NVLink. Collective: every rank makes
    the same sequence of submits. Keep x unchanged and y unread until wait()
    (or join())."""

    def __init__(self, D: DistMatrix, depth: int = 3):
        h = C.c_void_p()
        call("spmvb_dist_pipeline_create", D.handle, depth, C.byref(h))
        self.handle = h
        self.D = D
        self.rows = D.row_range()[1] - D.row_range()[0]
        self._keep = []

    def fork(self, stream):
        call("spmvb_dist_pipeline_fork", self.handle, _stream_ptr(stream))

    def submit(self, x_local: np.ndarray, y_local: np.ndarray, kernel: int = CSR_SCALAR, lanes: int = 4):
        dt = _np_dtype(self.D.dtype)
        if not isinstance(x_local, np.ndarray) or x_local.dtype != dt or not x_local.flags.c_contiguous \
                or x_local.size < self.rows:
            raise ValueError(f"x_local must be a C-contiguous {np.dtype(dt).name} array of at least "
                             f"{self.rows} entries")
        _host_out(y_local, dt, self.rows, "y_local")
        self._keep.append((x_local, y_local))
        call("spmvb_dist_pipeline_submit", self.handle, kernel, lanes, _ptr(x_local), _ptr(y_local))

    def join(self, stream):
        call("spmvb_dist_pipeline_join", self.handle, _stream_ptr(stream))

    def wait(self):
        call("spmvb_dist_pipeline_wait", self.handle)
        self._keep.clear()

    def close(self):
        if getattr(self, "handle", None):
            load().spmvb_dist_pipeline_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
