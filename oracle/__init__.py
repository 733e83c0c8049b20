"""Oracle - test infrastructure, never part of the product path.

ctypes-loaded libraries built by oracle/Makefile:
  liboracle.so             C restatement of SpMVBench's CPU path (oracle.c)
  _ref/libspmvref.so       SpMVBench's own CPU sources compiled in place, plus
                           the extern "C" shim ref_shim.cpp (present when the
                           reference tree was available at build time)
  _ref/libspmvref_cuda.so  SpMVBench's own GPU path (src/cuda) compiled in
                           place for sm_100a, plus ref_cuda_shim.cu (`make
                           ref_cuda`), to run the reference's kernels beside
                           this library's on the same device

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arms import this package, and only to check or time: the CUDA library in
spmvbench_b200/ never calls it.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
PORT_PATH = os.path.join(_HERE, "liboracle.so")
REF_PATH = os.path.join(_HERE, "_ref", "libspmvref.so")

_port = None
_ref = None

P = C.c_void_p


def _p(a):
    return a.ctypes.data_as(P) if a is not None and a.size else None


def port() -> C.CDLL:
    global _port
    if _port is None:
        if not os.path.exists(PORT_PATH):
            raise ImportError(f"{PORT_PATH} missing: run `make -C {_HERE}`")
        _port = C.CDLL(PORT_PATH)
        for suf in ("dd", "ff", "fd"):
            getattr(_port, f"orc_spmv_csr_{suf}").argtypes = [C.c_int32, P, P, P, P, P, C.c_int]
            getattr(_port, f"orc_spmv_ell_{suf}").argtypes = [C.c_int32, P, P, P, P, P, C.c_int]
            getattr(_port, f"orc_spmv_bcsr_{suf}").argtypes = [C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                                               C.c_int32, P, P, P, P, P, C.c_int]
            getattr(_port, f"orc_spmm_csr_{suf}").argtypes = [C.c_int32, C.c_int32, P, P, P, P, P, C.c_int]
        _port.orc_ell_width.argtypes = [C.c_int32, P]
        _port.orc_ell_width.restype = C.c_int32
        _port.orc_csr_to_ell.argtypes = [C.c_int32, P, P, P, C.c_int, P, P, P]
        _port.orc_csr_to_bcsr.argtypes = [C.c_int32, C.c_int32, C.c_int32, C.c_int32, P, P, P, C.c_int,
                                          C.POINTER(C.c_int32), C.POINTER(C.c_int64), P, P, P]
        _port.orc_row_stats.argtypes = [P, P, C.c_int32, C.c_int32, C.c_int64, P, P]
        _port.orc_choose_spmv.argtypes = [P, P]
        _port.orc_generate.argtypes = [C.c_int, C.c_uint64, C.c_int32, C.POINTER(C.c_int32),
                                       C.POINTER(C.c_int32), C.POINTER(C.c_int64), P, P, P]
        _port.orc_generate.restype = C.c_int
        _port.orc_generate_vector.argtypes = [C.c_uint64, C.c_int64, P]
    return _port


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


def reference_tree():
    """The SpMVBench source tree the tests may read, or None: $SPMVBENCH_REF,
    else the tree oracle/Makefile built _ref/libspmvref.so from (recorded in
    _ref/source_tree), if that directory exists on this machine."""
    path = os.environ.get("SPMVBENCH_REF")
    if not path:
        rec = os.path.join(_HERE, "_ref", "source_tree")
        if os.path.exists(rec):
            with open(rec) as f:
                path = f.read().strip()
    return path if path and os.path.isdir(path) else None


def ref() -> C.CDLL:
    """The reference's own CPU code (raises if it was not built)."""
    global _ref
    if _ref is None:
        if not ref_available():
            raise ImportError(f"{REF_PATH} missing: build it with `make -C {_HERE}` where the "
                              "SpMVBench sources are present")
        lib = C.CDLL(REF_PATH)
        for t, ct in (("d", P), ("f", P)):
            getattr(lib, f"ref_csr_create_{t}").argtypes = [C.c_int32, C.c_int32, C.c_int64, P, P, ct]
            getattr(lib, f"ref_csr_create_{t}").restype = P
            getattr(lib, f"ref_csr_destroy_{t}").argtypes = [P]
        for suf in ("dd", "ff", "fd"):
            getattr(lib, f"ref_spmv_csr_{suf}").argtypes = [P, P, P, C.c_int]
            getattr(lib, f"ref_spmm_csr_{suf}").argtypes = [P, P, P, C.c_int, C.c_int]
        lib.ref_spmv_merge_dd.argtypes = [P, P, P, C.c_int]
        lib.ref_read_mtx_d.argtypes = [C.c_char_p, C.c_char_p, C.c_int]
        lib.ref_read_mtx_d.restype = P
        lib.ref_csr_shape_d.argtypes = [P, C.POINTER(C.c_int32), C.POINTER(C.c_int32), C.POINTER(C.c_int64)]
        lib.ref_csr_arrays_d.argtypes = [P, P, P, P]
        lib.ref_ell_width_d.argtypes = [P]
        lib.ref_ell_width_d.restype = C.c_int32
        lib.ref_csr_to_ell_d.argtypes = [P, P, P, P]
        lib.ref_spmv_ell_dd.argtypes = [P, P, P, C.c_int]
        lib.ref_bcsr_shape_d.argtypes = [P, C.c_int, C.POINTER(C.c_int32), C.POINTER(C.c_int64)]
        lib.ref_csr_to_bcsr_d.argtypes = [P, C.c_int, P, P, P]
        lib.ref_spmv_bcsr_dd.argtypes = [P, C.c_int, P, P, C.c_int]
        lib.ref_row_stats.argtypes = [P, P, C.c_int32, C.c_int32, C.c_int64, P, P, C.c_int64]
        lib.ref_choose_spmv.argtypes = [P, P, C.c_char_p, C.c_int]
        _ref = lib
    return _ref


def ref_read_matrix_market(path: str):
    """The reference's read_matrix_market<double> (src/mtx_io.cpp:40-172),
    run from oracle/_ref: (m, n, rowptr, colind, values), or RuntimeError
    with the reference's message."""
    lib = ref()
    err = C.create_string_buffer(1024)
    h = lib.ref_read_mtx_d(os.fsencode(path), err, 1024)
    if not h:
        raise RuntimeError(err.value.decode(errors="replace"))
    m, n, nnz = C.c_int32(), C.c_int32(), C.c_int64()
    lib.ref_csr_shape_d(h, C.byref(m), C.byref(n), C.byref(nnz))
    rp = np.zeros(m.value + 1, np.int32)
    ci = np.zeros(max(nnz.value, 1), np.int32)
    va = np.zeros(max(nnz.value, 1), np.float64)
    lib.ref_csr_arrays_d(h, _p(rp), _p(ci), _p(va))
    lib.ref_csr_destroy_d(h)
    return m.value, n.value, rp, ci[:nnz.value], va[:nnz.value]


REF_CUDA_PATH = os.path.join(_HERE, "_ref", "libspmvref_cuda.so")
_ref_cuda = None


def ref_cuda_available() -> bool:
    """Whether the reference's own GPU path was built (oracle/Makefile
    `ref_cuda`: src/cuda compiled for sm_100a)."""
    return os.path.exists(REF_CUDA_PATH)


def ref_cuda() -> C.CDLL:
    """The reference's GPU path (its SpmvRunner and spmm_csr_tiled) through
    ref_cuda_shim.cu. Loading needs no GPU; the run functions do, and the
    reference aborts the process on a CUDA error."""
    global _ref_cuda
    if _ref_cuda is None:
        if not ref_cuda_available():
            raise ImportError(f"{REF_CUDA_PATH} missing: run `make -C {_HERE} ref_cuda` with the SpMVBench sources")
        lib = C.CDLL(REF_CUDA_PATH)
        lib.refcuda_available.restype = C.c_int
        lib.refcuda_spmv_dd.argtypes = [C.c_int32, C.c_int32, C.c_int64, P, P, P, P, C.c_int, C.c_int, C.c_int,
                                        C.c_int, C.c_int, P, C.POINTER(C.c_double)]
        lib.refcuda_spmm_dd.argtypes = [C.c_int32, C.c_int32, C.c_int64, P, P, P, P, C.c_int, C.c_int, C.c_int,
                                        C.c_int, C.c_int, P, C.POINTER(C.c_double)]
        lib.refcuda_runner_create_dd.argtypes = [C.c_int32, C.c_int32, C.c_int64, P, P, P, P]
        lib.refcuda_runner_create_dd.restype = P
        lib.refcuda_runner_run.argtypes = [P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_double), P]
        lib.refcuda_runner_destroy.argtypes = [P]
        _ref_cuda = lib
    return _ref_cuda


def ref_cuda_spmv(m, n, rowptr, colind, vals, x, kernel, lanes=4, block=4, iters=10, warmup=3):
    """y and the median launch time (ms) of the reference's kernel `kernel`
    (its KernelId 0..5) on a GPU, fp64."""
    rp = np.ascontiguousarray(rowptr, np.int32)
    ci = np.ascontiguousarray(colind, np.int32)
    va = np.ascontiguousarray(vals, np.float64)
    xx = np.ascontiguousarray(x, np.float64)
    y = np.empty(m, np.float64)
    ms = C.c_double()
    rc = ref_cuda().refcuda_spmv_dd(m, n, int(rp[m]) if m else 0, _p(rp), _p(ci), _p(va), _p(xx), kernel, lanes,
                                    block, iters, warmup, _p(y), C.byref(ms))
    if rc != 0:
        raise ValueError(f"refcuda_spmv_dd: bad kernel id {kernel}")
    return y, ms.value


def ref_cuda_spmm(m, n, rowptr, colind, vals, B, k, tile=32, balanced=False, iters=10, warmup=3):
    """Y (m x k) and the median time (ms) of the reference's spmm_csr_tiled_f64."""
    rp = np.ascontiguousarray(rowptr, np.int32)
    ci = np.ascontiguousarray(colind, np.int32)
    va = np.ascontiguousarray(vals, np.float64)
    BB = np.ascontiguousarray(B, np.float64)
    Y = np.empty((m, k), np.float64)
    ms = C.c_double()
    ref_cuda().refcuda_spmm_dd(m, n, int(rp[m]) if m else 0, _p(rp), _p(ci), _p(va), _p(BB), k, tile, int(balanced),
                               iters, warmup, _p(Y), C.byref(ms))
    return Y, ms.value


class RefCudaRunner:
    """The reference's SpmvRunner<double,double> on the current GPU, built
    once for a matrix (its eager ELL / BCSR uploads) with x loaded."""

    def __init__(self, m, n, rowptr, colind, vals, x):
        self._keep = [np.ascontiguousarray(rowptr, np.int32), np.ascontiguousarray(colind, np.int32),
                      np.ascontiguousarray(vals, np.float64), np.ascontiguousarray(x, np.float64)]
        rp, ci, va, xx = self._keep
        self.m = m
        self.h = ref_cuda().refcuda_runner_create_dd(m, n, int(rp[m]) if m else 0, _p(rp), _p(ci), _p(va), _p(xx))
        if not self.h:
            raise ValueError("refcuda_runner_create_dd: bad sizes")

    def run(self, kernel, lanes=4, block=4, iters=20, warmup=5, want_y=False):
        """(median ms of the reference's per-launch timing, y or None)."""
        ms = C.c_double()
        y = np.empty(self.m, np.float64) if want_y else None
        if ref_cuda().refcuda_runner_run(self.h, kernel, lanes, block, iters, warmup, C.byref(ms), _p(y)) != 0:
            raise ValueError(f"refcuda_runner_run: bad kernel id {kernel}")
        return ms.value, y

    def close(self):
        if self.h:
            ref_cuda().refcuda_runner_destroy(self.h)
            self.h = None


_SUF = {(np.float64, np.float64): "dd", (np.float32, np.float32): "ff", (np.float32, np.float64): "fd"}


def _suf(vals, acc):
    return _SUF[(np.dtype(vals.dtype).type, np.dtype(acc).type)]


# ---- the C restatement --------------------------------------------------------
def spmv_csr(m, rowptr, colind, vals, x, acc=None, nthreads=0):
    acc = vals.dtype if acc is None else acc
    y = np.empty(m, acc)
    getattr(port(), f"orc_spmv_csr_{_suf(vals, acc)}")(m, _p(rowptr), _p(colind), _p(vals), _p(x), _p(y), nthreads)
    return y


def spmv_ell(m, ecol, evals, row_lengths, x, acc=None, nthreads=0):
    acc = evals.dtype if acc is None else acc
    y = np.empty(m, acc)
    getattr(port(), f"orc_spmv_ell_{_suf(evals, acc)}")(m, _p(ecol), _p(evals), _p(row_lengths), _p(x), _p(y), nthreads)
    return y


def spmv_bcsr(m, n, R, Cc, browptr, bcol, bvals, x, acc=None, nthreads=0):
    acc = bvals.dtype if acc is None else acc
    y = np.empty(m, acc)
    mb = browptr.size - 1
    getattr(port(), f"orc_spmv_bcsr_{_suf(bvals, acc)}")(m, n, R, Cc, mb, _p(browptr), _p(bcol), _p(bvals),
                                                         _p(x), _p(y), nthreads)
    return y


def spmm_csr(m, k, rowptr, colind, vals, B, acc=None, nthreads=0):
    acc = vals.dtype if acc is None else acc
    Y = np.empty((m, k), acc)
    getattr(port(), f"orc_spmm_csr_{_suf(vals, acc)}")(m, k, _p(rowptr), _p(colind), _p(vals), _p(B), _p(Y), nthreads)
    return Y


def csr_to_ell(m, rowptr, colind, vals):
    w = port().orc_ell_width(m, _p(rowptr))
    ecol = np.zeros(m * w, np.int32)
    ev = np.zeros(m * w, vals.dtype)
    rl = np.zeros(m, np.int32)
    port().orc_csr_to_ell(m, _p(rowptr), _p(colind), _p(vals), vals.itemsize, _p(ecol), _p(ev), _p(rl))
    return w, ecol, ev, rl


def csr_to_bcsr(m, n, block, rowptr, colind, vals):
    mb, bn = C.c_int32(), C.c_int64()
    lib = port()
    lib.orc_csr_to_bcsr(m, n, block, block, _p(rowptr), _p(colind), _p(vals), vals.itemsize,
                        C.byref(mb), C.byref(bn), None, None, None)
    rp = np.zeros(mb.value + 1, np.int32)
    ci = np.zeros(max(bn.value, 1), np.int32)
    va = np.zeros(max(bn.value, 1) * block * block, vals.dtype)
    lib.orc_csr_to_bcsr(m, n, block, block, _p(rowptr), _p(colind), _p(vals), vals.itemsize,
                        C.byref(mb), C.byref(bn), _p(rp), _p(ci), _p(va))
    return rp, ci[:bn.value], va[:bn.value * block * block]


STAT_FIELDS = ["nnz", "rows", "cols", "mean_row_nnz", "median_row_nnz", "min_row_nnz", "max_row_nnz",
               "stddev_row_nnz", "cv_row_nnz", "max_over_mean", "ell_padding_overhead",
               "frac_dense_blocks_4x4", "density"]


def row_stats(m, n, rowptr, colind):
    out = np.zeros(13, np.float64)
    mx = int(np.max(np.diff(rowptr))) if m else 0
    hist = np.zeros(mx + 1, np.int64)
    nnz = int(rowptr[m]) if m else 0
    port().orc_row_stats(_p(rowptr), _p(colind) if colind is not None else None, m, n, nnz, _p(out), _p(hist))
    d = dict(zip(STAT_FIELDS, out.tolist()))
    d["row_nnz_histogram"] = hist
    return d


def choose_spmv(stats: dict):
    s = np.array([float(stats.get(f, 0)) for f in STAT_FIELDS], np.float64)
    out = np.zeros(5, np.int32)
    port().orc_choose_spmv(_p(s), _p(out))
    return {"kernel": int(out[0]), "lanes": int(out[1]), "block_r": int(out[2]), "block_c": int(out[3]),
            "rule": int(out[4])}


def generate(which: int, seed: int, scale_rows: int = 0):
    """Seeded workload `which` (1, 2, 4 or 5) from the oracle's own statement
    of the generator: (m, n, rowptr, colind, values). Identical to the
    library's spmvb_generate (tests/test_oracle.py), without loading it."""
    lib = port()
    m, n, nnz = C.c_int32(), C.c_int32(), C.c_int64()
    if lib.orc_generate(which, seed, scale_rows, C.byref(m), C.byref(n), C.byref(nnz), None, None, None) != 0:
        raise ValueError(f"orc_generate: workload {which} with {scale_rows} rows is not covered")
    rp = np.zeros(m.value + 1, np.int32)
    ci = np.zeros(max(nnz.value, 1), np.int32)
    va = np.zeros(max(nnz.value, 1), np.float64)
    lib.orc_generate(which, seed, scale_rows, C.byref(m), C.byref(n), C.byref(nnz), _p(rp), _p(ci), _p(va))
    return m.value, n.value, rp, ci[:nnz.value], va[:nnz.value]


def generate_vector(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float64)
    port().orc_generate_vector(seed, n, _p(out))
    return out


# ---- the reference itself -------------------------------------------------------
class RefCsr:
    """A CsrMatrix<T> owned by the reference library."""

    def __init__(self, m, n, rowptr, colind, vals):
        self.lib = ref()
        self.t = "d" if vals.dtype == np.float64 else "f"
        self._keep = (rowptr, colind, vals)
        self.h = getattr(self.lib, f"ref_csr_create_{self.t}")(m, n, int(rowptr[m]) if m else 0,
                                                               _p(rowptr), _p(colind), _p(vals))
        self.m, self.n, self.vdtype = m, n, vals.dtype

    def close(self):
        if self.h:
            getattr(self.lib, f"ref_csr_destroy_{self.t}")(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def spmv(self, x, acc=None, nthreads=0, out=None):
        acc = self.vdtype if acc is None else acc
        y = out if out is not None else np.empty(self.m, acc)
        getattr(self.lib, f"ref_spmv_csr_{_SUF[(np.dtype(self.vdtype).type, np.dtype(acc).type)]}")(
            self.h, _p(x), _p(y), nthreads)
        return y

    def spmm(self, B, k, acc=None, nthreads=0):
        acc = self.vdtype if acc is None else acc
        Y = np.empty((self.m, k), acc)
        getattr(self.lib, f"ref_spmm_csr_{_SUF[(np.dtype(self.vdtype).type, np.dtype(acc).type)]}")(
            self.h, _p(B), _p(Y), k, nthreads)
        return Y


def gamma_ratio(rowptr, colind, vals, x, ref_y, got_y, acc):
    """Largest per-row |got - ref| / (2*gamma_n(u)*sum|a x| + 1e-30), the
    reference's GPU-test criterion (tests/test_cuda_correctness.cpp:53-56,73-104);
    <= 1 passes. Returns (ratio, row)."""
    m = rowptr.size - 1
    if m == 0:
        return 0.0, -1
    u = 2.0 ** -53 if np.dtype(acc) == np.float64 else 2.0 ** -24
    lens = np.diff(rowptr).astype(np.int64)
    rows = np.repeat(np.arange(m), lens)
    abs_sum = np.bincount(rows, weights=np.abs(vals.astype(np.float64) * x.astype(np.float64)[colind]),
                          minlength=m)
    nu = lens * u
    bound = 2.0 * (nu / (1.0 - nu)) * abs_sum + 1e-30
    diff = np.abs(got_y.astype(np.float64) - ref_y.astype(np.float64))
    ratio = diff / bound
    i = int(np.argmax(ratio))
    return float(ratio[i]), i


def gamma_ratio_spmm(rowptr, colind, vals, B, k, ref_Y, got_Y, acc):
    """Per-element version for SpMM (tests/test_cuda_correctness.cpp:140-180)."""
    m = rowptr.size - 1
    if m == 0 or k == 0:
        return 0.0, (-1, -1)
    u = 2.0 ** -53 if np.dtype(acc) == np.float64 else 2.0 ** -24
    lens = np.diff(rowptr).astype(np.int64)
    rows = np.repeat(np.arange(m), lens)
    prod = np.abs(vals.astype(np.float64)[:, None] * B.astype(np.float64).reshape(-1, k)[colind])
    abs_sum = np.zeros((m, k))
    np.add.at(abs_sum, rows, prod)
    nu = lens * u
    bound = 2.0 * (nu / (1.0 - nu))[:, None] * abs_sum + 1e-30
    ratio = np.abs(got_Y.astype(np.float64) - ref_Y.astype(np.float64)) / bound
    idx = np.unravel_index(int(np.argmax(ratio)), ratio.shape)
    return float(ratio[idx]), (int(idx[0]), int(idx[1]))
