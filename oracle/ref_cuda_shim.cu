// ref_cuda_shim.cu - extern "C" entry points over the REFERENCE's own GPU
// path (its SpmvRunner and spmm_csr_tiled, src/cuda/spmv_cuda.cu and
// spmm_cuda.cu, compiled for sm_100a where they lie in the SpMVBench tree by
// oracle/Makefile's `ref_cuda` target) into oracle/_ref/libspmvref_cuda.so.
// Test infrastructure only: it lets a test run the reference's own kernels
// on the same B200 and inputs as this library's, as a parity and timing
// comparison. The reference aborts on a CUDA error (CUDA_CHECK).
//
// The reference namespace is renamed to spmvbench_refcuda at compile time
// (-Dspmvbench=spmvbench_refcuda), so nothing collides with the drop-in API.
#include <cstdint>
#include <vector>

#include "spmvbench/csr.hpp"
#include "spmvbench/spmm_cuda.cuh"
#include "spmvbench/spmv_cuda.cuh"

namespace R = spmvbench;

namespace {
R::CsrMatrix<double> make(int32_t m, int32_t n, int64_t nnz, const int32_t* rp, const int32_t* ci, const double* v) {
  R::CsrMatrix<double> A(m, n);
  A.nnz = nnz;
  A.rowptr.assign(rp, rp + m + 1);
  A.colind.assign(ci, ci + nnz);
  A.values.assign(v, v + nnz);
  return A;
}
}  // namespace

extern "C" {

// The reference's gpu_available() (never aborts).
int refcuda_available(void) { return R::gpu_available() ? 1 : 0; }

// y = A x with the reference's kernel `kernel` (its KernelId 0..5), `lanes`
// and `block` as its SpmvRunner::run takes them; `iters` timed launches after
// `warmup`. Writes y (m doubles) and the median launch time in ms.
int refcuda_spmv_dd(int32_t m, int32_t n, int64_t nnz, const int32_t* rp, const int32_t* ci, const double* v,
                    const double* x, int kernel, int lanes, int block, int iters, int warmup, double* y,
                    double* median_ms) {
  if (kernel < 0 || kernel > 5) return 1;
  const R::CsrMatrix<double> A = make(m, n, nnz, rp, ci, v);
  R::SpmvRunner<double, double> runner(A);
  runner.set_x(std::vector<double>(x, x + n));
  const R::SpmvResult r = runner.run(static_cast<R::KernelId>(kernel), iters, lanes, block, warmup);
  const std::vector<double> out = runner.result();
  for (int32_t i = 0; i < m; ++i) y[i] = out[i];
  *median_ms = r.median_ms;
  return 0;
}

// A reference SpmvRunner<double,double> built once (its eager uploads and
// conversions, src/cuda/spmv_cuda.cu:233-290) with x loaded, for timing
// several kernels on one matrix. NULL for a bad size.
void* refcuda_runner_create_dd(int32_t m, int32_t n, int64_t nnz, const int32_t* rp, const int32_t* ci,
                               const double* v, const double* x) {
  if (m < 0 || n < 0 || nnz < 0) return nullptr;
  const R::CsrMatrix<double> A = make(m, n, nnz, rp, ci, v);
  auto* runner = new R::SpmvRunner<double, double>(A);
  runner->set_x(std::vector<double>(x, x + n));
  return runner;
}

// SpmvRunner::run(kernel, iters, lanes, block, warmup): the median of its
// per-launch event pairs; y (m doubles) is copied out when non-null.
int refcuda_runner_run(void* h, int kernel, int lanes, int block, int iters, int warmup, double* median_ms,
                       double* y) {
  if (!h || kernel < 0 || kernel > 5) return 1;
  auto* runner = static_cast<R::SpmvRunner<double, double>*>(h);
  const R::SpmvResult r = runner->run(static_cast<R::KernelId>(kernel), iters, lanes, block, warmup);
  *median_ms = r.median_ms;
  if (y) {
    const std::vector<double> out = runner->result();
    for (size_t i = 0; i < out.size(); ++i) y[i] = out[i];
  }
  return 0;
}

void refcuda_runner_destroy(void* h) { delete static_cast<R::SpmvRunner<double, double>*>(h); }

// Y = A B (row-major, k columns) with the reference's spmm_csr_tiled_f64.
int refcuda_spmm_dd(int32_t m, int32_t n, int64_t nnz, const int32_t* rp, const int32_t* ci, const double* v,
                    const double* B, int k, int tile, int balanced, int iters, int warmup, double* Y,
                    double* median_ms) {
  const R::CsrMatrix<double> A = make(m, n, nnz, rp, ci, v);
  std::vector<double> out;
  const R::SpmmResult r = R::spmm_csr_tiled_f64(A, std::vector<double>(B, B + static_cast<size_t>(n) * k), k, tile,
                                                balanced != 0, iters, warmup, out);
  for (size_t i = 0; i < out.size(); ++i) Y[i] = out[i];
  *median_ms = r.median_ms;
  return 0;
}

}  // extern "C"
