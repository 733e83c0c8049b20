#pragma once
// Vendor baselines of the reference's bench: cuSPARSE CSR SpMV and CSR x
// dense SpMM with the same names and signatures as SpMVBench's
// cusparse_spmv_csr_f32/f64 (include/spmvbench/spmv_cuda.cuh:170-180) and
// cusparse_spmm_f32/f64 (include/spmvbench/spmm_cuda.cuh:42-49), so the
// reference's bench (bench/bench_main.cpp:643-650, 700-722) compiles and runs
// its comparison rows unchanged against this drop-in. They are comparisons
// only: nothing in libspmvb calls cuSPARSE.
//
// Header-only; included by spmv_cuda.cuh / spmm_cuda.cuh when
// SPMVBENCH_ENABLE_CUDA is defined and SPMVB_NO_CUSPARSE is not. Link with
// -lcusparse (CMake: CUDA::cusparse), as the reference's bench target does.
//
// Protocol, as the reference's baselines: upload A and x (B) once, `warmup`
// untimed calls, then `iters` calls each timed by its own event pair and
// summarized (mean / min / median / max); y (Y) is copied back; transfer_ms is
// the median of 10 rounds of one upload of x (B) and one download of y (Y).
// Errors throw std::runtime_error, as the rest of the drop-in does.
#if defined(SPMVBENCH_ENABLE_CUDA) && !defined(SPMVB_NO_CUSPARSE)

#include <cuda_runtime.h>
#include <cusparse.h>

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <vector>

#include "spmvbench/csr.hpp"
#include "spmvbench/timer.hpp"

namespace spmvbench {
namespace vendor {

inline void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
inline void check_sparse(cusparseStatus_t s, const char* what) {
  if (s != CUSPARSE_STATUS_SUCCESS) throw std::runtime_error(std::string(what) + ": " + cusparseGetErrorString(s));
}
template <typename T>
constexpr cudaDataType_t data_type() {
  return std::is_same_v<T, double> ? CUDA_R_64F : CUDA_R_32F;
}

// One device allocation, freed on scope exit (at least 1 byte, so empty
// operands still get a valid pointer).
class DeviceArray {
 public:
  explicit DeviceArray(std::size_t bytes) { check_cuda(cudaMalloc(&p_, bytes ? bytes : 1), "cudaMalloc"); }
  ~DeviceArray() {
    if (p_) cudaFree(p_);
  }
  DeviceArray(const DeviceArray&) = delete;
  DeviceArray& operator=(const DeviceArray&) = delete;
  template <typename U>
  U* as() const {
    return static_cast<U*>(p_);
  }
  void upload(const void* h, std::size_t bytes) {
    if (bytes) check_cuda(cudaMemcpy(p_, h, bytes, cudaMemcpyHostToDevice), "cudaMemcpy H2D");
  }

 private:
  void* p_ = nullptr;
};

// The handle, the CSR descriptor of A and the event pair one baseline call
// needs; the dense descriptors are added by the caller.
template <typename T>
class SparseCsr {
 public:
  explicit SparseCsr(const CsrMatrix<T>& A)
      : rowptr_(static_cast<std::size_t>(A.m + 1) * sizeof(Index)),
        colind_(static_cast<std::size_t>(A.nnz) * sizeof(Index)),
        values_(static_cast<std::size_t>(A.nnz) * sizeof(T)) {
    rowptr_.upload(A.rowptr.data(), static_cast<std::size_t>(A.m + 1) * sizeof(Index));
    colind_.upload(A.colind.data(), static_cast<std::size_t>(A.nnz) * sizeof(Index));
    values_.upload(A.values.data(), static_cast<std::size_t>(A.nnz) * sizeof(T));
    check_sparse(cusparseCreate(&handle_), "cusparseCreate");
    check_sparse(cusparseCreateCsr(&mat_, A.m, A.n, A.nnz, rowptr_.as<Index>(), colind_.as<Index>(),
                                   values_.as<T>(), CUSPARSE_INDEX_32I, CUSPARSE_INDEX_32I,
                                   CUSPARSE_INDEX_BASE_ZERO, data_type<T>()),
                 "cusparseCreateCsr");
    check_cuda(cudaEventCreate(&start_), "cudaEventCreate");
    check_cuda(cudaEventCreate(&stop_), "cudaEventCreate");
  }
  ~SparseCsr() {
    if (stop_) cudaEventDestroy(stop_);
    if (start_) cudaEventDestroy(start_);
    if (mat_) cusparseDestroySpMat(mat_);
    if (handle_) cusparseDestroy(handle_);
  }
  SparseCsr(const SparseCsr&) = delete;
  SparseCsr& operator=(const SparseCsr&) = delete;

  cusparseHandle_t handle() const { return handle_; }
  cusparseSpMatDescr_t mat() const { return mat_; }

  // Event-pair time of each of `iters` calls of f, after `warmup` untimed calls.
  template <typename F>
  std::vector<double> time_calls(F&& f, int iters, int warmup) {
    for (int i = 0; i < warmup; ++i) f();
    check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    std::vector<double> samples;
    samples.reserve(static_cast<std::size_t>(iters > 0 ? iters : 0));
    for (int i = 0; i < iters; ++i) {
      check_cuda(cudaEventRecord(start_), "cudaEventRecord");
      f();
      check_cuda(cudaEventRecord(stop_), "cudaEventRecord");
      check_cuda(cudaEventSynchronize(stop_), "cudaEventSynchronize");
      float ms = 0.f;
      check_cuda(cudaEventElapsedTime(&ms, start_, stop_), "cudaEventElapsedTime");
      samples.push_back(static_cast<double>(ms));
    }
    return samples;
  }

 private:
  DeviceArray rowptr_, colind_, values_;
  cusparseHandle_t handle_ = nullptr;
  cusparseSpMatDescr_t mat_ = nullptr;
  cudaEvent_t start_ = nullptr, stop_ = nullptr;
};

// Median time of 10 rounds of one upload of `in` and one download into `out`.
inline double transfer_ms(void* d_in, const void* h_in, std::size_t in_bytes, void* h_out, const void* d_out,
                          std::size_t out_bytes) {
  if (in_bytes == 0 || out_bytes == 0) return 0.0;
  cudaEvent_t a = nullptr, b = nullptr;
  check_cuda(cudaEventCreate(&a), "cudaEventCreate");
  check_cuda(cudaEventCreate(&b), "cudaEventCreate");
  std::vector<double> samples;
  for (int i = 0; i < 10; ++i) {
    cudaEventRecord(a);
    cudaMemcpy(d_in, h_in, in_bytes, cudaMemcpyHostToDevice);
    cudaMemcpy(h_out, d_out, out_bytes, cudaMemcpyDeviceToHost);
    cudaEventRecord(b);
    cudaEventSynchronize(b);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, a, b);
    samples.push_back(static_cast<double>(ms));
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  return summarize(samples).median_ms;
}

// y = A x through cusparseSpMV (CSR, CUSPARSE_SPMV_ALG_DEFAULT). Fills the
// summary fields of Result (SpmvResult).
template <typename Result, typename T>
Result spmv(const CsrMatrix<T>& A, const std::vector<T>& x, std::vector<T>& y, int iters, int warmup) {
  if (x.size() < static_cast<std::size_t>(A.n)) throw std::runtime_error("cusparse_spmv_csr: x shorter than n");
  SparseCsr<T> S(A);
  DeviceArray dx(static_cast<std::size_t>(A.n) * sizeof(T)), dy(static_cast<std::size_t>(A.m) * sizeof(T));
  dx.upload(x.data(), static_cast<std::size_t>(A.n) * sizeof(T));
  cusparseDnVecDescr_t vx = nullptr, vy = nullptr;
  check_sparse(cusparseCreateDnVec(&vx, A.n, dx.as<T>(), data_type<T>()), "cusparseCreateDnVec");
  check_sparse(cusparseCreateDnVec(&vy, A.m, dy.as<T>(), data_type<T>()), "cusparseCreateDnVec");
  const T one = T(1), zero = T(0);
  std::size_t bytes = 0;
  check_sparse(cusparseSpMV_bufferSize(S.handle(), CUSPARSE_OPERATION_NON_TRANSPOSE, &one, S.mat(), vx, &zero, vy,
                                       data_type<T>(), CUSPARSE_SPMV_ALG_DEFAULT, &bytes),
               "cusparseSpMV_bufferSize");
  DeviceArray work(bytes);
  const auto samples = S.time_calls(
      [&] {
        check_sparse(cusparseSpMV(S.handle(), CUSPARSE_OPERATION_NON_TRANSPOSE, &one, S.mat(), vx, &zero, vy,
                                  data_type<T>(), CUSPARSE_SPMV_ALG_DEFAULT, work.as<void>()),
                     "cusparseSpMV");
      },
      iters, warmup);
  y.assign(static_cast<std::size_t>(A.m), T(0));
  if (A.m) check_cuda(cudaMemcpy(y.data(), dy.as<T>(), y.size() * sizeof(T), cudaMemcpyDeviceToHost), "D2H y");
  Result r;
  const TimingSummary st = summarize(samples);
  r.mean_ms = st.mean_ms;
  r.min_ms = st.min_ms;
  r.median_ms = st.median_ms;
  r.max_ms = st.max_ms;
  r.iters = st.iters;
  r.transfer_ms = transfer_ms(dx.as<void>(), x.data(), static_cast<std::size_t>(A.n) * sizeof(T), y.data(),
                              dy.as<void>(), y.size() * sizeof(T));
  r.kernel = "cusparse_spmv";
  cusparseDestroyDnVec(vx);
  cusparseDestroyDnVec(vy);
  return r;
}

// Y (m x k) = A B (B n x k), both row-major, through cusparseSpMM (CSR x
// dense, CUSPARSE_SPMM_ALG_DEFAULT). Fills the summary fields of Result.
template <typename Result, typename T>
Result spmm(const CsrMatrix<T>& A, const std::vector<T>& B, int k, std::vector<T>& Y, int iters, int warmup) {
  if (k < 0) throw std::runtime_error("cusparse_spmm: negative k");
  const std::size_t bn = static_cast<std::size_t>(A.n) * k, yn = static_cast<std::size_t>(A.m) * k;
  if (B.size() < bn) throw std::runtime_error("cusparse_spmm: B holds fewer than n*k values");
  SparseCsr<T> S(A);
  DeviceArray dB(bn * sizeof(T)), dY(yn * sizeof(T));
  dB.upload(B.data(), bn * sizeof(T));
  cusparseDnMatDescr_t mb = nullptr, my = nullptr;
  check_sparse(cusparseCreateDnMat(&mb, A.n, k, k, dB.as<T>(), data_type<T>(), CUSPARSE_ORDER_ROW),
               "cusparseCreateDnMat");
  check_sparse(cusparseCreateDnMat(&my, A.m, k, k, dY.as<T>(), data_type<T>(), CUSPARSE_ORDER_ROW),
               "cusparseCreateDnMat");
  const T one = T(1), zero = T(0);
  std::size_t bytes = 0;
  check_sparse(cusparseSpMM_bufferSize(S.handle(), CUSPARSE_OPERATION_NON_TRANSPOSE, CUSPARSE_OPERATION_NON_TRANSPOSE,
                                       &one, S.mat(), mb, &zero, my, data_type<T>(), CUSPARSE_SPMM_ALG_DEFAULT,
                                       &bytes),
               "cusparseSpMM_bufferSize");
  DeviceArray work(bytes);
  const auto samples = S.time_calls(
      [&] {
        check_sparse(cusparseSpMM(S.handle(), CUSPARSE_OPERATION_NON_TRANSPOSE, CUSPARSE_OPERATION_NON_TRANSPOSE, &one,
                                  S.mat(), mb, &zero, my, data_type<T>(), CUSPARSE_SPMM_ALG_DEFAULT, work.as<void>()),
                     "cusparseSpMM");
      },
      iters, warmup);
  Y.assign(yn, T(0));
  if (yn) check_cuda(cudaMemcpy(Y.data(), dY.as<T>(), yn * sizeof(T), cudaMemcpyDeviceToHost), "D2H Y");
  Result r;
  const TimingSummary st = summarize(samples);
  r.mean_ms = st.mean_ms;
  r.min_ms = st.min_ms;
  r.median_ms = st.median_ms;
  r.max_ms = st.max_ms;
  r.iters = st.iters;
  r.transfer_ms = transfer_ms(dB.as<void>(), B.data(), bn * sizeof(T), Y.data(), dY.as<void>(), yn * sizeof(T));
  r.kernel = "cusparse_spmm";
  cusparseDestroyDnMat(mb);
  cusparseDestroyDnMat(my);
  return r;
}

}  // namespace vendor
}  // namespace spmvbench

#endif  // SPMVBENCH_ENABLE_CUDA && !SPMVB_NO_CUSPARSE
