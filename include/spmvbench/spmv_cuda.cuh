#pragma once
// GPU SpMV drop-in (same interface as SpMVBench's
// include/spmvbench/spmv_cuda.cuh; compiled only when SPMVBENCH_ENABLE_CUDA is
// defined, like the reference). SpmvRunner keeps its constructor, set_x, run,
// result and storage-size helpers; the kernels are libspmvb's sm_100a kernels
// behind include/spmvb.h. Errors throw std::runtime_error carrying the
// library's message (the reference aborts; an uncaught exception terminates).
// Formats are built on the device when first needed and outside the timed
// loop, instead of eagerly in the constructor.
#ifdef SPMVBENCH_ENABLE_CUDA

#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "spmvb.h"
#include "spmvbench/csr.hpp"
#include "spmvbench/select.hpp"
#include "spmvbench/timer.hpp"

namespace spmvbench {

namespace detail {
inline void check(spmvb_status s, const char* what) {
  if (s != SPMVB_OK) throw std::runtime_error(std::string(what) + ": " + spmvb_last_error());
}
inline void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
template <typename U>
constexpr spmvb_dtype dtype_of() {
  return std::is_same_v<U, double> ? SPMVB_F64 : SPMVB_F32;
}
}  // namespace detail

// Device views (include/spmvbench/spmv_cuda.cuh:53-84), kept for callers that
// name them.
template <typename T>
struct DeviceCsr {
  const Index* rowptr = nullptr;
  const Index* colind = nullptr;
  const T* values = nullptr;
  int m = 0;
  int n = 0;
  std::int64_t nnz = 0;
};
template <typename T>
struct DeviceEll {
  const Index* colind = nullptr;
  const T* values = nullptr;
  const int* row_lengths = nullptr;
  int m = 0;
  int n = 0;
  int max_row_nnz = 0;
};
template <typename T>
struct DeviceBcsr {
  const Index* rowptr = nullptr;
  const Index* colind = nullptr;
  const T* values = nullptr;
  int m = 0;
  int n = 0;
  int R = 1;
  int C = 1;
  int mb = 0;
  std::int64_t block_nnz = 0;
};

struct SpmvResult {
  double mean_ms = 0.0;
  double min_ms = 0.0;
  double median_ms = 0.0;
  double max_ms = 0.0;
  double transfer_ms = 0.0;
  int iters = 0;
  std::string kernel;
};

struct GpuInfo {
  std::string name;
  int major = 0;
  int minor = 0;
  double peak_gbs = 0.0;
  bool peak_known = false;
};

inline bool gpu_available() { return spmvb_gpu_available() != 0; }

inline GpuInfo query_gpu() {
  int dev = 0;
  detail::check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  spmvb_gpu_info g{};
  detail::check(spmvb_query_gpu(dev, &g), "query_gpu");
  return GpuInfo{g.name, g.major, g.minor, g.peak_gbs, g.peak_known != 0};
}

template <typename T, typename Acc>
class SpmvRunner {
  static_assert((std::is_same_v<T, float> && (std::is_same_v<Acc, float> || std::is_same_v<Acc, double>)) ||
                    (std::is_same_v<T, double> && std::is_same_v<Acc, double>),
                "instantiated for (float,float), (float,double), (double,double)");

 public:
  explicit SpmvRunner(const CsrMatrix<T>& A) : A_(A) {
    int dev = 0;
    detail::check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    detail::check(spmvb_context_create(dev, &ctx_), "spmvb_context_create");
    detail::check(spmvb_matrix_create_csr(ctx_, detail::dtype_of<T>(), A.m, A.n, A.nnz, A.rowptr.data(),
                                          A.colind.data(), A.values.data(), &mat_),
                  "spmvb_matrix_create_csr");
    detail::check_cuda(cudaMalloc(&d_x_, sizeof(T) * (A.n > 0 ? A.n : 1)), "cudaMalloc x");
    detail::check_cuda(cudaMalloc(&d_y_, sizeof(Acc) * (A.m > 0 ? A.m : 1)), "cudaMalloc y");
  }
  ~SpmvRunner() {
    cudaFree(d_x_);
    cudaFree(d_y_);
    spmvb_matrix_destroy(mat_);
    spmvb_context_destroy(ctx_);
  }
  SpmvRunner(const SpmvRunner&) = delete;
  SpmvRunner& operator=(const SpmvRunner&) = delete;

  // x must hold exactly n values (the reference copies x.size() values into
  // its n-entry device buffer whatever that size is).
  void set_x(const std::vector<T>& x) {
    if (x.size() != static_cast<std::size_t>(A_.n))
      throw std::runtime_error("set_x: x holds " + std::to_string(x.size()) + " values, n = " +
                               std::to_string(A_.n));
    host_x_ = x;
    if (!x.empty())
      detail::check_cuda(cudaMemcpy(d_x_, x.data(), x.size() * sizeof(T), cudaMemcpyHostToDevice), "set_x");
  }

  // `iters` timed launches of kernel `id` after `warmup` untimed ones; each
  // launch has its own event pair, summarized like the reference
  // (src/cuda/spmv_cuda.cu:466-497). The format the kernel needs is built
  // before timing.
  SpmvResult run(KernelId id, int iters, int lanes = 4, int block = 4, int warmup = 5) {
    const auto k = static_cast<spmvb_kernel>(id);
    detail::check(spmvb_matrix_prepare(mat_, k, k == SPMVB_BCSR ? (block <= 2 ? 2 : 4) : 0), "prepare");
    const spmvb_dtype acc = detail::dtype_of<Acc>();
    auto launch = [&] { detail::check(spmvb_spmv(mat_, k, lanes, block, d_x_, d_y_, acc, nullptr), "spmvb_spmv"); };
    for (int i = 0; i < warmup; ++i) launch();
    detail::check_cuda(cudaDeviceSynchronize(), "warmup");
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    std::vector<double> samples;
    for (int i = 0; i < iters; ++i) {
      cudaEventRecord(a);
      launch();
      cudaEventRecord(b);
      cudaEventSynchronize(b);
      float ms = 0.f;
      cudaEventElapsedTime(&ms, a, b);
      samples.push_back(ms);
    }
    detail::check(spmvb_context_check(ctx_), "spmv");
    const TimingSummary st = summarize(samples);
    SpmvResult r;
    r.iters = st.iters;
    r.mean_ms = st.mean_ms;
    r.min_ms = st.min_ms;
    r.median_ms = st.median_ms;
    r.max_ms = st.max_ms;
    r.transfer_ms = measure_transfer_ms(10, a, b);
    r.kernel = kernel_name(id);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return r;
  }

  std::vector<Acc> result() const {
    std::vector<Acc> y(static_cast<std::size_t>(A_.m));
    if (A_.m > 0)
      detail::check_cuda(cudaMemcpy(y.data(), d_y_, A_.m * sizeof(Acc), cudaMemcpyDeviceToHost), "result");
    return y;
  }

  std::int64_t ell_padded_nnz() const { return info().ell_padded_nnz; }
  std::int64_t ell_touched_nnz() const { return info().ell_touched_nnz; }
  std::int64_t bcsr_block_nnz(int block) const {
    const int b = block <= 2 ? 2 : 4;
    detail::check(spmvb_matrix_prepare(mat_, SPMVB_BCSR, b), "prepare bcsr");
    return b == 2 ? info().bcsr2_block_nnz : info().bcsr4_block_nnz;
  }

 private:
  spmvb_matrix_info info() const {
    spmvb_matrix_info i{};
    detail::check(spmvb_matrix_get_info(mat_, &i), "spmvb_matrix_get_info");
    return i;
  }
  double measure_transfer_ms(int iters, cudaEvent_t a, cudaEvent_t b) {
    if (A_.m == 0 || A_.n == 0 || host_x_.empty()) return 0.0;
    std::vector<Acc> host_y(static_cast<std::size_t>(A_.m));
    std::vector<double> samples;
    for (int i = 0; i < iters; ++i) {
      cudaEventRecord(a);
      cudaMemcpy(d_x_, host_x_.data(), host_x_.size() * sizeof(T), cudaMemcpyHostToDevice);
      cudaMemcpy(host_y.data(), d_y_, A_.m * sizeof(Acc), cudaMemcpyDeviceToHost);
      cudaEventRecord(b);
      cudaEventSynchronize(b);
      float ms = 0.f;
      cudaEventElapsedTime(&ms, a, b);
      samples.push_back(ms);
    }
    return summarize(samples).median_ms;
  }

  const CsrMatrix<T> A_;
  std::vector<T> host_x_;
  spmvb_context ctx_ = nullptr;
  spmvb_matrix mat_ = nullptr;
  T* d_x_ = nullptr;
  Acc* d_y_ = nullptr;
};

}  // namespace spmvbench

#include "spmvbench/cusparse_baseline.hpp"

#ifndef SPMVB_NO_CUSPARSE
namespace spmvbench {
// The reference bench's cuSPARSE SpMV baseline (spmv_cuda.cuh:170-180 of
// SpMVBench): a comparison row, not a library kernel.
inline SpmvResult cusparse_spmv_csr_f32(const CsrMatrix<float>& A, const std::vector<float>& x,
                                        std::vector<float>& y, int iters, int warmup) {
  return vendor::spmv<SpmvResult>(A, x, y, iters, warmup);
}
inline SpmvResult cusparse_spmv_csr_f64(const CsrMatrix<double>& A, const std::vector<double>& x,
                                        std::vector<double>& y, int iters, int warmup) {
  return vendor::spmv<SpmvResult>(A, x, y, iters, warmup);
}
}  // namespace spmvbench
#endif  // SPMVB_NO_CUSPARSE

#endif  // SPMVBENCH_ENABLE_CUDA
