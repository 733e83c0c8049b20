#pragma once
// GPU SpMM drop-in (same interface as SpMVBench's
// include/spmvbench/spmm_cuda.cuh:21-41): Y (m x k) = A (CSR) * B (n x k),
// row-major, timed over `iters` launches after `warmup`. `tile` in
// {16, 32, 64} (else 32), `balanced` selects the row-length-bucketed variant.
// Unlike the reference, the bucketed variant builds its buckets once per call
// on the matrix handle instead of allocating and syncing inside every launch.
#ifdef SPMVBENCH_ENABLE_CUDA

#include <vector>

#include "spmvbench/spmv_cuda.cuh"

namespace spmvbench {

struct SpmmResult {
  double mean_ms = 0.0;
  double min_ms = 0.0;
  double median_ms = 0.0;
  double max_ms = 0.0;
  double transfer_ms = 0.0;
  int iters = 0;
  std::string kernel;
};

namespace detail {
template <typename T>
SpmmResult run_spmm(const CsrMatrix<T>& A, const std::vector<T>& B, int k, int tile, bool balanced, int iters,
                    int warmup, std::vector<T>& Y) {
  if (k < 0 || B.size() < static_cast<size_t>(A.n) * static_cast<size_t>(k))
    throw std::runtime_error("spmm_csr_tiled: B holds " + std::to_string(B.size()) + " values, n*k = " +
                             std::to_string(static_cast<size_t>(A.n) * static_cast<size_t>(k < 0 ? 0 : k)));
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  spmvb_context ctx = nullptr;
  check(spmvb_context_create(dev, &ctx), "spmvb_context_create");
  spmvb_matrix mat = nullptr;
  check(spmvb_matrix_create_csr(ctx, dtype_of<T>(), A.m, A.n, A.nnz, A.rowptr.data(), A.colind.data(),
                                A.values.data(), &mat),
        "spmvb_matrix_create_csr");
  if (balanced) check(spmvb_matrix_prepare(mat, static_cast<spmvb_kernel>(-1), 0), "prepare buckets");
  const size_t xb = static_cast<size_t>(A.n) * k * sizeof(T), yb = static_cast<size_t>(A.m) * k * sizeof(T);
  void *dB = nullptr, *dY = nullptr;
  check_cuda(cudaMalloc(&dB, xb ? xb : 1), "cudaMalloc B");
  check_cuda(cudaMalloc(&dY, yb ? yb : 1), "cudaMalloc Y");
  if (xb) check_cuda(cudaMemcpy(dB, B.data(), xb, cudaMemcpyHostToDevice), "upload B");
  auto launch = [&] { check(spmvb_spmm(mat, tile, balanced ? 1 : 0, k, dB, dY, dtype_of<T>(), nullptr), "spmvb_spmm"); };
  for (int i = 0; i < warmup; ++i) launch();
  check_cuda(cudaDeviceSynchronize(), "warmup");
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  std::vector<double> samples, xfer;
  for (int i = 0; i < iters; ++i) {
    cudaEventRecord(a);
    launch();
    cudaEventRecord(b);
    cudaEventSynchronize(b);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, a, b);
    samples.push_back(ms);
  }
  Y.assign(static_cast<size_t>(A.m) * k, T(0));
  for (int i = 0; i < 10; ++i) {
    cudaEventRecord(a);
    if (xb) cudaMemcpy(dB, B.data(), xb, cudaMemcpyHostToDevice);
    if (yb) cudaMemcpy(Y.data(), dY, yb, cudaMemcpyDeviceToHost);
    cudaEventRecord(b);
    cudaEventSynchronize(b);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, a, b);
    xfer.push_back(ms);
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  cudaFree(dB);
  cudaFree(dY);
  spmvb_matrix_destroy(mat);
  spmvb_context_destroy(ctx);
  const TimingSummary st = summarize(samples);
  SpmmResult r;
  r.iters = st.iters;
  r.mean_ms = st.mean_ms;
  r.min_ms = st.min_ms;
  r.median_ms = st.median_ms;
  r.max_ms = st.max_ms;
  r.transfer_ms = summarize(xfer).median_ms;
  r.kernel = "spmm_csr_tiled";
  return r;
}
}  // namespace detail

inline SpmmResult spmm_csr_tiled_f32(const CsrMatrix<float>& A, const std::vector<float>& B, int k, int tile,
                                     bool balanced, int iters, int warmup, std::vector<float>& Y) {
  return detail::run_spmm<float>(A, B, k, tile, balanced, iters, warmup, Y);
}
inline SpmmResult spmm_csr_tiled_f64(const CsrMatrix<double>& A, const std::vector<double>& B, int k, int tile,
                                     bool balanced, int iters, int warmup, std::vector<double>& Y) {
  return detail::run_spmm<double>(A, B, k, tile, balanced, iters, warmup, Y);
}

}  // namespace spmvbench

#ifndef SPMVB_NO_CUSPARSE
namespace spmvbench {
// The reference bench's cuSPARSE SpMM baseline (spmm_cuda.cuh:42-49 of
// SpMVBench): a comparison row, not a library kernel.
inline SpmmResult cusparse_spmm_f32(const CsrMatrix<float>& A, const std::vector<float>& B, int k, int iters,
                                    int warmup, std::vector<float>& Y) {
  return vendor::spmm<SpmmResult>(A, B, k, Y, iters, warmup);
}
inline SpmmResult cusparse_spmm_f64(const CsrMatrix<double>& A, const std::vector<double>& B, int k, int iters,
                                    int warmup, std::vector<double>& Y) {
  return vendor::spmm<SpmmResult>(A, B, k, Y, iters, warmup);
}
}  // namespace spmvbench
#endif  // SPMVB_NO_CUSPARSE

#endif  // SPMVBENCH_ENABLE_CUDA
