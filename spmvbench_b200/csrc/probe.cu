// Random-gather ceiling of a device: the rate at which SMs can fetch 8-byte
// elements at random positions of an L2-resident vector. SpMV on matrices
// whose column indices have no locality is bounded by this rate rather than
// by HBM bandwidth (each gather moves a whole 32-byte L2 sector for 8 useful
// bytes), so bench.py reports a second roofline against it.
#include <algorithm>

#include "common.cuh"
#include "internal.hpp"

namespace spmvb {

__device__ __forceinline__ uint32_t mix32(uint32_t v) {
  v ^= v >> 16;
  v *= 0x7feb352du;
  v ^= v >> 15;
  v *= 0x846ca68bu;
  v ^= v >> 16;
  return v;
}

// Thread r gathers 16 pseudo-random elements of x (indices from a hash, so
// no index stream competes with the gathers) and writes their sum.
__global__ void __launch_bounds__(256) gather_probe(const double* __restrict__ x, double* __restrict__ y,
                                                    int64_t threads, uint32_t n) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= threads) return;
  const uint64_t pk = policy_evict_last();
  double v[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = ld_keep(x + mix32(static_cast<uint32_t>(r * 16 + j)) % n, pk);
  double s = 0.0;
#pragma unroll
  for (int j = 0; j < 16; ++j) s += v[j];
  y[r] = s;
}

}  // namespace spmvb

using namespace spmvb;

extern "C" spmvb_status spmvb_probe_gather_rate(spmvb_context ctx, int64_t n, int64_t gathers,
                                                double* gathers_per_s) {
  clear_error();
  if (!ctx || !gathers_per_s) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null argument");
  if (n < 1 || n > INT32_MAX || gathers < 16) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bad n or gathers");
  DeviceGuard g(ctx->device);
  const int64_t threads = gathers / 16;
  DevBuf x, y;
  SPMVB_TRY(x.alloc(static_cast<size_t>(n) * 8));
  SPMVB_TRY(y.alloc(static_cast<size_t>(threads) * 8));
  cudaEvent_t a, b;
  SPMVB_TRY_CUDA(cudaEventCreate(&a));
  SPMVB_TRY_CUDA(cudaEventCreate(&b));
  const int grid = static_cast<int>((threads + 255) / 256);
  float best = 1e30f;
  for (int rep = 0; rep < 8; ++rep) {
    cudaEventRecord(a);
    gather_probe<<<grid, 256>>>(x.as<double>(), y.as<double>(), threads, static_cast<uint32_t>(n));
    cudaEventRecord(b);
    cudaEventSynchronize(b);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, a, b);
    if (rep >= 2) best = std::min(best, ms);  // first launches warm x into L2
  }
  count_launch(8);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  SPMVB_TRY_CUDA(cudaGetLastError());
  *gathers_per_s = static_cast<double>(threads * 16) / (best * 1e-3);
  return SPMVB_OK;
}
