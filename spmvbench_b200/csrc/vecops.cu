// Vector kernels of the iterated solver loop (spmvb_dist_power_iterate):
// the 2-norm of the global vector held in a rank's padded x, and the scaling
// of x by 1 / norm.
//
// The norm is reproducible: block b of a fixed grid (a function of the
// global length m alone) sums the squares of global entries b*256 + t,
// b*256 + t + G*256, ... in a fixed shuffle tree, reading each from its slot
// of the padded layout, and one block adds the G partials in a fixed tree.
// Every rank that holds the same vector gets the same bits, for any number of
// ranks. Squares are summed in double for both value types.
#include <cmath>

#include "internal.hpp"

namespace spmvb {
namespace {

constexpr int kNormThreads = 256;
constexpr int kNormMaxBlocks = 1024;

__device__ __forceinline__ double block_sum(double v, double* sh) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sh[w] = v;
  __syncthreads();
  v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0;
  if (w == 0) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  }
  return v;  // valid in thread 0
}

// Slot of global entry i in the padded layout owner * max_rows + (i -
// bounds[owner]) (bounds has nranks + 1 entries; one rank: slot i).
__device__ __forceinline__ int64_t slot_of(int64_t i, const int* __restrict__ bounds, int nranks, int max_rows) {
  int lo = 0, hi = nranks;  // owner = last r with bounds[r] <= i
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (bounds[mid] <= i) lo = mid; else hi = mid;
  }
  return static_cast<int64_t>(lo) * max_rows + (i - bounds[lo]);
}

template <typename T>
__global__ void __launch_bounds__(kNormThreads) sumsq_partials(const T* __restrict__ x, int64_t m,
                                                               const int* __restrict__ bounds, int nranks,
                                                               int max_rows, double* __restrict__ partial) {
  __shared__ double sh[32];
  double s = 0.0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kNormThreads + threadIdx.x; i < m;
       i += static_cast<int64_t>(gridDim.x) * kNormThreads) {
    const double v = static_cast<double>(x[slot_of(i, bounds, nranks, max_rows)]);
    s = __dadd_rn(s, __dmul_rn(v, v));
  }
  s = block_sum(s, sh);
  if (threadIdx.x == 0) partial[blockIdx.x] = s;
}

__global__ void __launch_bounds__(kNormMaxBlocks) norm_final(const double* __restrict__ partial, int blocks,
                                                             double* __restrict__ norm) {
  __shared__ double sh[32];
  double v = threadIdx.x < blocks ? partial[threadIdx.x] : 0.0;
  v = block_sum(v, sh);
  if (threadIdx.x == 0) *norm = sqrt(v);
}

template <typename T>
__global__ void scale_by_inverse(T* __restrict__ x, int64_t n, const double* __restrict__ norm) {
  const double nv = *norm;
  const T inv = static_cast<T>(nv > 0.0 ? 1.0 / nv : 1.0);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    x[i] = x[i] * inv;
}

}  // namespace

int norm_blocks(int64_t n) {
  const int64_t b = (n + kNormThreads * 8 - 1) / (kNormThreads * 8);
  return static_cast<int>(b < 1 ? 1 : (b > kNormMaxBlocks ? kNormMaxBlocks : b));
}

spmvb_status launch_norm_and_scale(spmvb_dtype dtype, void* x, int64_t m, const int* bounds, int nranks,
                                   int max_rows, double* partials, double* norm, int sm_count, cudaStream_t s) {
  const int g = norm_blocks(m);
  const int64_t slots = static_cast<int64_t>(nranks) * max_rows;
  const int sg = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((slots + 255) / 256, int64_t(sm_count) * 8)));
  if (dtype == SPMVB_F64) {
    sumsq_partials<double><<<g, kNormThreads, 0, s>>>(static_cast<const double*>(x), m, bounds, nranks, max_rows,
                                                      partials);
    norm_final<<<1, kNormMaxBlocks, 0, s>>>(partials, g, norm);
    scale_by_inverse<double><<<sg, 256, 0, s>>>(static_cast<double*>(x), slots, norm);
  } else {
    sumsq_partials<float><<<g, kNormThreads, 0, s>>>(static_cast<const float*>(x), m, bounds, nranks, max_rows,
                                                     partials);
    norm_final<<<1, kNormMaxBlocks, 0, s>>>(partials, g, norm);
    scale_by_inverse<float><<<sg, 256, 0, s>>>(static_cast<float*>(x), slots, norm);
  }
  count_launch(3);
  SPMVB_TRY_CUDA(cudaGetLastError());
  return SPMVB_OK;
}

}  // namespace spmvb
