// ELL SpMV with the matrix stream on the TMA engine: ell_tma.
//
// On B200 the uniform-random ELL product is bound by the rate at which each
// SM sends random x gathers to L2, and the column-index / value stream of
// ell_rows goes through the same load path (L1TEX) as those gathers. Here
// every warp owns chunks of 32 consecutive rows and keeps a private ring of
// STAGES shared-memory slots: lane 0 asks the TMA engine for the chunk's
// W x 32 column indices and values (two 2-D tiled bulk copies of the
// column-major ELL, one tensor map each, completion counted on the slot's
// mbarrier), so the load path carries only the x gathers. The lanes wait on
// the slot's barrier (bounded), read their row's entries from shared memory,
// issue all of the row's x gathers, then add the products left to right from
// zero - csr_omp's order, so y is bit-identical to it - and lane 0 refills the
// slot with the warp's chunk STAGES turns ahead. No barrier spans more than
// one warp. Chunks are dealt to warps round-robin by a persistent grid.
//
// Requirements (checked by the launcher, otherwise ell_rows runs): width <=
// WMAX, m a multiple of 4 (the tensor maps' row stride m * 4 bytes must be a
// multiple of 16); chunk starts are multiples of 32 rows, so every copy's
// innermost coordinate is 16-byte aligned. The last chunk may reach past m:
// the copy fills those rows with zeros and they are not stored.
#pragma once

#include <cuda.h>

#include <cstdint>

#include "common.cuh"
#include "views.hpp"

namespace spmvb {

constexpr int kEllTmaWarps = 4;

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* tm, int x, int y, uint32_t bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <typename T, int WMAX>
struct EllTmaStage {
  static constexpr int kColBytes = WMAX * 32 * 4;
  static constexpr int kBytes = kColBytes + WMAX * 32 * static_cast<int>(sizeof(T));
};

template <typename T, typename Acc, int WMAX, int STAGES>
__global__ void __launch_bounds__(kEllTmaWarps * 32)
    ell_tma(const __grid_constant__ CUtensorMap tm_col, const __grid_constant__ CUtensorMap tm_val, EllView E,
            const T* __restrict__ x, Acc* __restrict__ y, int* __restrict__ err) {
  using Stage = EllTmaStage<T, WMAX>;
  extern __shared__ __align__(128) unsigned char ring_raw[];
  __shared__ __align__(8) unsigned long long bars[kEllTmaWarps][STAGES];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  // Copy destinations on 128-byte boundaries (the launch adds 128 bytes).
  unsigned char* ring_all = ring_raw + ((128u - (smem_addr(ring_raw) & 127u)) & 127u);
  unsigned char* ring = ring_all + static_cast<size_t>(wib) * STAGES * Stage::kBytes;
  const int W = E.width;
  const uint32_t tx = static_cast<uint32_t>(32 * W) * (4 + sizeof(T));
  const int64_t chunks = (static_cast<int64_t>(E.m) + 31) / 32;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kEllTmaWarps + wib;
  const int64_t step = static_cast<int64_t>(gridDim.x) * kEllTmaWarps;
  const uint64_t ps = policy_evict_first();
  const uint64_t pk = policy_evict_last();

  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(smem_addr(&bars[wib][s]), 1);
    mbar_fence_init();
  }
  __syncwarp();
  auto issue = [&](int s, int64_t c) {
    const uint32_t bar = smem_addr(&bars[wib][s]);
    const uint32_t dst = smem_addr(ring + static_cast<size_t>(s) * Stage::kBytes);
    mbar_expect_tx(bar, tx);
    tma_load_2d(dst, &tm_col, static_cast<int>(c * 32), 0, bar, ps);
    tma_load_2d(dst + Stage::kColBytes, &tm_val, static_cast<int>(c * 32), 0, bar, ps);
  };
  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      const int64_t c = c0 + s * step;
      if (c < chunks) issue(s, c);
    }
  }
  int k = 0;  // this warp's chunk counter
  for (int64_t c = c0; c < chunks; c += step, ++k) {
    const int s = k % STAGES;
    const uint32_t parity = static_cast<uint32_t>(k / STAGES) & 1u;
    const int64_t row = c * 32 + lane;
    const int L = row < E.m ? E.row_lengths[row] : 0;
    const bool ok = mbar_wait(smem_addr(&bars[wib][s]), parity);
    if (!__all_sync(0xffffffffu, ok)) {
      // Gave up: record it, then let the copies this warp still has in
      // flight land (bounded) before the CTA's shared memory goes away.
      if (lane == 0) {
        atomicExch(err, 3);
        for (int q = 0; q < STAGES; ++q) {
          const int64_t cq = c + q * step;
          if (cq >= chunks) break;
          const int kq = k + q;
          mbar_wait(smem_addr(&bars[wib][kq % STAGES]), static_cast<uint32_t>(kq / STAGES) & 1u);
        }
      }
      __syncwarp();
      return;
    }
    const unsigned char* slot = ring + static_cast<size_t>(s) * Stage::kBytes;
    const int* scol = reinterpret_cast<const int*>(slot);
    const T* sval = reinterpret_cast<const T*>(slot + Stage::kColBytes);
    T av[WMAX], xv[WMAX];
#pragma unroll
    for (int j = 0; j < WMAX; ++j) {
      if (j < L) {
        av[j] = sval[j * 32 + lane];
        xv[j] = ld_keep(x + scol[j * 32 + lane], pk);
      }
    }
    Acc sum = Acc(0);
#pragma unroll
    for (int j = 0; j < WMAX; ++j)
      if (j < L) sum = add_rn(sum, prod<Acc>(av[j], xv[j]));
    if (row < E.m) y[row] = sum;
    // Every lane's shared-memory reads are done (their values were used)
    // before lane 0 lets the copy engine overwrite the slot.
    __syncwarp();
    if (lane == 0) {
      const int64_t cn = c + STAGES * step;
      if (cn < chunks) {
        fence_proxy_async_smem();
        issue(s, cn);
      }
    }
  }
}

}  // namespace spmvb
