// SpMM Y (m x k) = A (m x n, CSR) * X (n x k), X and Y row-major.
//
// Reference: spmm_tiled_kernel / spmm_tiled_bucketed_kernel
// (src/cuda/spmm_cuda.cu:31-96): one warp per row, k tiled into TileK-wide
// shared-memory accumulators, one sparse entry per inner step.
//
// Here a group of G lanes owns one row and a tile of TILE = G*W columns; the
// accumulators live in registers (W per lane). The group loads G (col, val)
// pairs at once and broadcasts them with shuffles, then every lane gathers its
// W columns of X's row with one 16-byte load (VEC) and four entries are kept
// in flight per lane. Each output column is summed over the row's entries in
// CSR order from zero with separately rounded multiply and add, the order of
// spmm_csr_cpu (src/cpu/spmm_cpu.cpp:15-27), so Y is bit-identical to it.
// Rows longer than 64 entries in the bucketed variant are split across the 8
// warps of a CTA and combined in warp order (re-associated, deterministic).
#pragma once

#include <cstdint>

#include "common.cuh"
#include "views.hpp"

namespace spmvb {

template <typename T, int W>
struct XRow;
template <>
struct XRow<double, 2> {
  __device__ static void load(const double* p, uint64_t pol, double (&v)[2]) {
    const double2 a = ld_keep2(p, pol);
    v[0] = a.x; v[1] = a.y;
  }
};
template <>
struct XRow<float, 4> {
  __device__ static void load(const float* p, uint64_t pol, float (&v)[4]) {
    const float4 a = ld_keep4(p, pol);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  }
};

// Columns covered by lane `gl` in a pass starting at t0: VEC -> W consecutive
// columns at t0 + gl*W; scalar -> columns t0 + gl + w*G.
template <int G, int W, bool VEC>
__device__ __forceinline__ int lane_col(int t0, int gl, int w) {
  return VEC ? t0 + gl * W + w : t0 + gl + w * G;
}

template <typename T, int W, int G, bool VEC>
__device__ __forceinline__ void gather_xrow(const T* __restrict__ X, int64_t c,
                                            int k, int t0, int gl, uint64_t pk,
                                            T (&xv)[W]) {
  const T* rowp = X + c * k;
  if constexpr (VEC) {
    const int c0 = t0 + gl * W;
    if (c0 + W <= k) {
      XRow<T, W>::load(rowp + c0, pk, xv);
    } else {
#pragma unroll
      for (int w = 0; w < W; ++w) xv[w] = (c0 + w < k) ? ld_keep(rowp + c0 + w, pk) : T(0);
    }
  } else {
#pragma unroll
    for (int w = 0; w < W; ++w) {
      const int col = t0 + gl + w * G;
      xv[w] = (col < k) ? ld_keep(rowp + col, pk) : T(0);
    }
  }
}

template <typename T, typename Acc, int G, int W, bool VEC>
__global__ void __launch_bounds__(256)
    spmm_rows(CsrView A, const int* __restrict__ rows, int nrows,
              const T* __restrict__ X, Acc* __restrict__ Y, int k) {
  constexpr int TILE = G * W;
  constexpr int RPW = kWarp / G;
  const T* __restrict__ vals = static_cast<const T*>(A.values);
  const uint64_t ps = policy_evict_first();
  const uint64_t pk = policy_evict_last();
  const int lane = threadIdx.x & (kWarp - 1);
  const int gl = lane & (G - 1);
  const int grp = lane / G;
  const unsigned mask = (G == kWarp) ? 0xffffffffu : (((1u << G) - 1u) << (grp * G));
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / kWarp;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * blockDim.x / kWarp;
  for (int64_t r0 = warp * RPW; r0 < nrows; r0 += nwarps * RPW) {
    const int64_t slot = r0 + grp;
    const bool valid = slot < nrows;
    const int row = valid ? (rows ? rows[slot] : static_cast<int>(slot)) : 0;
    const int s = valid ? A.rowptr[row] : 0;
    const int e = valid ? A.rowptr[row + 1] : 0;
    for (int t0 = 0; t0 < k; t0 += TILE) {
      Acc acc[W];
#pragma unroll
      for (int w = 0; w < W; ++w) acc[w] = Acc(0);
      for (int p0 = s; p0 < e; p0 += G) {
        int my_c = 0;
        T my_a = T(0);
        if (p0 + gl < e) {
          my_c = ld_stream(A.colind + p0 + gl, ps);
          my_a = ld_stream(vals + p0 + gl, ps);
        }
        const int cnt = min(G, e - p0);
        int j = 0;
        for (; j + 4 <= cnt; j += 4) {
          int c[4];
          T a[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            c[u] = __shfl_sync(mask, my_c, j + u, G);
            a[u] = __shfl_sync(mask, my_a, j + u, G);
          }
          T xv[4][W];
#pragma unroll
          for (int u = 0; u < 4; ++u) gather_xrow<T, W, G, VEC>(X, c[u], k, t0, gl, pk, xv[u]);
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int w = 0; w < W; ++w) acc[w] = add_rn(acc[w], prod<Acc>(a[u], xv[u][w]));
        }
        for (; j < cnt; ++j) {
          const int c = __shfl_sync(mask, my_c, j, G);
          const T a = __shfl_sync(mask, my_a, j, G);
          T xv[W];
          gather_xrow<T, W, G, VEC>(X, c, k, t0, gl, pk, xv);
#pragma unroll
          for (int w = 0; w < W; ++w) acc[w] = add_rn(acc[w], prod<Acc>(a, xv[w]));
        }
      }
      if (valid) {
        Acc* yrow = Y + static_cast<int64_t>(row) * k;
#pragma unroll
        for (int w = 0; w < W; ++w) {
          const int col = lane_col<G, W, VEC>(t0, gl, w);
          if (col < k) st_stream(yrow + col, acc[w]);
        }
      }
    }
  }
}

// Column-band pass of the plain SpMM (spmm_bands in spmv_launch.cuh): the
// columns of A (rows of X) are cut into bands that fit the L2 and the whole
// product is swept band by band, so the X rows one pass gathers stay
// resident. Row i's entries of band b are [start, end) = split[b-1][i] ..
// split[b][i] (rowptr ends at b = 0 and b = B-1). Pass 0 starts each output
// from zero; later passes load the running values of Y and keep adding. The
// rows' columns are ascending, so every output element still receives its
// terms left to right in CSR order, as spmm_csr_cpu adds them: bit-identical.
// X is gathered with L2 evict-last, Y and A streamed with evict-first.
template <typename T, typename Acc, int G, int W, bool VEC>
__global__ void __launch_bounds__(256)
    spmm_band(CsrView A, const int* __restrict__ lo_split, const int* __restrict__ hi_split, bool first,
              const T* __restrict__ X, Acc* __restrict__ Y, int k) {
  constexpr int TILE = G * W;
  constexpr int RPW = kWarp / G;
  const T* __restrict__ vals = static_cast<const T*>(A.values);
  const uint64_t ps = policy_evict_first();
  const uint64_t pk = policy_evict_last();
  const int lane = threadIdx.x & (kWarp - 1);
  const int gl = lane & (G - 1);
  const int grp = lane / G;
  const unsigned mask = (G == kWarp) ? 0xffffffffu : (((1u << G) - 1u) << (grp * G));
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / kWarp;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * blockDim.x / kWarp;
  for (int64_t r0 = warp * RPW; r0 < A.m; r0 += nwarps * RPW) {
    const int64_t row = r0 + grp;
    const bool valid = row < A.m;
    const int s = valid ? (lo_split ? lo_split[row] : A.rowptr[row]) : 0;
    const int e = valid ? (hi_split ? hi_split[row] : A.rowptr[row + 1]) : 0;
    Acc* yrow = Y + row * k;
    for (int t0 = 0; t0 < k; t0 += TILE) {
      Acc acc[W];
#pragma unroll
      for (int w = 0; w < W; ++w) {
        const int col = lane_col<G, W, VEC>(t0, gl, w);
        acc[w] = (!first && valid && col < k) ? ld_stream(yrow + col, ps) : Acc(0);
      }
      for (int p0 = s; p0 < e; p0 += G) {
        int my_c = 0;
        T my_a = T(0);
        if (p0 + gl < e) {
          my_c = ld_stream(A.colind + p0 + gl, ps);
          my_a = ld_stream(vals + p0 + gl, ps);
        }
        const int cnt = min(G, e - p0);
        int j = 0;
        for (; j + 4 <= cnt; j += 4) {
          int c[4];
          T a[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            c[u] = __shfl_sync(mask, my_c, j + u, G);
            a[u] = __shfl_sync(mask, my_a, j + u, G);
          }
          T xv[4][W];
#pragma unroll
          for (int u = 0; u < 4; ++u) gather_xrow<T, W, G, VEC>(X, c[u], k, t0, gl, pk, xv[u]);
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int w = 0; w < W; ++w) acc[w] = add_rn(acc[w], prod<Acc>(a[u], xv[u][w]));
        }
        for (; j < cnt; ++j) {
          const int c = __shfl_sync(mask, my_c, j, G);
          const T a = __shfl_sync(mask, my_a, j, G);
          T xv[W];
          gather_xrow<T, W, G, VEC>(X, c, k, t0, gl, pk, xv);
#pragma unroll
          for (int w = 0; w < W; ++w) acc[w] = add_rn(acc[w], prod<Acc>(a, xv[w]));
        }
      }
      if (valid) {
#pragma unroll
        for (int w = 0; w < W; ++w) {
          const int col = lane_col<G, W, VEC>(t0, gl, w);
          if (col < k) st_stream(yrow + col, acc[w]);
        }
      }
    }
  }
}

// Band boundaries of every row: split[(b - 1) * m + i] = the first entry of
// row i with column >= b * band_cols (b = 1 .. bands-1), by binary search
// over the row's ascending columns.
__global__ void spmm_band_splits(CsrView A, int bands, int band_cols, int* __restrict__ split);

// Long rows (bucketed variant): one CTA of 8 warps per row; warp w takes the
// w-th contiguous eighth of the row's entries, partial tiles meet in shared
// memory and are added in warp order.
template <typename T, typename Acc, int W, bool VEC>
__global__ void __launch_bounds__(256)
    spmm_long_rows(CsrView A, const int* __restrict__ rows, int nrows,
                   const T* __restrict__ X, Acc* __restrict__ Y, int k) {
  constexpr int G = kWarp;
  constexpr int TILE = G * W;
  constexpr int NW = 8;
  __shared__ Acc s_part[NW][TILE];
  const T* __restrict__ vals = static_cast<const T*>(A.values);
  const uint64_t ps = policy_evict_first();
  const uint64_t pk = policy_evict_last();
  const int lane = threadIdx.x & (kWarp - 1);
  const int wid = threadIdx.x / kWarp;
  for (int slot = blockIdx.x; slot < nrows; slot += gridDim.x) {
    const int row = rows[slot];
    const int s = A.rowptr[row];
    const int e = A.rowptr[row + 1];
    const int len = e - s;
    const int chunk = (len + NW - 1) / NW;
    const int ws = s + min(len, wid * chunk);
    const int we = s + min(len, (wid + 1) * chunk);
    for (int t0 = 0; t0 < k; t0 += TILE) {
      Acc acc[W];
#pragma unroll
      for (int w = 0; w < W; ++w) acc[w] = Acc(0);
      for (int p0 = ws; p0 < we; p0 += G) {
        int my_c = 0;
        T my_a = T(0);
        if (p0 + lane < we) {
          my_c = ld_stream(A.colind + p0 + lane, ps);
          my_a = ld_stream(vals + p0 + lane, ps);
        }
        const int cnt = min(G, we - p0);
        for (int j = 0; j < cnt; ++j) {
          const int c = __shfl_sync(0xffffffffu, my_c, j);
          const T a = __shfl_sync(0xffffffffu, my_a, j);
          T xv[W];
          gather_xrow<T, W, G, VEC>(X, c, k, t0, lane, pk, xv);
#pragma unroll
          for (int w = 0; w < W; ++w) acc[w] = add_rn(acc[w], prod<Acc>(a, xv[w]));
        }
      }
#pragma unroll
      for (int w = 0; w < W; ++w) {
        const int idx = VEC ? lane * W + w : lane + w * G;
        s_part[wid][idx] = acc[w];
      }
      __syncthreads();
      for (int idx = threadIdx.x; idx < TILE; idx += blockDim.x) {
        const int col = t0 + idx;
        if (col < k) {
          Acc tot = s_part[0][idx];
          for (int w = 1; w < NW; ++w) tot = add_rn(tot, s_part[w][idx]);
          Y[static_cast<int64_t>(row) * k + col] = tot;
        }
      }
      __syncthreads();
    }
  }
}

}  // namespace spmvb
