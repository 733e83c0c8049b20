// SpMV kernels for sm_100a. Templated on the storage type T and the
// accumulator type Acc, like the reference kernels (src/cuda/spmv_cuda.cu).
//
// Kernel map (reference kernel -> this file):
//   csr_scalar_kernel (spmv_cuda.cu:43-54)   -> csr_scalar_warp
//   csr_vector_kernel (spmv_cuda.cu:56-80)   -> csr_vector<G>
//   csr_warp_kernel   (spmv_cuda.cu:83-97)   -> csr_vector<32>
//   csr_merge_kernel  (spmv_cuda.cu:100-125) -> csr_merge + merge_fixup (a real
//                                              merge-path, not a row queue)
//   ell_kernel        (spmv_cuda.cu:128-142) -> ell_rows
//   bcsr_kernel       (spmv_cuda.cu:145-170) -> bcsr_rows
//   (new) hybrid ELL(K)+CSR                 -> hyb_rows
//
// Summation order. csr_scalar_warp, ell_rows and hyb's ELL part add each
// row's terms left to right from zero with separately rounded multiply and
// add, exactly as csr_omp does (src/cpu/spmv_cpu.cpp:19-25), so their output
// is bit-identical to it. bcsr_rows follows spmv_bcsr_cpu's order
// (src/cpu/spmv_cpu.cpp:85-97: per-block partial, then added), so it is
// bit-identical to that kernel. The vector/warp/merge/long-row kernels
// re-associate the sum and are bounded by 2*gamma_n*sum|a_ij x_j|
// (tests/test_cuda_correctness.cpp:1-11 of the reference).
#pragma once

#include <climits>
#include <cstdint>

#include "common.cuh"
#include "views.hpp"

namespace spmvb {

// Shared-memory slot of staged product q. One pad word per 16 doubles (per 32
// floats) keeps thread-per-row reads of 16-entry rows conflict free.
template <typename Acc>
__device__ __forceinline__ int swz(int q) {
  return sizeof(Acc) == 8 ? q + (q >> 4) : q + (q >> 5);
}
template <typename Acc>
constexpr int swz_size(int cap) {
  return sizeof(Acc) == 8 ? cap + cap / 16 + 1 : cap + cap / 32 + 1;
}

// Load 4 consecutive values starting at a 4-aligned index.
__device__ __forceinline__ void ld_stream_quad(const double* p, uint64_t pol,
                                               double (&v)[4]) {
  const double2 a = ld_stream2(p, pol);
  const double2 b = ld_stream2(p + 2, pol);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
__device__ __forceinline__ void ld_stream_quad(const float* p, uint64_t pol,
                                               float (&v)[4]) {
  const float4 a = ld_stream4(p, pol);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}

// Products Acc(values[p]) * Acc(x[colind[p]]) for p in [c0, c1), c0 a
// multiple of 4, written to s_prod[swz(p - c0)]. Threads take groups of 4
// consecutive entries, so a warp reads 512 contiguous bytes of colind with
// one 16-byte load per lane. Entries up to the next multiple of 4 past c1
// are computed too (the arrays carry kPad padding); callers ignore them.
// GROUPS = groups of 4 per thread per pass, all loads of a pass are issued
// before any product is formed.
template <typename T, typename Acc, int NT, int GROUPS>
__device__ __forceinline__ void stage_products(
    const int* __restrict__ colind, const T* __restrict__ vals,
    const T* __restrict__ x, int64_t c0, int64_t c1, Acc* s_prod,
    uint64_t pol_stream, uint64_t pol_keep) {
  const int span = static_cast<int>(c1 - c0);
  for (int base = 0; base < span; base += NT * 4 * GROUPS) {
    int4 c[GROUPS];
    bool ok[GROUPS];
#pragma unroll
    for (int g = 0; g < GROUPS; ++g) {
      const int q = base + (g * NT + static_cast<int>(threadIdx.x)) * 4;
      ok[g] = q < span;
      c[g] = ok[g] ? ld_stream4(colind + c0 + q, pol_stream)
                   : make_int4(0, 0, 0, 0);
    }
    // Values do not depend on the column indices: issue them before the
    // x gathers so they are in flight while colind returns.
    T av[GROUPS][4];
#pragma unroll
    for (int g = 0; g < GROUPS; ++g) {
      const int q = base + (g * NT + static_cast<int>(threadIdx.x)) * 4;
      if (ok[g]) ld_stream_quad(vals + c0 + q, pol_stream, av[g]);
    }
    T xv[GROUPS][4];
#pragma unroll
    for (int g = 0; g < GROUPS; ++g) {
      if (ok[g]) {
        xv[g][0] = ld_keep(x + c[g].x, pol_keep);
        xv[g][1] = ld_keep(x + c[g].y, pol_keep);
        xv[g][2] = ld_keep(x + c[g].z, pol_keep);
        xv[g][3] = ld_keep(x + c[g].w, pol_keep);
      }
    }
#pragma unroll
    for (int g = 0; g < GROUPS; ++g) {
      const int q = base + (g * NT + static_cast<int>(threadIdx.x)) * 4;
      if (ok[g]) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          s_prod[swz<Acc>(q + i)] = prod<Acc>(av[g][i], xv[g][i]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// CSR scalar, warp-staged: the kernel behind SPMVB_CSR_SCALAR.
//
// On B200 the random x gathers, not the matrix stream, bound short-row SpMV:
// 16M random 8-byte gathers from an L2-resident x take ~62 us on their own.
// What matters is how many independent gathers each SM keeps in flight, so
// this kernel has no CTA-wide barrier at all. Each warp owns 32 consecutive
// rows; their entries are one contiguous range of the CSR arrays, which the
// warp reads in chunks of CH entries with 16-byte vector loads (lane l takes
// entries 4l..4l+3 of every 128-entry block, so each load instruction covers
// 512 contiguous bytes), issuing every gather of the chunk before forming any
// product. Products go to the warp's own slice of shared memory; after a
// __syncwarp each lane adds its row's products in order, carrying the running
// sum across chunks, so every row is summed left to right from zero exactly
// as csr_omp sums it. Rows of any length work (long rows simply span chunks).
// ---------------------------------------------------------------------------
template <typename T, typename Acc, int CH>
__global__ void __launch_bounds__(256)
    csr_scalar_warp(CsrView A, const T* __restrict__ x, Acc* __restrict__ y) {
  constexpr int WARPS = 8;
  constexpr int GROUPS = CH / (kWarp * 4);  // groups of 4 entries per lane per chunk
  static_assert(CH % (kWarp * 4) == 0, "CH must be a multiple of 128");
  constexpr int SLOT = swz_size<Acc>(CH);
  __shared__ Acc s_prod_all[WARPS * SLOT];
  const int lane = threadIdx.x & (kWarp - 1);
  const int wib = threadIdx.x / kWarp;
  Acc* s_prod = s_prod_all + wib * SLOT;
  const T* __restrict__ vals = static_cast<const T*>(A.values);
  const uint64_t ps = policy_evict_first();
  const uint64_t pk = policy_evict_last();
  const int64_t warp = static_cast<int64_t>(blockIdx.x) * WARPS + wib;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * WARPS;
  for (int64_t r0 = warp * kWarp; r0 < A.m; r0 += nwarps * kWarp) {
    const int64_t row = r0 + lane;
    const bool live = row < A.m;
    const int64_t last = (A.m - r0 < kWarp) ? A.m - r0 - 1 : kWarp - 1;
    int64_t rs = 0, re = 0;
    if (live) {
      rs = A.rowptr[row];
      re = A.rowptr[row + 1];
    }
    const int64_t P0 = __shfl_sync(0xffffffffu, rs, 0);
    const int64_t P1 = __shfl_sync(0xffffffffu, re, static_cast<int>(last));
    Acc sum = Acc(0);
    for (int64_t c0 = P0 & ~int64_t(3); c0 < P1; c0 += CH) {
      const int span = static_cast<int>((P1 - c0) < CH ? (P1 - c0) : CH);
      int4 c[GROUPS];
      T av[GROUPS][4];
      T xv[GROUPS][4];
#pragma unroll
      for (int g = 0; g < GROUPS; ++g) {
        const int q = (g * kWarp + lane) * 4;
        c[g] = q < span ? ld_stream4(A.colind + c0 + q, ps) : make_int4(0, 0, 0, 0);
      }
#pragma unroll
      for (int g = 0; g < GROUPS; ++g) {
        const int q = (g * kWarp + lane) * 4;
        if (q < span) ld_stream_quad(vals + c0 + q, ps, av[g]);
      }
#pragma unroll
      for (int g = 0; g < GROUPS; ++g) {
        const int q = (g * kWarp + lane) * 4;
        if (q < span) {
          xv[g][0] = ld_keep(x + c[g].x, pk);
          xv[g][1] = ld_keep(x + c[g].y, pk);
          xv[g][2] = ld_keep(x + c[g].z, pk);
          xv[g][3] = ld_keep(x + c[g].w, pk);
        }
      }
#pragma unroll
      for (int g = 0; g < GROUPS; ++g) {
        const int q = (g * kWarp + lane) * 4;
        if (q < span) {
#pragma unroll
          for (int i = 0; i < 4; ++i) s_prod[swz<Acc>(q + i)] = prod<Acc>(av[g][i], xv[g][i]);
        }
      }
      __syncwarp();
      if (live) {
        const int64_t c1 = c0 + span;
        const int a = static_cast<int>((rs > c0 ? rs : c0) - c0);
        const int b = static_cast<int>((re < c1 ? re : c1) - c0);
        for (int q = a; q < b; ++q) sum = add_rn(sum, s_prod[swz<Acc>(q)]);
      }
      __syncwarp();
    }
    if (live) y[row] = sum;
  }
}

// ---------------------------------------------------------------------------
// CSR vector: G lanes per row (G = 2..32; G = 32 is the warp kernel). Lanes
// of a group read the row with 16-byte vector loads (2 doubles / 4 floats
// and the matching column indices) after a scalar head that reaches vector
// alignment, then reduce with a butterfly. Trip counts are warp-uniform so
// the full-mask shuffles are always legal.
// ---------------------------------------------------------------------------
template <typename T, typename Acc, int G>
__global__ void __launch_bounds__(256)
    csr_vector(CsrView A, const T* __restrict__ x, Acc* __restrict__ y) {
  constexpr int V = 16 / sizeof(T);  // elements per vector load
  constexpr int RPW = kWarp / G;     // rows per warp per iteration
  const T* __restrict__ vals = static_cast<const T*>(A.values);
  const uint64_t ps = policy_evict_first();
  const uint64_t pk = policy_evict_last();
  const int lane = threadIdx.x & (kWarp - 1);
  const int gl = lane & (G - 1);
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / kWarp;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * blockDim.x / kWarp;
  for (int64_t r0 = warp * RPW; r0 < A.m; r0 += nwarps * RPW) {
    const int64_t row = r0 + lane / G;
    Acc sum = Acc(0);
    if (row < A.m) {
      const int s = A.rowptr[row];
      const int e = A.rowptr[row + 1];
      const int head_end = min(e, (s + V - 1) & ~(V - 1));
      // head (up to V-1 entries) and tail are strided by G: G may be < V-1
      for (int p = s + gl; p < head_end; p += G)
        sum = add_rn(sum, prod<Acc>(ld_stream(vals + p, ps), ld_keep(x + ld_stream(A.colind + p, ps), pk)));
      const int nvec = (e - head_end) / V;  // full vectors after the head
      const int body_end = head_end + nvec * V;
#pragma unroll 2
      for (int q = head_end + gl * V; q < body_end; q += G * V) {
        if constexpr (V == 2) {
          const int2 c = ld_stream2(A.colind + q, ps);
          const double2 a = ld_stream2(reinterpret_cast<const double*>(vals) + q, ps);
          const T x0 = ld_keep(x + c.x, pk);
          const T x1 = ld_keep(x + c.y, pk);
          sum = add_rn(sum, prod<Acc>(static_cast<T>(a.x), x0));
          sum = add_rn(sum, prod<Acc>(static_cast<T>(a.y), x1));
        } else {
          const int4 c = ld_stream4(A.colind + q, ps);
          const float4 a = ld_stream4(reinterpret_cast<const float*>(vals) + q, ps);
          const T x0 = ld_keep(x + c.x, pk);
          const T x1 = ld_keep(x + c.y, pk);
          const T x2 = ld_keep(x + c.z, pk);
          const T x3 = ld_keep(x + c.w, pk);
          sum = add_rn(sum, prod<Acc>(static_cast<T>(a.x), x0));
          sum = add_rn(sum, prod<Acc>(static_cast<T>(a.y), x1));
          sum = add_rn(sum, prod<Acc>(static_cast<T>(a.z), x2));
          sum = add_rn(sum, prod<Acc>(static_cast<T>(a.w), x3));
        }
      }
      for (int p = body_end + gl; p < e; p += G)
        sum = add_rn(sum, prod<Acc>(ld_stream(vals + p, ps), ld_keep(x + ld_stream(A.colind + p, ps), pk)));
    }
    sum = group_sum<G>(sum);
    if (row < A.m && gl == 0) y[row] = sum;
  }
}

// ---------------------------------------------------------------------------
// CSR merge-path (Merrill & Garland, "Merge-based parallel sparse
// matrix-vector multiplication", SC'16): the merge of the m row-end offsets
// with the nnz entry indices is cut into tiles of NT*IPT consecutive items,
// so every thread gets IPT items whatever the row lengths. A CTA stages its
// tile's row ends and products in shared memory with coalesced loads, then
// each thread walks its IPT items. Partial row sums that cross threads are
// combined in thread order; a partial that crosses into the next tile is
// written to the carry scratch and added by merge_fixup in tile order, so
// results are deterministic run to run.
// ---------------------------------------------------------------------------
template <int NT, int IPT>
struct MergeShape {
  static constexpr int kTile = NT * IPT;
};

template <typename T, typename Acc, int NT, int IPT>
__global__ void __launch_bounds__(NT)
    csr_merge(CsrView A, MergeView M, const T* __restrict__ x, Acc* __restrict__ y) {
  constexpr int TILE = NT * IPT;
  __shared__ int s_rowend[TILE + 1];
  __shared__ Acc s_prod[swz_size<Acc>(TILE + 8)];
  __shared__ int s_crow[NT];
  __shared__ Acc s_cval[NT];
  const T* __restrict__ vals = static_cast<const T*>(A.values);
  const uint64_t ps = policy_evict_first();
  const uint64_t pk = policy_evict_last();
  const int t = threadIdx.x;
  const int tile = blockIdx.x;
  const int64_t d0 = static_cast<int64_t>(tile) * TILE;
  const int64_t d1 = min(d0 + TILE, M.num_items);
  const int row0 = M.tile_row[tile];
  const int row1 = M.tile_row[tile + 1];
  const int64_t j0 = d0 - row0;
  const int64_t j1 = d1 - row1;
  const int nrows_local = row1 - row0;          // row ends inside the tile
  const int nnz_local = static_cast<int>(j1 - j0);

  for (int i = t; i <= nrows_local; i += NT) {
    const int r = row0 + i;
    s_rowend[i] = (r < A.m) ? A.rowptr[r + 1] : INT_MAX;
  }
  const int64_t pa = j0 & ~int64_t(3);
  stage_products<T, Acc, NT, 2>(A.colind, vals, x, pa, j1, s_prod, ps, pk);
  __syncthreads();

  // Merge-path search for this thread's start inside the tile.
  const int items = static_cast<int>(d1 - d0);
  const int k = min(t * IPT, items);
  int lo = max(0, k - nnz_local);
  int hi = min(k, nrows_local);
  while (lo < hi) {
    const int pivot = (lo + hi) >> 1;
    if (s_rowend[pivot] <= j0 + k - pivot - 1)
      lo = pivot + 1;
    else
      hi = pivot;
  }
  int row = row0 + lo;
  int64_t nz = j0 + k - lo;
  const int start_row = row;
  const int my_items = min(IPT, items - k);

  Acc sum = Acc(0);
  bool have = false;       // consumed an entry of `row` since it started
  int held_row = -1;       // first completed row, if it is the start row
  Acc held_val = Acc(0);
  for (int i = 0; i < my_items; ++i) {
    if (nz < s_rowend[row - row0]) {
      sum = add_rn(sum, s_prod[swz<Acc>(static_cast<int>(nz - pa))]);
      have = true;
      ++nz;
    } else {
      if (row == start_row && held_row < 0) {
        held_row = row;
        held_val = sum;
      } else {
        y[row] = sum;
      }
      sum = Acc(0);
      have = false;
      ++row;
    }
  }
  s_crow[t] = have ? row : -1;
  s_cval[t] = sum;
  __syncthreads();

  if (held_row >= 0) {
    int t0 = t;
    while (t0 > 0 && s_crow[t0 - 1] == held_row) --t0;
    if (t0 < t) {
      Acc c = s_cval[t0];
      for (int u = t0 + 1; u < t; ++u) c = add_rn(c, s_cval[u]);
      y[held_row] = add_rn(c, held_val);
    } else {
      y[held_row] = held_val;
    }
  }
  if (t == NT - 1) {
    const int r = s_crow[NT - 1];
    if (r >= 0) {
      int t0 = NT - 1;
      while (t0 > 0 && s_crow[t0 - 1] == r) --t0;
      Acc c = s_cval[t0];
      for (int u = t0 + 1; u < NT; ++u) c = add_rn(c, s_cval[u]);
      M.carry_row[tile] = r;
      static_cast<Acc*>(M.carry_val)[tile] = c;
    } else {
      M.carry_row[tile] = -1;
    }
  }
}

// Adds the carries of consecutive tiles that end inside the same row, in tile
// order, to the row's value written by the tile that completed it.
template <typename Acc>
__global__ void merge_fixup(MergeView M, Acc* __restrict__ y) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= M.num_tiles) return;
  const int r = M.carry_row[b];
  if (r < 0) return;
  if (b > 0 && M.carry_row[b - 1] == r) return;  // not the first of the run
  const Acc* cv = static_cast<const Acc*>(M.carry_val);
  Acc s = cv[b];
  for (int u = b + 1; u < M.num_tiles && M.carry_row[u] == r; ++u)
    s = add_rn(s, cv[u]);
  y[r] = add_rn(y[r], s);
}

// Tile start rows of the merge path: for diagonal d = t*tile_items, the
// number of row ends that precede it (binary search over rowptr).
__global__ void merge_partition(CsrView A, int64_t num_items, int tile_items,
                                int num_tiles, int* __restrict__ tile_row);

// ---------------------------------------------------------------------------
// ELL: one row per thread, column-major slots j*ld + row (coalesced across
// the warp), only the row's real entries are read (row_lengths), csr_omp
// order. SKIP_LONG: rows with row_lengths < 0 belong to the hybrid format's
// long-row kernel and are not written here.
// ---------------------------------------------------------------------------
// Sum of ELL row `row` (L real entries), left to right from zero.
template <typename T, typename Acc>
__device__ __forceinline__ Acc ell_row_sum(const EllView& E, int row, int L, const T* __restrict__ x,
                                           uint64_t ps, uint64_t pk) {
  const T* __restrict__ vals = static_cast<const T*>(E.values);
  Acc sum = Acc(0);
  int64_t p = row;
  int j = 0;
  for (; j + 4 <= L; j += 4) {
    int c[4];
    T a[4], xv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) c[u] = ld_stream(E.colind + p + u * E.ld, ps);
#pragma unroll
    for (int u = 0; u < 4; ++u) a[u] = ld_stream(vals + p + u * E.ld, ps);
#pragma unroll
    for (int u = 0; u < 4; ++u) xv[u] = ld_keep(x + c[u], pk);
#pragma unroll
    for (int u = 0; u < 4; ++u) sum = add_rn(sum, prod<Acc>(a[u], xv[u]));
    p += 4 * E.ld;
  }
  for (; j < L; ++j) {
    sum = add_rn(sum, prod<Acc>(ld_stream(vals + p, ps),
                                ld_keep(x + ld_stream(E.colind + p, ps), pk)));
    p += E.ld;
  }
  return sum;
}

template <typename T, typename Acc, bool SKIP_LONG>
__global__ void __launch_bounds__(256)
    ell_rows(EllView E, const T* __restrict__ x, Acc* __restrict__ y) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= E.m) return;
  const int L = E.row_lengths[row];
  if (SKIP_LONG && L < 0) return;
  y[row] = ell_row_sum<T, Acc>(E, row, L, x, policy_evict_first(), policy_evict_last());
}

// Hybrid ELL(K) + CSR, one launch (see HybView for the layout).
//
// ELL blocks: one thread per row with len <= K, csr_omp order (bit-identical).
//
// Chunk blocks, one warp per chunk of at most kHybChunk entries: lane l loads
// entries l, l+32, ... (coalesced) and every gather of the chunk is in flight
// before any product is formed.
//  - Packed chunk (whole rows): the products go to the warp's slice of shared
//    memory and lane l adds rows chunk_row[c]+l, +l+32, ... left to right from
//    zero, the csr_omp order, so these rows are bit-identical too. The lane's
//    first row's bounds and id are loaded with the chunk's entries.
//  - Segment of a row longer than kHybChunk: the warp reduces it in a fixed
//    order (lane partials over p = l + 32i, then a butterfly) into partial[c];
//    the warp whose partial completes the row (per-row counter) adds the
//    row's partials in chunk order (lane partials, butterfly) and writes y.
//    Deterministic, re-associated (bounded by 2*gamma_n*sum|a_ij x_j|).
//
// Remaining blocks: y = 0 for the empty rows when K = 0.
template <typename T, typename Acc, int NT>
__global__ void __launch_bounds__(NT)
    hyb_rows(HybView H, const T* __restrict__ x, Acc* __restrict__ y) {
  constexpr int W = NT / kWarp;
  constexpr int PER = kHybChunk / kWarp;
  __shared__ Acc s_prod[W][swz_size<Acc>(kHybChunk)];  // padded: conflict-free row sums
  const uint64_t ps = policy_evict_first();
  const uint64_t pk = policy_evict_last();
  if (static_cast<int>(blockIdx.x) < H.ell_blocks) {
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row < H.ell.m) {
      const int L = H.ell.row_lengths[row];
      if (L >= 0) y[row] = ell_row_sum<T, Acc>(H.ell, row, L, x, ps, pk);
    }
    return;
  }
  const int cb_index = static_cast<int>(blockIdx.x) - H.ell_blocks;
  if (cb_index >= H.chunk_blocks) {
    const int i = (cb_index - H.chunk_blocks) * blockDim.x + threadIdx.x;
    if (i < H.n_empty) y[H.empty_rows[i]] = Acc(0);
    return;
  }
  const int wib = threadIdx.x / kWarp;
  const int lane = threadIdx.x & (kWarp - 1);
  const int c = cb_index * W + wib;
  if (c >= H.n_chunks) return;
  const T* __restrict__ tv = static_cast<const T*>(H.tail_values);
  const int64_t e0 = H.chunk_start[c];
  const int span = static_cast<int>(H.chunk_start[c + 1] - e0);
  const int li0 = H.chunk_row[c];
  const int li_end = H.chunk_row[c + 1];  // packed: rows li0 .. li_end-1

  int col[PER];
  T val[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int q = lane + i * kWarp;
    col[i] = q < span ? ld_stream(H.tail_colind + e0 + q, ps) : 0;
    val[i] = q < span ? ld_stream(tv + e0 + q, ps) : T(0);
  }
  const int64_t rs0 = H.tail_ptr[li0];
  const int64_t re0 = H.tail_ptr[li0 + 1];
  // The lane's first row (packed chunks), loaded alongside the entries.
  const int my = li0 + lane;
  int64_t my_s = 0, my_e = 0;
  int my_row = 0;
  if (my < li_end) {
    my_s = H.tail_ptr[my];
    my_e = H.tail_ptr[my + 1];
    my_row = H.long_rows[my];
  }
  Acc pr[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i)
    pr[i] = (lane + i * kWarp < span) ? prod<Acc>(val[i], ld_keep(x + col[i], pk)) : Acc(0);

  if (re0 - rs0 > kHybChunk) {
    // Segment of a cut row.
    Acc v = Acc(0);
#pragma unroll
    for (int i = 0; i < PER; ++i) v = add_rn(v, pr[i]);  // entries past the span add exact zeros
    v = group_sum<kWarp>(v);
    Acc* part = static_cast<Acc*>(H.partial);
    const int si = H.chunk_split[c];
    const int first = H.split_first[si];
    const int pieces = static_cast<int>((re0 - rs0 + kHybChunk - 1) / kHybChunk);
    int last = 0;
    if (lane == 0) {
      part[c] = v;
      __threadfence();  // the partial is visible before the count
      last = atomicAdd(H.split_count + si, 1) == pieces - 1;
    }
    if (__shfl_sync(0xffffffffu, last, 0)) {
      __threadfence();
      Acc t = Acc(0);
      for (int k = lane; k < pieces; k += kWarp) t = add_rn(t, __ldcg(part + first + k));
      t = group_sum<kWarp>(t);
      if (lane == 0) {
        y[H.long_rows[li0]] = t;
        H.split_count[si] = 0;  // ready for the next launch
      }
    }
    return;
  }
  // Packed chunk: whole rows.
#pragma unroll
  for (int i = 0; i < PER; ++i) s_prod[wib][swz<Acc>(lane + i * kWarp)] = pr[i];
  __syncwarp();
  for (int li = my; li < li_end; li += kWarp) {
    if (li != my) {
      my_s = H.tail_ptr[li];
      my_e = H.tail_ptr[li + 1];
      my_row = H.long_rows[li];
    }
    const int a = static_cast<int>(my_s - e0);
    const int b = static_cast<int>(my_e - e0);
    Acc v = Acc(0);
    for (int q = a; q < b; ++q) v = add_rn(v, s_prod[wib][swz<Acc>(q)]);
    y[my_row] = v;
  }
}

// ---------------------------------------------------------------------------
// BCSR R x C: one thread per (block row, r). The R threads of a block row
// read its blocks' rows (C contiguous values, one or two 16-byte loads) and
// share the C-wide slice of x. Order per row: per-block partial over c, then
// added to the row total (spmv_bcsr_cpu order). VEC_X: x is 16-byte aligned
// so full slices are vector loads; the last partial block column is read
// element by element with the column bound the reference applies.
// ---------------------------------------------------------------------------
template <typename T, int C>
struct BlockRow;
template <>
struct BlockRow<double, 4> {
  __device__ static void load(const double* p, uint64_t pol, double (&v)[4]) {
    const double2 a = ld_stream2(p, pol), b = ld_stream2(p + 2, pol);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  }
  __device__ static void load_x(const double* p, uint64_t pol, double (&v)[4]) {
    const double2 a = ld_keep2(p, pol), b = ld_keep2(p + 2, pol);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  }
};
template <>
struct BlockRow<double, 2> {
  __device__ static void load(const double* p, uint64_t pol, double (&v)[2]) {
    const double2 a = ld_stream2(p, pol);
    v[0] = a.x; v[1] = a.y;
  }
  __device__ static void load_x(const double* p, uint64_t pol, double (&v)[2]) {
    const double2 a = ld_keep2(p, pol);
    v[0] = a.x; v[1] = a.y;
  }
};
template <>
struct BlockRow<float, 4> {
  __device__ static void load(const float* p, uint64_t pol, float (&v)[4]) {
    const float4 a = ld_stream4(p, pol);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  }
  __device__ static void load_x(const float* p, uint64_t pol, float (&v)[4]) {
    const float4 a = ld_keep4(p, pol);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  }
};
template <>
struct BlockRow<float, 2> {
  __device__ static void load(const float* p, uint64_t pol, float (&v)[2]) {
    const float2 a = ld_stream2(p, pol);
    v[0] = a.x; v[1] = a.y;
  }
  __device__ static void load_x(const float* p, uint64_t pol, float (&v)[2]) {
    const float2 a = ld_keep2(p, pol);
    v[0] = a.x; v[1] = a.y;
  }
};

template <typename T, typename Acc, int R, int C, bool VEC_X, int UB>
__global__ void __launch_bounds__(256)
    bcsr_rows(BcsrView B, const T* __restrict__ x, Acc* __restrict__ y) {
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t bi = gid / R;
  const int r = static_cast<int>(gid % R);
  if (bi >= B.mb) return;
  const T* __restrict__ vals = static_cast<const T*>(B.values);
  const uint64_t ps = policy_evict_first();
  const uint64_t pk = policy_evict_last();
  const int s = B.rowptr[bi];
  const int e = B.rowptr[bi + 1];
  Acc acc = Acc(0);
  // UB blocks per batch: all their indices, block rows and x slices are
  // requested before any product is formed.
  for (int bp0 = s; bp0 < e; bp0 += UB) {
    int bj[UB];
    T v[UB][C];
    T xv[UB][C];
#pragma unroll
    for (int u = 0; u < UB; ++u) bj[u] = (bp0 + u < e) ? ld_stream(B.colind + bp0 + u, ps) : 0;
#pragma unroll
    for (int u = 0; u < UB; ++u)
      if (bp0 + u < e) BlockRow<T, C>::load(vals + static_cast<int64_t>(bp0 + u) * (R * C) + r * C, ps, v[u]);
#pragma unroll
    for (int u = 0; u < UB; ++u) {
      const int gc0 = bj[u] * C;
      if (bp0 + u < e) {
        if (VEC_X && gc0 + C <= B.n) {
          BlockRow<T, C>::load_x(x + gc0, pk, xv[u]);
        } else {
#pragma unroll
          for (int c = 0; c < C; ++c) xv[u][c] = (gc0 + c < B.n) ? ld_keep(x + gc0 + c, pk) : T(0);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < UB; ++u) {
      if (bp0 + u < e) {
        const int gc0 = bj[u] * C;
        Acc part = Acc(0);
#pragma unroll
        for (int c = 0; c < C; ++c) {
          if (gc0 + c >= B.n) break;  // trailing partial block column
          part = add_rn(part, prod<Acc>(v[u][c], xv[u][c]));
        }
        acc = add_rn(acc, part);
      }
    }
  }
  const int64_t gi = bi * R + r;
  if (gi < B.m) y[gi] = acc;
}

// ---------------------------------------------------------------------------
// BCSR 4x4, fp64, on the tensor cores (an experiment; SPMVB_BCSR_MMA=1 selects
// it, bcsr_rows is the default). sm_100's fp64 tensor path is the warp-level
// mma.sync m8n8k4 (tcgen05 has no f64 kind). A warp owns block rows P = 2q
// and Q = 2q + 1 and walks their blocks pairwise: A (8 x 4) stacks the j-th
// block of P (rows 0-3) over the j-th block of Q (rows 4-7); B (4 x 8) holds
// P's x slice in column 0 and Q's in column 1 (zeros elsewhere); D
// accumulates over j, and D[0..3][0], D[4..7][1] are the two block rows' y -
// 8 useful outputs of the 64 each MMA computes, since every block meets its
// own x slice. The tensor core adds each block's four products in its own
// order, so y is within the gamma_n bound of spmv_bcsr_cpu, not bit-identical.
// Fragments (PTX m8n8k4 .f64): lane l holds A[l/4][l%4], B[l%4][l/4] and
// D[l/4][2*(l%4) + {0,1}].
// ---------------------------------------------------------------------------
__device__ __forceinline__ void dmma_8x8x4(double (&d)[2], double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
               : "+d"(d[0]), "+d"(d[1])
               : "d"(a), "d"(b));
}

// UB: block pairs whose fragments are loaded before their MMAs.
template <int UB>
__global__ void __launch_bounds__(256) bcsr4_dmma(BcsrView B, const double* __restrict__ x, double* __restrict__ y) {
  const double* __restrict__ vals = static_cast<const double*>(B.values);
  const uint64_t ps = policy_evict_first();
  const uint64_t pk = policy_evict_last();
  const int lane = threadIdx.x & (kWarp - 1);
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / kWarp;
  const int64_t P = warp * 2;
  if (P >= B.mb) return;
  const bool hasQ = P + 1 < B.mb;
  const int r = lane >> 2;  // A row / B column of this lane
  const int k = lane & 3;   // A column / B row of this lane
  const int sP = B.rowptr[P], eP = B.rowptr[P + 1];
  const int sQ = hasQ ? B.rowptr[P + 1] : 0, eQ = hasQ ? B.rowptr[P + 2] : 0;
  const int len = max(eP - sP, eQ - sQ);
  const bool mine_P = r < 4;
  double d[2] = {0.0, 0.0};
  for (int j0 = 0; j0 < len; j0 += UB) {
    double a[UB], b[UB];
#pragma unroll
    for (int u = 0; u < UB; ++u) {
      const int j = j0 + u;
      const int pP = sP + j, pQ = sQ + j;
      // A: this lane's element of the j-th block of P (rows 0-3) or Q (4-7).
      const int pa = mine_P ? pP : pQ;
      const bool va = mine_P ? (pP < eP) : (pQ < eQ);
      a[u] = va ? ld_stream(vals + static_cast<int64_t>(pa) * 16 + (r & 3) * 4 + k, ps) : 0.0;
      // B: column 0 = P's x slice, column 1 = Q's; lane holds B[k][r].
      double bv = 0.0;
      if (r == 0 && pP < eP) {
        const int gc = ld_stream(B.colind + pP, ps) * 4 + k;
        if (gc < B.n) bv = ld_keep(x + gc, pk);
      } else if (r == 1 && pQ < eQ) {
        const int gc = ld_stream(B.colind + pQ, ps) * 4 + k;
        if (gc < B.n) bv = ld_keep(x + gc, pk);
      }
      b[u] = bv;
    }
#pragma unroll
    for (int u = 0; u < UB; ++u) dmma_8x8x4(d, a[u], b[u]);
  }
  // D[r][0] for r < 4 (block row P) and D[r][1] for r >= 4 (block row Q)
  // sit in the lanes with k == 0.
  if (k == 0) {
    const int64_t gi = mine_P ? P * 4 + r : (P + 1) * 4 + (r - 4);
    if (gi < B.m && (mine_P || hasQ)) y[gi] = mine_P ? d[0] : d[1];
  }
}

}  // namespace spmvb
