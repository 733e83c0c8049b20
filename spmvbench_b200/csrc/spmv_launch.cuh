// Host launchers for the SpMV kernels of one (T, Acc) pair. Included by the
// three instantiation units spmv_f64f64.cu, spmv_f32f32.cu, spmv_f32f64.cu.
// Launch shapes replace SpmvRunner::run's switch (src/cuda/spmv_cuda.cu:385-464).
#pragma once

#include <algorithm>

#include <cstdlib>
#include <type_traits>

#include "ell_tma.cuh"
#include "internal.hpp"
#include "spmm_kernels.cuh"
#include "spmv_kernels.cuh"

namespace spmvb {

constexpr int kRowThreads = 256;
// Threads per CTA of ell_rows (see its launch): 64, or 32 for at most
// kEllSmallRows rows.
constexpr int kEllThreads = 64;
constexpr int kEllSmallRows = 160000;
// Threads per CTA of hyb_rows: 4 chunk warps per CTA instead of 8, so a
// CTA's slot frees as soon as fewer chunks are done: 32.7 against 33.9 us
// fp64 on the power-law matrix (bit-identical), fp32 unchanged.
constexpr int kHybThreads = 128;
// BCSR: blocks requested per batch per thread.
constexpr int kBcsrBatch = 2;
// BCSR: threads per CTA (64: 25.96 against 26.39 us with 256 on the 500k-row
// 4x4-block matrix; the L2-resident banded matrix is unchanged).
constexpr int kBcsrThreads = 64;
// Warp-staged scalar kernel: entries per warp chunk.
constexpr int kScalarWarpChunk = 512;

template <typename T, typename Acc, int G>
static void launch_vector(const CsrView& v, int sms, const T* x, Acc* y,
                          cudaStream_t s) {
  const int64_t rows_per_block = (kRowThreads / kWarp) * (kWarp / G);
  const int64_t need = (v.m + rows_per_block - 1) / rows_per_block;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(need, int64_t(sms) * 16)));
  csr_vector<T, Acc, G><<<grid, kRowThreads, 0, s>>>(v, x, y);
}

// SPMVB_BCSR_MMA=1: fp64 BCSR 4x4 on the tensor cores (bcsr4_dmma), an
// experiment measured against bcsr_rows.
static bool bcsr_mma_requested() {
  const char* e = std::getenv("SPMVB_BCSR_MMA");
  return e && *e == '1';
}

// ELL widths ell_tma serves (wider matrices run ell_rows).
constexpr int kEllTmaMaxWidth = 16;

// ell_tma with STAGES ring slots per warp on a persistent grid of as many
// CTAs as fit on every SM (shared memory bounds it: 4 warps x STAGES slots
// of 32 rows x width entries).
template <typename T, typename Acc, int WMAX, int STAGES>
static spmvb_status launch_ell_tma(spmvb_matrix A, const EllView& e, const T* x, Acc* y, cudaStream_t s) {
  auto kern = ell_tma<T, Acc, WMAX, STAGES>;
  constexpr int smem = kEllTmaWarps * STAGES * EllTmaStage<T, WMAX>::kBytes + 128;
  static int per_sm = [&] {
    int n = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kEllTmaWarps * 32, smem) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    return n;
  }();
  if (per_sm < 1) return fail(SPMVB_ERR_CUDA, "ell_tma cannot be resident on this device");
  const int64_t warps_needed = (static_cast<int64_t>(A->m) + 31) / 32;
  const int64_t ctas_needed = (warps_needed + kEllTmaWarps - 1) / kEllTmaWarps;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ctas_needed, int64_t(A->ctx->sm_count) * per_sm)));
  kern<<<grid, kEllTmaWarps * 32, smem, s>>>(A->ell_tm_col, A->ell_tm_val, e, x, y, A->ctx->err.as<int>());
  return SPMVB_OK;
}

template <typename T, typename Acc>
spmvb_status launch_spmv(spmvb_matrix A, spmvb_kernel kernel, int lanes,
                         int block, const T* x, Acc* y, cudaStream_t stream) {
  const CsrView v = A->csr_view();
  const int sms = A->ctx->sm_count;
  if (A->m == 0) return SPMVB_OK;
  switch (kernel) {
    case SPMVB_CSR_SCALAR: {
      const int64_t groups = (int64_t(A->m) + kWarp - 1) / kWarp;  // 32 rows per warp
      const int64_t need = (groups + 7) / 8;
      const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(need, int64_t(sms) * 16)));
      csr_scalar_warp<T, Acc, kScalarWarpChunk><<<grid, 256, 0, stream>>>(v, x, y);
      count_launch();
      break;
    }
    case SPMVB_CSR_VECTOR: {
      // Reference lane selection: 2/4/8/16, anything else -> 32
      // (src/cuda/spmv_cuda.cu:394-420).
      switch (lanes) {
        case 2: launch_vector<T, Acc, 2>(v, sms, x, y, stream); break;
        case 4: launch_vector<T, Acc, 4>(v, sms, x, y, stream); break;
        case 8: launch_vector<T, Acc, 8>(v, sms, x, y, stream); break;
        case 16: launch_vector<T, Acc, 16>(v, sms, x, y, stream); break;
        default: launch_vector<T, Acc, 32>(v, sms, x, y, stream); break;
      }
      count_launch();
      break;
    }
    case SPMVB_CSR_WARP:
      launch_vector<T, Acc, 32>(v, sms, x, y, stream);
      count_launch();
      break;
    case SPMVB_CSR_MERGE: {
      SPMVB_TRY(build_merge(A));
      MergeView mv;
      mv.tile_row = A->merge_tile_row.as<int>();
      mv.carry_row = A->merge_carry_row.as<int>();
      mv.carry_val = A->merge_carry_val.get();
      mv.num_items = static_cast<int64_t>(A->m) + A->nnz;
      mv.num_tiles = A->merge_tiles;
      mv.tile_items = kMergeTile;
      csr_merge<T, Acc, kMergeThreads, kMergeIpt>
          <<<mv.num_tiles, kMergeThreads, 0, stream>>>(v, mv, x, y);
      merge_fixup<Acc><<<(mv.num_tiles + 255) / 256, 256, 0, stream>>>(mv, y);
      count_launch(2);
      break;
    }
    case SPMVB_ELL: {
      SPMVB_TRY(build_ell(A));
      EllView e;
      e.colind = A->ell_colind.as<int>();
      e.values = A->ell_values.get();
      e.row_lengths = A->ell_rowlen.as<int>();
      e.m = A->m;
      e.n = A->n;
      e.width = A->ell_width;
      e.ld = A->m;
      SPMVB_TRY(build_ell_tma(A, kEllTmaMaxWidth));
      if (A->ell_tma_state == 1) {
        // The matrix stream through the TMA engine, the gathers alone on the
        // load path (ell_tma.cuh).
        const char* st = std::getenv("SPMVB_ELL_TMA_STAGES");
        const int stages = st ? std::atoi(st) : 4;
        if (stages == 2) SPMVB_TRY((launch_ell_tma<T, Acc, kEllTmaMaxWidth, 2>(A, e, x, y, stream)));
        else if (stages == 4) SPMVB_TRY((launch_ell_tma<T, Acc, kEllTmaMaxWidth, 4>(A, e, x, y, stream)));
        else SPMVB_TRY((launch_ell_tma<T, Acc, kEllTmaMaxWidth, 3>(A, e, x, y, stream)));
      } else {
        // Small CTAs: a row block that fills less than one wave (an 8-way
        // shard of 1M rows: 125k rows) spreads over the SMs within 2 % with
        // 64-thread CTAs instead of the 21 % that 256-thread CTAs leave
        // (11.4 against 12.6 us), and 32-thread CTAs gain 2 % more there
        // (11.0 against 11.2 us); from 250k rows on 64 is 1 % faster.
        const int threads = A->m <= kEllSmallRows ? 32 : kEllThreads;
        ell_rows<T, Acc, false><<<(A->m + threads - 1) / threads, threads, 0, stream>>>(e, x, y);
      }
      count_launch();
      break;
    }
    case SPMVB_HYB: {
      SPMVB_TRY(build_hyb(A, 0));
      HybView h;
      h.ell.colind = A->hyb_colind.as<int>();
      h.ell.values = A->hyb_values.get();
      h.ell.row_lengths = A->hyb_rowlen.as<int>();
      h.ell.m = A->m;
      h.ell.n = A->n;
      h.ell.width = A->hyb_K;
      h.ell.ld = A->m;
      h.long_rows = A->hyb_long_rows.as<int>();
      h.tail_ptr = A->hyb_tail_ptr.as<int64_t>();
      h.tail_colind = A->hyb_tail_colind.as<int>();
      h.tail_values = A->hyb_tail_values.get();
      h.chunk_start = A->hyb_chunk_start.as<int64_t>();
      h.chunk_row = A->hyb_chunk_row.as<int>();
      h.chunk_split = A->hyb_chunk_split.as<int>();
      h.split_rows = A->hyb_split_rows.as<int>();
      h.split_first = A->hyb_split_first.as<int>();
      h.split_count = A->hyb_split_count.as<int>();
      h.empty_rows = A->hyb_empty_rows.as<int>();
      h.partial = A->hyb_partial.get();
      h.tail_nnz = A->hyb_tail_nnz;
      h.n_long = A->hyb_n_long;
      h.n_chunks = A->hyb_n_chunks;
      h.n_split = A->hyb_n_split;
      h.n_empty = A->hyb_n_empty;
      h.ell_blocks = A->hyb_K > 0 ? (A->m + kHybThreads - 1) / kHybThreads : 0;
      h.chunk_blocks = (h.n_chunks + kHybThreads / kWarp - 1) / (kHybThreads / kWarp);
      const int empty_blocks = (h.n_empty + kHybThreads - 1) / kHybThreads;
      const int grid = h.ell_blocks + h.chunk_blocks + empty_blocks;
      if (grid > 0) {
        hyb_rows<T, Acc, kHybThreads><<<grid, kHybThreads, 0, stream>>>(h, x, y);
        count_launch();
      }
      break;
    }
    case SPMVB_BCSR: {
      // Reference: block <= 2 -> 2x2, else 4x4 (src/cuda/spmv_cuda.cu:449-457).
      const int bs = block <= 2 ? 2 : 4;
      SPMVB_TRY(build_bcsr(A, bs));
      const auto& b = bs == 2 ? A->bcsr2 : A->bcsr4;
      BcsrView bv;
      bv.rowptr = b.rowptr.as<int>();
      bv.colind = b.colind.as<int>();
      bv.values = b.values.get();
      bv.m = A->m;
      bv.n = A->n;
      bv.R = bs;
      bv.C = bs;
      bv.mb = b.mb;
      bv.block_nnz = b.block_nnz;
      const bool vec_x = (reinterpret_cast<uintptr_t>(x) % 16) == 0;
      const int64_t threads = int64_t(b.mb) * bs;
      const int grid = static_cast<int>(std::max<int64_t>(1, (threads + kBcsrThreads - 1) / kBcsrThreads));
      if (bs == 2) {
        if (vec_x) bcsr_rows<T, Acc, 2, 2, true, kBcsrBatch><<<grid, kBcsrThreads, 0, stream>>>(bv, x, y);
        else bcsr_rows<T, Acc, 2, 2, false, kBcsrBatch><<<grid, kBcsrThreads, 0, stream>>>(bv, x, y);
      } else if (std::is_same<T, double>::value && std::is_same<Acc, double>::value && bcsr_mma_requested()) {
        // Tensor-core experiment (bcsr4_dmma): a warp per pair of block rows.
        const int64_t warps = (int64_t(b.mb) + 1) / 2;
        const int g = static_cast<int>(std::max<int64_t>(1, (warps * kWarp + kRowThreads - 1) / kRowThreads));
        bcsr4_dmma<4><<<g, kRowThreads, 0, stream>>>(bv, reinterpret_cast<const double*>(x), reinterpret_cast<double*>(y));
      } else {
        if (vec_x) bcsr_rows<T, Acc, 4, 4, true, kBcsrBatch><<<grid, kBcsrThreads, 0, stream>>>(bv, x, y);
        else bcsr_rows<T, Acc, 4, 4, false, kBcsrBatch><<<grid, kBcsrThreads, 0, stream>>>(bv, x, y);
      }
      count_launch();
      break;
    }
    default:
      return fail(SPMVB_ERR_INVALID_ARGUMENT, "unknown SpMV kernel id " + std::to_string(int(kernel)));
  }
  SPMVB_TRY_CUDA(cudaGetLastError());
  return SPMVB_OK;
}

// ---- SpMM ------------------------------------------------------------------
template <typename T, typename Acc, int G, int W, bool VEC>
static void launch_spmm_rows(const CsrView& v, const int* rows, int nrows,
                             int sms, const T* X, Acc* Y, int k,
                             cudaStream_t s) {
  if (nrows <= 0) return;
  const int64_t rows_per_block = (kRowThreads / kWarp) * (kWarp / G);
  const int64_t need = (nrows + rows_per_block - 1) / rows_per_block;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(need, int64_t(sms) * 16)));
  spmm_rows<T, Acc, G, W, VEC><<<grid, kRowThreads, 0, s>>>(v, rows, nrows, X, Y, k);
  count_launch();
}

template <typename T, typename Acc, bool VEC>
static void launch_spmm_tile(const CsrView& v, int tile, const int* rows,
                             int nrows, int sms, const T* X, Acc* Y, int k,
                             cudaStream_t s) {
  constexpr int V = 16 / sizeof(T);
  if constexpr (VEC) {
    if (tile == 64) launch_spmm_rows<T, Acc, 64 / V, V, true>(v, rows, nrows, sms, X, Y, k, s);
    else if (tile == 16) launch_spmm_rows<T, Acc, 16 / V, V, true>(v, rows, nrows, sms, X, Y, k, s);
    else launch_spmm_rows<T, Acc, 32 / V, V, true>(v, rows, nrows, sms, X, Y, k, s);
  } else {
    if (tile == 64) launch_spmm_rows<T, Acc, 32, 2, false>(v, rows, nrows, sms, X, Y, k, s);
    else if (tile == 16) launch_spmm_rows<T, Acc, 16, 1, false>(v, rows, nrows, sms, X, Y, k, s);
    else launch_spmm_rows<T, Acc, 32, 1, false>(v, rows, nrows, sms, X, Y, k, s);
  }
}

// Column bands of the plain SpMM sweep: the handle's setting
// (spmvb_matrix_set_spmm_bands; 1 = one row-order pass), or with 0 (auto)
// a single pass.
static int spmm_band_count(spmvb_matrix A, int k, size_t es) {
  if (A->spmm_bands > 0) return A->spmm_bands;
  (void)k;
  (void)es;
  return 1;
}

// The plain SpMM swept in `bands` column bands (spmm_band): one launch per
// band, stream-ordered, each carrying Y over from the previous one.
template <typename T, typename Acc, int G, int W, bool VEC>
static void launch_spmm_bands(spmvb_matrix A, int bands, int sms, const T* X, Acc* Y, int k, cudaStream_t s) {
  const CsrView v = A->csr_view();
  const int64_t rows_per_block = (kRowThreads / kWarp) * (kWarp / G);
  const int64_t need = (A->m + rows_per_block - 1) / rows_per_block;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(need, int64_t(sms) * 16)));
  const int* split = A->band_split.as<int>();
  const int64_t m = A->m;
  for (int b = 0; b < bands; ++b) {
    const int* lo = b == 0 ? nullptr : split + (b - 1) * m;
    const int* hi = b == bands - 1 ? nullptr : split + b * m;
    spmm_band<T, Acc, G, W, VEC><<<grid, kRowThreads, 0, s>>>(v, lo, hi, b == 0, X, Y, k);
  }
  count_launch(bands);
}

template <typename T, typename Acc>
spmvb_status launch_spmm(spmvb_matrix A, int tile, int bucketed, int k,
                         const T* X, Acc* Y, cudaStream_t stream) {
  constexpr int V = 16 / sizeof(T);
  if (A->m == 0 || k == 0) return SPMVB_OK;
  const CsrView v = A->csr_view();
  const int sms = A->ctx->sm_count;
  // Reference tile selection: 16, 64, anything else -> 32 (src/cuda/spmm_cuda.cu:155-168).
  const int t = (tile == 16 || tile == 64) ? tile : 32;
  const bool vec = (k % V) == 0 && (reinterpret_cast<uintptr_t>(X) % 16) == 0;
  const int bands = (!bucketed && A->sorted_rows && vec && t == 64) ? spmm_band_count(A, k, sizeof(T)) : 1;
  if (bands > 1) {
    SPMVB_TRY(build_band_splits(A, bands));
    launch_spmm_bands<T, Acc, 64 / V, V, true>(A, bands, sms, X, Y, k, stream);
  } else if (!bucketed) {
    if (vec) launch_spmm_tile<T, Acc, true>(v, t, nullptr, A->m, sms, X, Y, k, stream);
    else launch_spmm_tile<T, Acc, false>(v, t, nullptr, A->m, sms, X, Y, k, stream);
  } else {
    SPMVB_TRY(build_buckets(A));
    const int* rows = A->bucket_rows.as<int>();
    const int n_sm = A->b_short + A->b_med;
    if (vec) launch_spmm_tile<T, Acc, true>(v, t, rows, n_sm, sms, X, Y, k, stream);
    else launch_spmm_tile<T, Acc, false>(v, t, rows, n_sm, sms, X, Y, k, stream);
    if (A->b_long > 0) {
      const int grid = std::min(A->b_long, sms * 8);
      if (vec)
        spmm_long_rows<T, Acc, V, true><<<grid, kRowThreads, 0, stream>>>(v, rows + n_sm, A->b_long, X, Y, k);
      else
        spmm_long_rows<T, Acc, 2, false><<<grid, kRowThreads, 0, stream>>>(v, rows + n_sm, A->b_long, X, Y, k);
      count_launch();
    }
  }
  SPMVB_TRY_CUDA(cudaGetLastError());
  return SPMVB_OK;
}

}  // namespace spmvb
