// Lazily built storage formats of a matrix handle.
//
//  ELL   - reference layout of csr_to_ell (src/formats.cpp:14-43): width =
//          longest row, column-major slots j*m + i, padding column 0 / value
//          0, row_lengths. Built on the device from the uploaded CSR.
//  HYB   - new: ELL(K) holding each row's first min(len, K) entries plus a
//          CSR tail with the rest of the rows longer than K. Built on device.
//  BCSR  - layout of csr_to_bcsr<T,R,C> (src/formats.cpp:45-105): blocks of a
//          block row in ascending block-column order, R*C row-major values,
//          zero fill, and for repeated (row, column) entries the last one in
//          CSR order wins. Built on the device by one stable radix sort of
//          the entries' (block, slot) keys (convert.cu) instead of the
//          reference's O(L^2) host search.
//  merge - merge-path tile start rows (device binary search) and the carry
//          scratch of the merge kernel.
//  buckets - SpMM row ids grouped by length (<= 8, <= 64, > 64), each group
//          ascending, built on the host from rowptr.
#include <algorithm>
#include <cstdlib>
#include <climits>
#include <cstring>
#include <numeric>
#include <string>
#include <vector>

#include <cudaTypedefs.h>

#include "internal.hpp"
#include "spmv_kernels.cuh"

namespace spmvb {

// ---- kernels ---------------------------------------------------------------
__global__ void merge_partition(CsrView A, int64_t num_items, int tile_items,
                                int num_tiles, int* __restrict__ tile_row) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t > num_tiles) return;
  const int64_t diag = min(static_cast<int64_t>(t) * tile_items, num_items);
  int64_t lo = diag - A.nnz > 0 ? diag - A.nnz : 0;
  int64_t hi = diag < A.m ? diag : static_cast<int64_t>(A.m);
  while (lo < hi) {
    const int64_t pivot = (lo + hi) >> 1;
    if (A.rowptr[pivot + 1] <= diag - pivot - 1)
      lo = pivot + 1;
    else
      hi = pivot;
  }
  tile_row[t] = static_cast<int>(lo);
}

__global__ void spmm_band_splits(CsrView A, int bands, int band_cols, int* __restrict__ split) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= A.m) return;
  const int s = A.rowptr[i], e = A.rowptr[i + 1];
  for (int b = 1; b < bands; ++b) {
    const int64_t bound = static_cast<int64_t>(b) * band_cols;
    int lo = s, hi = e;  // first p in [s, e) with colind[p] >= bound
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (A.colind[mid] < bound) lo = mid + 1; else hi = mid;
    }
    split[static_cast<int64_t>(b - 1) * A.m + i] = lo;
  }
}

// Copies each row's first min(len, cap) entries into column-major slots and
// records row lengths (len, or -1 when len > cap and long_marker is set).
template <typename W>
__global__ void ell_fill(const int* __restrict__ rowptr, const int* __restrict__ colind,
                         const W* __restrict__ vals, int m, int cap, bool long_marker,
                         int* __restrict__ ecol, W* __restrict__ eval,
                         int* __restrict__ rowlen) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= m) return;
  const int s = rowptr[r];
  const int len = rowptr[r + 1] - s;
  const bool is_long = long_marker && len > cap;
  const int take = is_long ? 0 : min(len, cap);  // long rows live whole in the CSR part
  rowlen[r] = is_long ? -1 : len;
  for (int j = 0; j < take; ++j) {
    const int64_t p = static_cast<int64_t>(j) * m + r;
    ecol[p] = colind[s + j];
    eval[p] = vals[s + j];
  }
}

// Copies each long row whole into the CSR part (one warp per row).
template <typename W>
__global__ void hyb_tail_fill(const int* __restrict__ rowptr, const int* __restrict__ colind,
                              const W* __restrict__ vals, const int* __restrict__ long_rows,
                              const int64_t* __restrict__ tail_ptr, int n_long,
                              int* __restrict__ tcol, W* __restrict__ tval) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (w >= n_long) return;
  const int r = long_rows[w];
  const int s = rowptr[r];
  const int e = rowptr[r + 1];
  const int64_t o = tail_ptr[w];
  for (int p = s + lane; p < e; p += 32) {
    tcol[o + (p - s)] = colind[p];
    tval[o + (p - s)] = vals[p];
  }
}

namespace {

template <typename W>
void launch_ell_fill(spmvb_matrix A, int cap, bool marker, int* ecol, void* eval, int* rowlen) {
  ell_fill<W><<<(A->m + 255) / 256, 256>>>(A->rowptr.as<int>(), A->colind.as<int>(),
                                           A->values.as<W>(), A->m, cap, marker, ecol,
                                           static_cast<W*>(eval), rowlen);
  count_launch();
}

spmvb_status check_fits(spmvb_matrix A, double bytes, const char* what) {
  size_t free_b = 0, total_b = 0;
  SPMVB_TRY_CUDA(cudaMemGetInfo(&free_b, &total_b));
  if (bytes > 0.85 * static_cast<double>(free_b)) {
    char msg[256];
    std::snprintf(msg, sizeof(msg),
                  "%s needs %.3g GB of device memory but only %.3g GB are free "
                  "(m=%d, longest row %d); use the hybrid ELL+CSR format",
                  what, bytes / 1e9, free_b / 1e9, A->m, A->max_row);
    return fail(SPMVB_ERR_UNSUPPORTED, msg);
  }
  return SPMVB_OK;
}

}  // namespace

spmvb_status build_ell(spmvb_matrix A) {
  std::lock_guard<std::mutex> lk(A->build_mu);
  if (A->ell_built) return SPMVB_OK;
  DeviceGuard g(A->device);
  const size_t es = dtype_size(A->dtype);
  const int64_t slots = static_cast<int64_t>(A->m) * A->max_row;
  SPMVB_TRY(check_fits(A, static_cast<double>(slots) * (4 + es) + 4.0 * A->m, "ELL"));
  SPMVB_TRY(A->ell_colind.alloc(std::max<int64_t>(slots, 1) * 4));
  SPMVB_TRY(A->ell_values.alloc(std::max<int64_t>(slots, 1) * es));
  SPMVB_TRY(A->ell_rowlen.alloc(std::max<int64_t>(A->m, 1) * 4));
  if (A->m > 0) {
    if (es == 8)
      launch_ell_fill<unsigned long long>(A, A->max_row, false, A->ell_colind.as<int>(), A->ell_values.get(), A->ell_rowlen.as<int>());
    else
      launch_ell_fill<unsigned int>(A, A->max_row, false, A->ell_colind.as<int>(), A->ell_values.get(), A->ell_rowlen.as<int>());
    SPMVB_TRY_CUDA(cudaGetLastError());
    SPMVB_TRY_CUDA(cudaStreamSynchronize(0));
  }
  A->ell_width = A->max_row;
  A->ell_built = true;
  return SPMVB_OK;
}

// Automatic K: the smallest width that leaves at most m/64 rows in the tail,
// capped so the ELL part holds at most 4x the matrix's nonzeros.
// Width of the ELL part. Heavy-tailed rows (longest > 32 x mean): K = 0,
// every non-empty row goes to the chunked CSR part, which is balanced
// whatever the lengths, while one thread per row would idle most lanes.
// Otherwise K = the smallest power of two at least the mean row length.
static int choose_hyb_width(int m, int64_t nnz, int max_row) {
  if (m == 0 || max_row == 0) return 1;
  const double mean = static_cast<double>(nnz) / m;
  if (max_row > 32.0 * mean) return 0;
  int K = 1;
  while (K < mean && K < max_row) K <<= 1;
  return std::min(K, max_row);
}

spmvb_status build_hyb(spmvb_matrix A, int forced_k) {
  std::lock_guard<std::mutex> lk(A->build_mu);
  if (A->hyb_built && (forced_k == 0 || (forced_k > 0 && forced_k == A->hyb_K) || (forced_k < 0 && A->hyb_K == 0)))
    return SPMVB_OK;
  DeviceGuard g(A->device);
  const size_t es = dtype_size(A->dtype);
  const int K = forced_k > 0   ? std::min(forced_k, std::max(A->max_row, 1))
                : forced_k < 0 ? 0
                               : choose_hyb_width(A->m, A->nnz, A->max_row);
  std::vector<int32_t> long_rows, empty_rows;
  std::vector<int64_t> tail_ptr(1, 0);
  int64_t ell_nnz = 0;
  for (int i = 0; i < A->m; ++i) {
    const int len = A->h_rowptr[i + 1] - A->h_rowptr[i];
    if (len > K) {
      long_rows.push_back(i);
      tail_ptr.push_back(tail_ptr.back() + len);
    } else {
      ell_nnz += len;
      if (K == 0) empty_rows.push_back(i);
    }
  }
  const int n_long = static_cast<int>(long_rows.size());
  const int64_t slots = static_cast<int64_t>(A->m) * K;
  const int64_t tail = tail_ptr.back();
  // Chunks of the CSR part: whole rows packed greedily up to kHybChunk
  // entries; a row longer than that cut into kHybChunk-entry segments.
  std::vector<int64_t> chunk_start;
  std::vector<int32_t> chunk_row, chunk_split, split_rows, split_first;
  for (int li = 0; li < n_long;) {
    const int64_t len = tail_ptr[li + 1] - tail_ptr[li];
    if (len > kHybChunk) {
      split_rows.push_back(li);
      split_first.push_back(static_cast<int32_t>(chunk_start.size()));
      for (int64_t o = 0; o < len; o += kHybChunk) {
        chunk_start.push_back(tail_ptr[li] + o);
        chunk_row.push_back(li);
        chunk_split.push_back(static_cast<int32_t>(split_rows.size()) - 1);
      }
      ++li;
      continue;
    }
    chunk_start.push_back(tail_ptr[li]);
    chunk_row.push_back(li);
    chunk_split.push_back(-1);
    const int64_t start = tail_ptr[li];
    while (li < n_long && tail_ptr[li + 1] - tail_ptr[li] <= kHybChunk && tail_ptr[li + 1] - start <= kHybChunk) ++li;
  }
  if (chunk_start.size() > static_cast<size_t>(INT32_MAX / 2)) return fail(SPMVB_ERR_UNSUPPORTED, "HYB: too many chunks");
  const int n_chunks = static_cast<int>(chunk_start.size());
  chunk_start.push_back(tail);
  chunk_row.push_back(n_long);

  SPMVB_TRY(check_fits(A, static_cast<double>(slots + tail) * (4 + es) + 8.0 * A->m, "HYB"));
  SPMVB_TRY(A->hyb_colind.alloc(std::max<int64_t>(slots, 1) * 4));
  SPMVB_TRY(A->hyb_values.alloc(std::max<int64_t>(slots, 1) * es));
  SPMVB_TRY(A->hyb_rowlen.alloc(std::max<int64_t>(A->m, 1) * 4));
  SPMVB_TRY(upload(A->hyb_long_rows, long_rows.data(), long_rows.size() * 4, std::max<size_t>(long_rows.size(), 1) * 4));
  SPMVB_TRY(upload(A->hyb_tail_ptr, tail_ptr.data(), tail_ptr.size() * 8, tail_ptr.size() * 8));
  SPMVB_TRY(A->hyb_tail_colind.alloc((tail + kPad) * 4));
  SPMVB_TRY(A->hyb_tail_values.alloc((tail + kPad) * es));
  SPMVB_TRY(upload(A->hyb_chunk_start, chunk_start.data(), chunk_start.size() * 8, chunk_start.size() * 8));
  SPMVB_TRY(upload(A->hyb_chunk_row, chunk_row.data(), chunk_row.size() * 4, chunk_row.size() * 4));
  SPMVB_TRY(upload(A->hyb_chunk_split, chunk_split.data(), chunk_split.size() * 4, std::max<size_t>(chunk_split.size(), 1) * 4));
  SPMVB_TRY(upload(A->hyb_split_rows, split_rows.data(), split_rows.size() * 4, std::max<size_t>(split_rows.size(), 1) * 4));
  SPMVB_TRY(upload(A->hyb_split_first, split_first.data(), split_first.size() * 4, std::max<size_t>(split_first.size(), 1) * 4));
  SPMVB_TRY(A->hyb_split_count.alloc(std::max<size_t>(split_rows.size(), 1) * 4));  // zero-filled
  SPMVB_TRY(upload(A->hyb_empty_rows, empty_rows.data(), empty_rows.size() * 4, std::max<size_t>(empty_rows.size(), 1) * 4));
  SPMVB_TRY(A->hyb_partial.alloc(std::max<size_t>(n_chunks, 1) * 8));
  if (A->m > 0) {
    if (K > 0) {
      if (es == 8)
        launch_ell_fill<unsigned long long>(A, K, true, A->hyb_colind.as<int>(), A->hyb_values.get(), A->hyb_rowlen.as<int>());
      else
        launch_ell_fill<unsigned int>(A, K, true, A->hyb_colind.as<int>(), A->hyb_values.get(), A->hyb_rowlen.as<int>());
    }
    if (n_long > 0) {
      const int grid = (n_long + 7) / 8;
      if (es == 8)
        hyb_tail_fill<unsigned long long><<<grid, 256>>>(A->rowptr.as<int>(), A->colind.as<int>(), A->values.as<unsigned long long>(),
                                                         A->hyb_long_rows.as<int>(), A->hyb_tail_ptr.as<int64_t>(), n_long,
                                                         A->hyb_tail_colind.as<int>(), A->hyb_tail_values.as<unsigned long long>());
      else
        hyb_tail_fill<unsigned int><<<grid, 256>>>(A->rowptr.as<int>(), A->colind.as<int>(), A->values.as<unsigned int>(),
                                                   A->hyb_long_rows.as<int>(), A->hyb_tail_ptr.as<int64_t>(), n_long,
                                                   A->hyb_tail_colind.as<int>(), A->hyb_tail_values.as<unsigned int>());
      count_launch();
    }
    SPMVB_TRY_CUDA(cudaGetLastError());
    SPMVB_TRY_CUDA(cudaStreamSynchronize(0));
  }
  A->hyb_K = K;
  A->hyb_ell_nnz = ell_nnz;
  A->hyb_tail_nnz = tail;
  A->hyb_n_long = n_long;
  A->hyb_n_chunks = n_chunks;
  A->hyb_n_split = static_cast<int>(split_rows.size());
  A->hyb_n_empty = static_cast<int>(empty_rows.size());
  A->hyb_built = true;
  return SPMVB_OK;
}

spmvb_status build_bcsr(spmvb_matrix A, int block) {
  std::lock_guard<std::mutex> lk(A->build_mu);
  auto& B = block == 2 ? A->bcsr2 : A->bcsr4;
  if (B.built) return SPMVB_OK;
  DeviceGuard g(A->device);
  // Worst case every entry is its own block; the sort needs keys, entry
  // indices, block numbers and their double buffers beside it.
  const size_t es = dtype_size(A->dtype);
  const double rc = static_cast<double>(block) * block;
  SPMVB_TRY(check_fits(A, static_cast<double>(A->nnz) * (rc * es + 4 + 40) + 4.0 * A->m, "BCSR"));
  SPMVB_TRY(convert_bcsr_device(A, block));
  B.built = true;
  return SPMVB_OK;
}

namespace {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      p = nullptr;
    }
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// 2-D view {m rows (contiguous), width slots} of a column-major ELL array,
// boxes of 32 rows x width slots.
bool encode_ell_map(CUtensorMap* tm, CUtensorMapDataType type, size_t elem, void* base, int m, int width) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(m), static_cast<cuuint64_t>(width)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(m) * elem};
  const cuuint32_t box[2] = {32u, static_cast<cuuint32_t>(width)};
  const cuuint32_t estr[2] = {1u, 1u};
  return enc(tm, type, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

spmvb_status build_ell_tma(spmvb_matrix A, int max_width) {
  std::lock_guard<std::mutex> lk(A->build_mu);
  if (A->ell_tma_state != 0) return SPMVB_OK;
  // ell_rows (plain loads) is the default: on B200 it measured faster than
  // ell_tma on the uniform 1M-row matrix (68.7 us against 71.0 us with a
  // 4-slot ring, 112 us with 2 or 3). SPMVB_ELL_STREAM=tma selects ell_tma.
  const char* e = std::getenv("SPMVB_ELL_STREAM");
  const bool off = !(e && std::strcmp(e, "tma") == 0);
  const size_t es = dtype_size(A->dtype);
  if (off || !A->ell_built || A->ell_width < 1 || A->ell_width > max_width || A->m % 4 != 0 || A->m < 32) {
    A->ell_tma_state = -1;
    return SPMVB_OK;
  }
  const bool ok =
      encode_ell_map(&A->ell_tm_col, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, A->ell_colind.get(), A->m, A->ell_width) &&
      encode_ell_map(&A->ell_tm_val, es == 8 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT64 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, es,
                     A->ell_values.get(), A->m, A->ell_width);
  A->ell_tma_state = ok ? 1 : -1;
  return SPMVB_OK;
}

spmvb_status build_band_splits(spmvb_matrix A, int bands) {
  std::lock_guard<std::mutex> lk(A->build_mu);
  if (A->band_count == bands) return SPMVB_OK;
  DeviceGuard g(A->device);
  A->band_count = 0;
  A->band_split.reset();
  if (bands > 1) {
    SPMVB_TRY(A->band_split.alloc(static_cast<size_t>(bands - 1) * std::max(A->m, 1) * 4));
    const int band_cols = (A->n + bands - 1) / bands;
    spmm_band_splits<<<(A->m + 255) / 256, 256>>>(A->csr_view(), bands, band_cols, A->band_split.as<int>());
    count_launch();
    SPMVB_TRY_CUDA(cudaGetLastError());
    SPMVB_TRY_CUDA(cudaStreamSynchronize(0));
  }
  A->band_count = bands;
  return SPMVB_OK;
}

spmvb_status build_merge(spmvb_matrix A) {
  std::lock_guard<std::mutex> lk(A->build_mu);
  if (A->merge_built) return SPMVB_OK;
  DeviceGuard g(A->device);
  const int64_t items = static_cast<int64_t>(A->m) + A->nnz;
  const int64_t tiles = (items + kMergeTile - 1) / kMergeTile;
  if (tiles > INT32_MAX - 1) return fail(SPMVB_ERR_UNSUPPORTED, "too many merge tiles");
  A->merge_tiles = static_cast<int>(tiles);
  SPMVB_TRY(A->merge_tile_row.alloc((tiles + 1) * 4));
  SPMVB_TRY(A->merge_carry_row.alloc(std::max<int64_t>(tiles, 1) * 4));
  SPMVB_TRY(A->merge_carry_val.alloc(std::max<int64_t>(tiles, 1) * 8));
  if (tiles > 0) {
    merge_partition<<<static_cast<int>((tiles + 1 + 255) / 256), 256>>>(
        A->csr_view(), items, kMergeTile, static_cast<int>(tiles), A->merge_tile_row.as<int>());
    count_launch();
    SPMVB_TRY_CUDA(cudaGetLastError());
    SPMVB_TRY_CUDA(cudaStreamSynchronize(0));
  }
  A->merge_built = true;
  return SPMVB_OK;
}

spmvb_status build_buckets(spmvb_matrix A) {
  std::lock_guard<std::mutex> lk(A->build_mu);
  if (A->buckets_built) return SPMVB_OK;
  DeviceGuard g(A->device);
  std::vector<int32_t> s, md, l;
  for (int i = 0; i < A->m; ++i) {
    const int len = A->h_rowptr[i + 1] - A->h_rowptr[i];
    if (len <= 8) s.push_back(i);
    else if (len <= 64) md.push_back(i);
    else l.push_back(i);
  }
  std::vector<int32_t> rows;
  rows.reserve(A->m);
  rows.insert(rows.end(), s.begin(), s.end());
  rows.insert(rows.end(), md.begin(), md.end());
  rows.insert(rows.end(), l.begin(), l.end());
  SPMVB_TRY(upload(A->bucket_rows, rows.data(), rows.size() * 4, std::max<size_t>(rows.size(), 1) * 4));
  A->b_short = static_cast<int>(s.size());
  A->b_med = static_cast<int>(md.size());
  A->b_long = static_cast<int>(l.size());
  A->buckets_built = true;
  return SPMVB_OK;
}

}  // namespace spmvb
