// Row statistics with the definitions of compute_row_stats
// (src/stats.cpp:13-123): population standard deviation accumulated in row
// order, median of the sorted lengths (mean of the two middle values for even
// m), histogram over 0..max, ELL padding m*max/nnz, and the fraction of all
// possible 4x4 blocks holding more than 8 stored entries (duplicates counted,
// as the reference counts them). The dense-block count sorts each block row's
// block columns instead of the reference's linear search (O(L log L) instead
// of O(L^2) per block row); the counts are identical. spmvb_matrix_row_stats
// takes the census from the device (one radix sort of block keys,
// convert.cu) and the rest from the handle's host rowptr, in the same order.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <vector>

#include "../internal.hpp"

using namespace spmvb;

namespace {

// Everything but the 4x4 block census, from rowptr: the reference's
// accumulation order (lengths in row order, variance summed in row order).
spmvb_status length_stats(const int32_t* h_rowptr, int32_t m, int32_t n, int64_t nnz, spmvb_row_stats* out,
                          int64_t* h_histogram, int64_t hist_cap) {
  spmvb_row_stats s{};
  s.nnz = nnz;
  s.rows = m;
  s.cols = n;
  s.density = (static_cast<double>(m) * n > 0) ? static_cast<double>(nnz) / (static_cast<double>(m) * n) : 0.0;
  s.ell_padding_overhead = 1.0;
  if (m <= 0) {
    if (h_histogram && hist_cap >= 1) h_histogram[0] = 0;
    *out = s;
    return SPMVB_OK;
  }
  std::vector<int> row_nnz(m);
  long long sum = 0;
  int mn = 0, mx = 0;
  for (int i = 0; i < m; ++i) {
    const int r = static_cast<int>(h_rowptr[i + 1] - h_rowptr[i]);
    row_nnz[i] = r;
    sum += r;
    if (i == 0 || r < mn) mn = r;
    if (i == 0 || r > mx) mx = r;
  }
  s.min_row_nnz = mn;
  s.max_row_nnz = mx;
  s.mean_row_nnz = static_cast<double>(sum) / m;
  {
    std::vector<int> sorted = row_nnz;
    std::sort(sorted.begin(), sorted.end());
    if (m % 2 == 1)
      s.median_row_nnz = sorted[m / 2];
    else
      s.median_row_nnz = 0.5 * static_cast<double>(static_cast<int64_t>(sorted[m / 2 - 1]) + sorted[m / 2]);
  }
  double var = 0.0;
  for (int i = 0; i < m; ++i) {
    const double d = row_nnz[i] - s.mean_row_nnz;
    var += d * d;
  }
  var /= m;
  s.stddev_row_nnz = std::sqrt(var);
  s.cv_row_nnz = (s.mean_row_nnz > 0) ? s.stddev_row_nnz / s.mean_row_nnz : 0.0;
  s.max_over_mean = (s.mean_row_nnz > 0) ? s.max_row_nnz / s.mean_row_nnz : 0.0;
  if (h_histogram) {
    if (hist_cap < static_cast<int64_t>(mx) + 1)
      return fail(SPMVB_ERR_INVALID_ARGUMENT, "histogram capacity below max_row_nnz+1");
    std::fill(h_histogram, h_histogram + mx + 1, 0);
    for (int i = 0; i < m; ++i) h_histogram[row_nnz[i]]++;
  }
  s.ell_padding_overhead = (nnz > 0) ? static_cast<double>(m) * mx / static_cast<double>(nnz) : 1.0;
  *out = s;
  return SPMVB_OK;
}

void census_fields(spmvb_row_stats* s, int32_t m, int32_t n, int64_t dense_blocks, int64_t stored_blocks) {
  const int64_t possible = static_cast<int64_t>((m + 3) / 4) * ((n + 3) / 4);
  s->frac_dense_blocks_4x4 = (possible > 0) ? static_cast<double>(dense_blocks) / possible : 0.0;
  s->dense_share_of_stored_4x4 =
      (stored_blocks > 0) ? static_cast<double>(dense_blocks) / static_cast<double>(stored_blocks) : 0.0;
}

}  // namespace

extern "C" spmvb_status spmvb_compute_row_stats(const int32_t* h_rowptr, const int32_t* h_colind,
                                        int32_t m, int32_t n, int64_t nnz,
                                        spmvb_row_stats* out, int64_t* h_histogram,
                                        int64_t hist_cap) {
  clear_error();
  if (!out) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null output");
  if (m < 0 || n < 0 || nnz < 0) return fail(SPMVB_ERR_INVALID_ARGUMENT, "negative size");
  if (m > 0 && !h_rowptr) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null rowptr");
  spmvb_row_stats s{};
  SPMVB_TRY(length_stats(h_rowptr, m, n, nnz, &s, h_histogram, hist_cap));
  if (m <= 0) {
    *out = s;
    return SPMVB_OK;
  }
  const int R = 4, C = 4;
  const int mb = (m + R - 1) / R;
  int64_t dense_blocks = 0, stored_blocks = 0;
  if (h_colind != nullptr && nnz > 0) {
    std::vector<int32_t> bcols;
    for (int bi = 0; bi < mb; ++bi) {
      bcols.clear();
      for (int r = 0; r < R; ++r) {
        const int i = bi * R + r;
        if (i >= m) break;
        for (int32_t p = h_rowptr[i]; p < h_rowptr[i + 1]; ++p) bcols.push_back(h_colind[p] / C);
      }
      std::sort(bcols.begin(), bcols.end());
      for (size_t a = 0; a < bcols.size();) {
        size_t b = a;
        while (b < bcols.size() && bcols[b] == bcols[a]) ++b;
        if (static_cast<int>(b - a) > (R * C) / 2) dense_blocks++;
        stored_blocks++;
        a = b;
      }
    }
  }
  census_fields(&s, m, n, dense_blocks, stored_blocks);
  *out = s;
  return SPMVB_OK;
}

extern "C" spmvb_status spmvb_matrix_row_stats(spmvb_matrix A, spmvb_row_stats* out, int64_t* h_histogram,
                                               int64_t hist_cap) {
  clear_error();
  if (!A || !out) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null argument");
  DeviceGuard g(A->device);
  spmvb_row_stats s{};
  SPMVB_TRY(length_stats(A->h_rowptr.data(), A->m, A->n, A->nnz, &s, h_histogram, hist_cap));
  if (A->m > 0) {
    int64_t dense_blocks = 0, stored_blocks = 0;
    SPMVB_TRY(block_census_device(A, &dense_blocks, &stored_blocks));
    census_fields(&s, A->m, A->n, dense_blocks, stored_blocks);
  }
  *out = s;
  return SPMVB_OK;
}
