#pragma once
// Row statistics (same fields and definitions as SpMVBench's RowStats,
// include/spmvbench/stats.hpp:14-52), computed by libspmvb
// (spmvb_compute_row_stats). dense_share_of_stored_4x4 is an addition.
#include <algorithm>
#include <cstdint>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "spmvb.h"
#include "spmvbench/csr.hpp"

namespace spmvbench {

struct RowStats {
  std::int64_t nnz = 0;
  int rows = 0;
  int cols = 0;
  double mean_row_nnz = 0.0;
  double median_row_nnz = 0.0;
  int min_row_nnz = 0;
  int max_row_nnz = 0;
  double stddev_row_nnz = 0.0;
  double cv_row_nnz = 0.0;
  double max_over_mean = 0.0;
  std::vector<std::int64_t> row_nnz_histogram;
  double ell_padding_overhead = 1.0;
  double frac_dense_blocks_4x4 = 0.0;
  double density = 0.0;
  double dense_share_of_stored_4x4 = 0.0;

  std::string to_string() const {
    std::ostringstream os;
    os << "rows=" << rows << " cols=" << cols << " nnz=" << nnz << " density=" << density << "\n";
    os << "row_nnz: mean=" << mean_row_nnz << " median=" << median_row_nnz << " min=" << min_row_nnz
       << " max=" << max_row_nnz << " stddev=" << stddev_row_nnz << " cv=" << cv_row_nnz
       << " max/mean=" << max_over_mean << "\n";
    os << "ell_padding_overhead=" << ell_padding_overhead << " frac_dense_blocks_4x4=" << frac_dense_blocks_4x4;
    return os.str();
  }
};

inline spmvb_row_stats to_c(const RowStats& s) {
  spmvb_row_stats c{};
  c.nnz = s.nnz;
  c.rows = s.rows;
  c.cols = s.cols;
  c.mean_row_nnz = s.mean_row_nnz;
  c.median_row_nnz = s.median_row_nnz;
  c.min_row_nnz = s.min_row_nnz;
  c.max_row_nnz = s.max_row_nnz;
  c.stddev_row_nnz = s.stddev_row_nnz;
  c.cv_row_nnz = s.cv_row_nnz;
  c.max_over_mean = s.max_over_mean;
  c.ell_padding_overhead = s.ell_padding_overhead;
  c.frac_dense_blocks_4x4 = s.frac_dense_blocks_4x4;
  c.density = s.density;
  c.dense_share_of_stored_4x4 = s.dense_share_of_stored_4x4;
  return c;
}

inline RowStats compute_row_stats(const Index* rowptr, const Index* colind, int m, int n, std::int64_t nnz) {
  spmvb_row_stats c{};
  int mx = 0;
  for (int i = 0; i < m; ++i) mx = std::max<int>(mx, rowptr[i + 1] - rowptr[i]);
  RowStats s;
  s.row_nnz_histogram.assign(static_cast<std::size_t>(mx) + 1, 0);
  if (spmvb_compute_row_stats(rowptr, colind, m, n, nnz, &c, s.row_nnz_histogram.data(),
                              static_cast<std::int64_t>(s.row_nnz_histogram.size())) != SPMVB_OK)
    throw std::runtime_error(std::string("compute_row_stats: ") + spmvb_last_error());
  s.nnz = c.nnz;
  s.rows = c.rows;
  s.cols = c.cols;
  s.mean_row_nnz = c.mean_row_nnz;
  s.median_row_nnz = c.median_row_nnz;
  s.min_row_nnz = c.min_row_nnz;
  s.max_row_nnz = c.max_row_nnz;
  s.stddev_row_nnz = c.stddev_row_nnz;
  s.cv_row_nnz = c.cv_row_nnz;
  s.max_over_mean = c.max_over_mean;
  s.ell_padding_overhead = c.ell_padding_overhead;
  s.frac_dense_blocks_4x4 = c.frac_dense_blocks_4x4;
  s.density = c.density;
  s.dense_share_of_stored_4x4 = c.dense_share_of_stored_4x4;
  return s;
}

template <typename T>
RowStats compute_row_stats(const CsrMatrix<T>& A) {
  return compute_row_stats(A.rowptr.data(), A.colind.data(), A.m, A.n, A.nnz);
}

}  // namespace spmvbench
