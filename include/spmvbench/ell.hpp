#pragma once
// ELL storage and csr_to_ell with the layout of SpMVBench's csr_to_ell
// (src/formats.cpp:14-43): width = longest row, column-major slot j*m + i,
// padding column 0 / value 0, row_lengths.
#include <algorithm>
#include <cstdint>
#include <vector>

#include "spmvbench/csr.hpp"

namespace spmvbench {

template <typename T>
struct EllMatrix {
  using value_type = T;
  int m = 0;
  int n = 0;
  int max_row_nnz = 0;
  std::int64_t nnz = 0;
  std::int64_t padded_nnz = 0;
  std::vector<Index> colind;
  std::vector<T> values;
  std::vector<int> row_lengths;

  double padding_overhead() const {
    return nnz == 0 ? 1.0 : static_cast<double>(padded_nnz) / static_cast<double>(nnz);
  }
};

template <typename T>
EllMatrix<T> csr_to_ell(const CsrMatrix<T>& A) {
  EllMatrix<T> E;
  E.m = A.m;
  E.n = A.n;
  E.nnz = A.nnz;
  int w = 0;
  for (int i = 0; i < A.m; ++i) w = std::max(w, static_cast<int>(A.rowptr[i + 1] - A.rowptr[i]));
  E.max_row_nnz = w;
  E.padded_nnz = static_cast<std::int64_t>(A.m) * w;
  E.colind.assign(static_cast<std::size_t>(E.padded_nnz), 0);
  E.values.assign(static_cast<std::size_t>(E.padded_nnz), T(0));
  E.row_lengths.resize(static_cast<std::size_t>(A.m));
  for (int i = 0; i < A.m; ++i) {
    const Index s = A.rowptr[i];
    const int len = static_cast<int>(A.rowptr[i + 1] - s);
    E.row_lengths[static_cast<std::size_t>(i)] = len;
    for (int j = 0; j < len; ++j) {
      const std::size_t slot = static_cast<std::size_t>(j) * A.m + i;
      E.colind[slot] = A.colind[s + j];
      E.values[slot] = A.values[s + j];
    }
  }
  return E;
}

}  // namespace spmvbench
