#pragma once
// Host CSR matrix (same fields as SpMVBench's CsrMatrix<T>,
// include/spmvbench/csr.hpp:16-35). Columns inside a row may be unsorted.
#include <cstdint>
#include <string>
#include <vector>

#include "spmvbench/dtypes.hpp"

namespace spmvbench {

template <typename T>
struct CsrMatrix {
  using value_type = T;
  int m = 0;
  int n = 0;
  std::int64_t nnz = 0;
  std::vector<Index> rowptr;
  std::vector<Index> colind;
  std::vector<T> values;

  CsrMatrix() = default;
  CsrMatrix(int rows, int cols) : m(rows), n(cols), rowptr(rows + 1, 0) {}

  std::int64_t storage_bytes() const {
    return nnz * static_cast<std::int64_t>(sizeof(T) + sizeof(Index)) +
           static_cast<std::int64_t>(m + 1) * static_cast<std::int64_t>(sizeof(Index));
  }
};

struct MatrixInfo {
  std::string name;
  int m = 0;
  int n = 0;
  std::int64_t nnz = 0;
};

}  // namespace spmvbench
